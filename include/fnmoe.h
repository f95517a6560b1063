/*
 * fnmoe.h -- C ABI of the B200 (sm_100a) Flash-Next sparse-MoE decode path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void*` (NULL = legacy default stream).  Nothing here allocates
 * device memory: scratch comes from a caller-provided workspace whose size
 * the matching *_workspace_size call reports -- except
 * fnmoe_moe_execute_static, whose scratch is a fixed array inside the
 * library, and fnmoe_ep_create, which allocates an expert-parallel exchange
 * window once at set-up.  A workspace may start at any address: the library rounds its
 * start up to a 256-byte boundary, and the reported sizes include the 256
 * bytes that rounding can skip.  Each call returns FNMOE_OK (0) or a negative
 * FNMOE_ERR_* code; fnmoe_get_last_error() returns the message of the
 * calling thread's last failure.
 *
 * Reference interfaces replaced (paths inside 1architect/macqwen-releases):
 *   fnmoe_available / fnmoe_get_last_error
 *       flashnext_native_available / flashnext_native_get_last_error
 *       (models/flashnext/tests/bench/metal_runtime_native.mm:196-209)
 *   FnMoEArgs + fnmoe_moe_execute
 *       FlashNextMoEArgs + flashnext_native_moe_execute
 *       (metal_runtime_native.mm:175-194, :258-396) and the op-level
 *       MetalMoEExecutor.execute (models/flashnext/metal_runtime.py:764-932)
 *   fnmoe_weighted_combine   weighted_combine (metal_runtime.py:145-191)
 *   fnmoe_router_topk        adaptive_topk._moe_call router chain
 *       (models/flashnext/adaptive_topk.py:53-64,256-261; compiled.py:61-71)
 *   fnmoe_group_tokens       _gather_sort grouping for ragged batches
 *       (models/flashnext/expert_cache.py:1790-1810)
 *   fnmoe_moe_layer          the patched sparse-MoE block
 *       (adaptive_topk.py:53-292 with StreamingSwitchGLU, expert_cache.py:1584-1810)
 *   fnmoe_dequantize         mx.dequantize affine Q4 (metal_runtime.py:751-758)
 *   fnmoe_swiglu             fused up-SwiGLU bfloat16 epilogue (metal_runtime.py:262-285)
 *   fnmoe_paged_decode       paged_attention decode (models/qwen27b/paged_kv.py:417-495)
 *   fnmoe_tile_experts       no direct counterpart: the B200 analogue of packing
 *       expert records once for fast reads (models/flashnext/slab_pack.py:96-153),
 *       into a tile-major HBM layout the decode kernels stream with bulk copies
 */
#ifndef FNMOE_H
#define FNMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FNMOE_API __attribute__((visibility("default")))
#else
#define FNMOE_API
#endif

#define FNMOE_ABI_VERSION 4u

/* A route value marking an empty slot (skipped without an error). */
#define FNMOE_ROUTE_NONE 0xFFFFFFFFu

/* Size of the library-owned scratch used by fnmoe_moe_execute_static. */
#define FNMOE_STATIC_SCRATCH_BYTES (16ull << 20)

/* Status codes (negative = failure), mirroring the native bridge's
 * "0 ok / negative specific failure" convention. */
#define FNMOE_OK 0
#define FNMOE_ERR_NULL (-1)        /* a required pointer is NULL            */
#define FNMOE_ERR_SHAPE (-2)       /* a size is zero, misaligned or too big */
#define FNMOE_ERR_UNSUPPORTED (-3) /* dtype / group size / layout           */
#define FNMOE_ERR_DEVICE (-4)      /* no usable sm_100 device               */
#define FNMOE_ERR_WORKSPACE (-5)   /* workspace missing or too small        */
#define FNMOE_ERR_LAUNCH (-6)      /* CUDA launch or runtime error          */
#define FNMOE_ERR_ABI (-7)         /* abi_version mismatch                  */
#define FNMOE_ERR_VALUE (-8)       /* argument value out of range           */

/* Element types. */
#define FNMOE_DTYPE_BF16 0u
#define FNMOE_DTYPE_F32 1u

/* FnMoEArgs.flags */
#define FNMOE_FLAG_RETURN_ALL 0x1u   /* write gate/up/down per slot, no combine */
#define FNMOE_FLAG_NO_COMBINE 0x2u   /* scores absent: write per-slot down only */

/* Part order inside an expert record (slab_pack.py:96-153). */
#define FNMOE_PART_GATE_W 0
#define FNMOE_PART_GATE_S 1
#define FNMOE_PART_GATE_B 2
#define FNMOE_PART_UP_W 3
#define FNMOE_PART_UP_S 4
#define FNMOE_PART_UP_B 5
#define FNMOE_PART_DOWN_W 6
#define FNMOE_PART_DOWN_S 7
#define FNMOE_PART_DOWN_B 8

/* HBM-resident expert table: a header followed by fixed-stride expert
 * records, each holding the nine tensors at `part_offset`.  A route with bit
 * 31 set addresses record (route & 0x7FFFFFFF) (expert_pool.py:38,
 * metal_runtime.py:198-228). */
typedef struct FnExpertTable {
  const void *base;
  uint64_t header_bytes;
  uint64_t record_stride;
  uint64_t part_offset[9];
  uint32_t records;
  uint32_t reserved;
} FnExpertTable;

/* One MoE executor call: gate -> up -> SwiGLU -> down -> combine.
 * The first 19 fields follow FlashNextMoEArgs' order. */
/* Tiled expert tables: the routed experts' projections (and optionally the
 * shared expert's, as the last record) repacked once by fnmoe_tile_experts
 * into one 2560-byte chunk per (row group, 128-byte block) in MMA fragment
 * order, scales and biases included.  Record r of gate_up holds expert r's
 * gate and up rows (inter/8 groups of 8 + 8 rows), record r of down its down
 * rows (hidden/16 groups of 16).  Sizes: fnmoe_tiled_record_bytes. */
typedef struct FnTiledExperts {
  const void *gate_up;         /* [records][gate_up_record_bytes], 16-byte aligned, or NULL */
  const void *down;            /* [records][down_record_bytes], 16-byte aligned */
  uint64_t gate_up_record_bytes;
  uint64_t down_record_bytes;
  uint32_t records;            /* expert_count, +1 when the shared expert is the last record */
  uint32_t has_shared;         /* 1: the last record is the shared expert */
} FnTiledExperts;

typedef struct FnMoEArgs {
  uint32_t abi_version;        /* FNMOE_ABI_VERSION */
  uint32_t flags;              /* FNMOE_FLAG_* */
  const void *x;               /* [tokens, hidden]  (x_dtype) */
  const uint32_t *gate_weight; /* [experts, inter, hidden/8] packed Q4 */
  const void *gate_scales;     /* [experts, inter, hidden/group] bf16 */
  const void *gate_biases;
  const uint32_t *up_weight;
  const void *up_scales;
  const void *up_biases;
  const uint32_t *down_weight; /* [experts, hidden, inter/8] */
  const void *down_scales;     /* [experts, hidden, inter/group] bf16 */
  const void *down_biases;
  const uint32_t *routes;      /* [tokens, slots]; bit 31 = table record;
                                  FNMOE_ROUTE_NONE = empty slot (no expert runs,
                                  its per-slot output is left untouched) */
  const void *scores;          /* [tokens, slots] (scores_dtype) or NULL */
  void *output;                /* [tokens, hidden] bf16 (combined) */
  uint32_t tokens;
  uint32_t slots;
  uint32_t hidden_size;
  uint32_t inter_size;
  uint32_t expert_count;       /* experts in the *_weight arrays */
  /* extensions */
  uint32_t group_size;         /* 32 or 64 */
  uint32_t x_dtype;            /* FNMOE_DTYPE_BF16, or FNMOE_DTYPE_F32: float32
                                  activations (metal_runtime.py:371-373) -- then
                                  output, gate_out/up_out/down_out, shared_y,
                                  shared and shared_gate are float32 too, and
                                  every intermediate is rounded to float32 instead
                                  of bfloat16 (the reference's kernels with
                                  T = float) */
  uint32_t scores_dtype;       /* FNMOE_DTYPE_F32 or FNMOE_DTYPE_BF16 */
  uint32_t reserved0;
  const void *shared_y;        /* [tokens, hidden] bf16 or NULL */
  const void *shared;          /* [tokens, hidden] bf16 or NULL (with shared_gate) */
  const void *shared_gate;     /* [tokens] bf16 or NULL */
  FnExpertTable table;         /* base NULL = no table */
  /* Optional records for routes WITHOUT bit 31 (the reference's stream pack,
   * metal_runtime.py:202-207): when base != NULL such a route r addresses
   * record r of this table instead of the *_weight arrays. */
  FnExpertTable stream_table;
  void *gate_out;              /* RETURN_ALL: [tokens, slots, inter] bf16 */
  void *up_out;                /* RETURN_ALL: [tokens, slots, inter] bf16 */
  void *down_out;              /* RETURN_ALL / NO_COMBINE: [tokens, slots, hidden] bf16 */
  void *workspace;
  uint64_t workspace_bytes;
  /* When tiled.gate_up != NULL, routes without bit 31 address records of these
   * tiled tables (fnmoe_tile_experts) instead of the *_weight arrays. */
  FnTiledExperts tiled;
} FnMoEArgs;



/* A whole sparse-MoE block: router -> top-k -> renorm -> routed experts +
 * sigmoid-gated shared expert -> combine. */
typedef struct FnMoELayerArgs {
  uint32_t abi_version;
  uint32_t top_k;
  const void *x;               /* [tokens, hidden] bf16 */
  const void *router_weight;   /* [experts, hidden] bf16 */
  float renorm_blend;          /* 1.0 = shipped renorm */
  uint32_t tokens;
  uint32_t hidden_size;
  uint32_t inter_size;         /* routed expert intermediate */
  uint32_t expert_count;
  uint32_t group_size;
  uint32_t shared_inter_size;  /* 0 = no shared expert */
  const uint32_t *gate_weight; const void *gate_scales; const void *gate_biases;
  const uint32_t *up_weight; const void *up_scales; const void *up_biases;
  const uint32_t *down_weight; const void *down_scales; const void *down_biases;
  const uint32_t *shared_gate_weight; const void *shared_gate_scales; const void *shared_gate_biases;
  const uint32_t *shared_up_weight; const void *shared_up_scales; const void *shared_up_biases;
  const uint32_t *shared_down_weight; const void *shared_down_scales; const void *shared_down_biases;
  const void *shared_expert_gate; /* [hidden] bf16 (w_g of sigmoid(x.w_g)) */
  FnExpertTable table;         /* when base != NULL, experts come from the table */
  const uint32_t *table_routes_of_expert; /* [expert_count] route per expert, or NULL */
  void *output;                /* [tokens, hidden] bf16 */
  void *logits_out;            /* optional [tokens, experts] bf16 */
  uint32_t *inds_out;          /* optional [tokens, top_k] */
  void *scores_out;            /* optional [tokens, top_k] bf16 (renormalised) */
  void *workspace;
  uint64_t workspace_bytes;
  /* When tiled.gate_up != NULL the routed (and, with has_shared, the shared)
   * expert projections come from these tables; the *_weight arrays and
   * `table` are then ignored / must be NULL respectively. */
  FnTiledExperts tiled;
  uint32_t flags;              /* FNMOE_LAYER_* */
  uint32_t reserved1;
  /* Adaptive keep (adaptive_topk.py:43-50,75-261): with 0 < keep_threshold < 1
   * each token keeps its first max(min_keep, n) top-k slots, n the first
   * position whose cumulative share of the top-k mass (IEEE double, as the
   * reference's Python floats) reaches the threshold; dropped slots report
   * slot 0's expert with score 0, run no expert, and the renorm uses the kept
   * mass.  0 (or >= 1) keeps every slot. */
  double keep_threshold;
  uint32_t min_keep;           /* 0 or 1: at least one slot */
  uint32_t reserved2;
} FnMoELayerArgs;

/* FnMoELayerArgs.flags: by default a layer with tiled tables (group size 32,
 * hidden and inter multiples of 256) and at least FNMOE_PREFILL_PAIRS
 * (token, slot) pairs runs its experts as tcgen05 GEMMs on dequantised bf16
 * weights (float32 accumulation; results within float32 rounding of the
 * decode kernels, not bit-identical); smaller batches run the exact decode
 * kernels.  These flags force one path. */
#define FNMOE_LAYER_FORCE_PREFILL 1u
#define FNMOE_LAYER_FORCE_DECODE 2u
#define FNMOE_PREFILL_PAIRS 4096u

/* Repack experts [0, experts) of reference-layout projection arrays into
 * records [first_record, first_record + experts) of tiled tables. */
typedef struct FnTileArgs {
  uint32_t abi_version;
  uint32_t experts;
  uint32_t hidden_size;
  uint32_t inter_size;         /* multiple of 8; hidden a multiple of 16 */
  uint32_t group_size;         /* 32 or 64 */
  uint32_t first_record;
  const uint32_t *gate_weight; const void *gate_scales; const void *gate_biases;
  const uint32_t *up_weight; const void *up_scales; const void *up_biases;
  const uint32_t *down_weight; const void *down_scales; const void *down_biases;
  FnTiledExperts tiled;        /* destination tables (records = capacity) */
} FnTileArgs;

/* Paged-KV decode attention (one query token per sequence). */
typedef struct FnPagedArgs {
  uint32_t abi_version;
  uint32_t batch;              /* sequences */
  uint32_t q_heads;
  uint32_t kv_heads;
  uint32_t head_dim;           /* 64..256, multiple of 64 */
  uint32_t page_size;          /* tokens per page */
  uint32_t max_pages;          /* block_table row length */
  uint32_t num_pages;          /* physical pages in k/v caches */
  float scale;
  uint32_t split_tokens;       /* tokens per split-K chunk (multiple of page_size) */
  const void *q;               /* [batch, q_heads, head_dim] bf16 */
  const void *k_cache;         /* [num_pages, page_size, kv_heads, head_dim] bf16 */
  const void *v_cache;
  const int32_t *block_table;  /* [batch, max_pages] */
  const int32_t *context_lens; /* [batch] */
  void *out;                   /* [batch, q_heads, head_dim] bf16 */
  void *workspace;
  uint64_t workspace_bytes;
} FnPagedArgs;

/* Quantized embedding / n-gram row lookup (fnmoe_rows_dequantize).  The
 * table -- every shard of a sharded table, concatenated in shard order -- is
 * resident on the device: weight [table_rows][dims * bits / 32] uint32 (value
 * j of a word in bits [j*bits, (j+1)*bits), MLX affine packing), scales and
 * biases [table_rows][dims / group_size] bf16.  out[i, k] = bf16(s*q + b),
 * rounded once, of row r(i): indices[i] when it lies in [0, table_rows),
 * else shard 0's row clamp(indices[i], 0, first_shard_rows - 1) (the sharded
 * lookup's clamping, ngram.py:106-119).  count == 0 is a no-op. */
typedef struct FnRowsArgs {
  uint32_t abi_version;
  uint32_t dims;               /* values per row, a multiple of group_size */
  uint32_t bits;               /* 2, 4 or 8 */
  uint32_t group_size;         /* 32, 64 or 128 */
  uint64_t table_rows;         /* rows of the whole (concatenated) table */
  uint64_t first_shard_rows;   /* rows of shard 0 (table_rows for one table) */
  uint64_t count;              /* rows to look up */
  const uint32_t *weight;      /* 8-byte aligned */
  const void *scales;          /* bf16 */
  const void *biases;          /* bf16 */
  const int64_t *indices;      /* [count] device */
  void *out;                   /* [count, dims] bf16, 16-byte aligned */
} FnRowsArgs;

/* 1 when an sm_100 device is current and the library initialised, else 0.
 * Replaces flashnext_native_available (metal_runtime_native.mm:196-201). */
FNMOE_API int fnmoe_available(void);

/* Copy the calling thread's last error message (NUL-terminated).
 * Replaces flashnext_native_get_last_error (metal_runtime_native.mm:203-209). */
FNMOE_API int fnmoe_get_last_error(char *buf, uint32_t max_len);

/* FNMOE_ABI_VERSION of the loaded library. */
FNMOE_API uint32_t fnmoe_abi_version(void);

/* Workspace bytes fnmoe_moe_execute needs for these sizes. */
FNMOE_API int fnmoe_moe_workspace_size(const FnMoEArgs *args, uint64_t *bytes);

/* Executor: replaces flashnext_native_moe_execute (metal_runtime_native.mm:258)
 * and MetalMoEExecutor.execute's packed path (metal_runtime.py:764-932). */
FNMOE_API int fnmoe_moe_execute(const FnMoEArgs *args, void *stream);

/* fnmoe_moe_execute without a caller workspace and without allocating: the
 * scratch is a fixed 16 MiB device array inside the library
 * (FNMOE_STATIC_SCRATCH_BYTES); args->workspace and args->workspace_bytes
 * are ignored.  For callers that hold only device pointers and no device
 * allocator (a C or ctypes bridge like the reference's native one, which
 * keeps process-wide scratch instead of per-call buffers).  No reference
 * counterpart: the reference's bridge allocates and caches its scratch.
 * A call whose scratch (fnmoe_moe_workspace_size less its 256 bytes of
 * alignment slack, which the aligned array does not need) exceeds the static
 * size fails with FNMOE_ERR_WORKSPACE.  The scratch is shared by every call
 * on a device: calls that may overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller.  Its contents persist
 * between calls; nothing in it needs to start at zero (each call rewrites
 * what it reads).  Every call resolves the array's address on the current
 * device (cudaGetSymbolAddress; no allocation, no synchronisation); the first
 * call on a device may load the library's device code, so make that first
 * call before any stream capture. */
FNMOE_API int fnmoe_moe_execute_static(const FnMoEArgs *args, void *stream);

/* Combine-only probe: out[t,h] = sum_s outputs[t,s,h]*scores[t,s] (float32),
 * or outputs[t, routes[t,s], h] when experts > 0 (metal_runtime.py:145-191). */
FNMOE_API int fnmoe_weighted_combine(const float *outputs, const int32_t *routes,
                           const float *scores, float *out, uint32_t tokens,
                           uint32_t slots, uint32_t experts, uint32_t hidden,
                           void *stream);

/* Router chain: logits = bf16(x W^T); softmax (precise) -> top-k (ties to the
 * lower expert) -> renorm.  Writes inds [tokens,k] (uint32), scores [tokens,k]
 * bf16 (renormalised), mass [tokens] bf16 (top-k mass) and optionally logits. */
FNMOE_API int fnmoe_router_topk(const void *x, const void *router_weight, uint32_t tokens,
                      uint32_t hidden, uint32_t experts, uint32_t top_k,
                      float renorm_blend, uint32_t *inds, void *scores,
                      void *mass, void *logits, void *stream);

/* fnmoe_router_topk plus the shared expert's sigmoid gate (adaptive_topk.py:
 * 263-264): shared_gate_weight [hidden] bf16 is run as one more router row;
 * shared_logit [tokens] bf16 receives x.w_g, shared_gate [tokens] bf16
 * sigmoid of it (bfloat16 op sequence).  Used by the expert-parallel layer,
 * which computes the gate on the token's own rank. */
FNMOE_API int fnmoe_router_topk_shared(const void *x, const void *router_weight,
                                       const void *shared_gate_weight, uint32_t tokens,
                                       uint32_t hidden, uint32_t experts, uint32_t top_k,
                                       float renorm_blend, uint32_t *inds, void *scores,
                                       void *mass, void *logits, void *shared_logit,
                                       void *shared_gate, void *stream);

/* fnmoe_router_topk_shared with a caller workspace (adaptive_topk.py:59-64,
 * 263-264, the same outputs): from 64 tokens the logits come from the integer
 * tensor-core GEMM on byte planes of the fixed points, which the workspace
 * holds; fewer tokens take the GEMV path and need none.
 * fnmoe_router_workspace_size reports the bytes (0 when none are needed);
 * a smaller workspace is FNMOE_ERR_WORKSPACE.  Used by the expert-parallel
 * layer, which routes each rank's decode batch. */
FNMOE_API int fnmoe_router_workspace_size(uint32_t tokens, uint32_t hidden, uint32_t experts,
                                          uint32_t with_shared_gate, uint64_t *bytes);
FNMOE_API int fnmoe_router_topk_shared_ws(const void *x, const void *router_weight,
                                          const void *shared_gate_weight, uint32_t tokens,
                                          uint32_t hidden, uint32_t experts, uint32_t top_k,
                                          float renorm_blend, uint32_t *inds, void *scores,
                                          void *mass, void *logits, void *shared_logit,
                                          void *shared_gate, void *workspace,
                                          uint64_t workspace_bytes, void *stream);

/* Slot-ordered combine of per-slot expert outputs (metal_runtime.py:301-333):
 * out[t] = bf16(sum_s float(slot_outputs[t,s]) * score[t,s]) in slot order
 * (float32, no fused multiply-add; slots whose route is >= expert_count are
 * skipped), then + shared_y, or + bf16(shared * shared_gate) when shared and
 * shared_gate are given (one of the two or neither).  slot_outputs
 * [tokens, slots, hidden] bf16, routes [tokens, slots], scores
 * [tokens, slots] (scores_dtype), shared_y/shared [tokens, hidden] bf16,
 * shared_gate [tokens] bf16, out [tokens, hidden] bf16.  The combine stage of
 * fnmoe_moe_execute on its own, for callers whose slot outputs come from
 * elsewhere (the expert-parallel layer). */
FNMOE_API int fnmoe_combine(const void *slot_outputs, const uint32_t *routes, const void *scores,
                            uint32_t scores_dtype, uint32_t tokens, uint32_t slots, uint32_t hidden,
                            uint32_t expert_count, const void *shared_y, const void *shared,
                            const void *shared_gate, void *out, void *stream);

/* Softmax (precise) -> top-k -> renorm on given bf16 logits [tokens, experts]
 * (compiled.router + compiled.renorm, compiled.py:61-71,96-112).  raw_scores
 * (optional) receives the un-normalised top-k probabilities, scores
 * (optional) the renormalised ones. */
FNMOE_API int fnmoe_softmax_topk(const void *logits, uint32_t tokens, uint32_t experts,
                                 uint32_t top_k, float renorm_blend, uint32_t *inds,
                                 void *raw_scores, void *scores, void *mass, void *stream);

/* Stable grouping of routes by key: counts [n_keys], offsets [n_keys+1],
 * order [tokens*slots] (pair indices sorted by key).  Routes with bit 31 map
 * to key array_experts + (route & 0x7FFFFFFF). */
FNMOE_API int fnmoe_group_tokens(const uint32_t *routes, uint32_t pairs,
                       uint32_t array_experts, uint32_t table_records,
                       int32_t *counts, int32_t *offsets, int32_t *order,
                       void *workspace, uint64_t workspace_bytes, void *stream);

FNMOE_API int fnmoe_moe_layer_workspace_size(const FnMoELayerArgs *args, uint64_t *bytes);
FNMOE_API int fnmoe_moe_layer(const FnMoELayerArgs *args, void *stream);

/* Bytes of one tiled record for these sizes (no device work). */
FNMOE_API int fnmoe_tiled_record_bytes(uint32_t hidden_size, uint32_t inter_size, uint32_t group_size,
                                       uint64_t *gate_up_record_bytes, uint64_t *down_record_bytes);
/* Repack projections into tiled tables on `stream` (see FnTileArgs). */
FNMOE_API int fnmoe_tile_experts(const FnTileArgs *args, void *stream);

/* Affine Q4 dequantisation to bf16: out[r, k] = bf16(s*q + b), rounded once. */
FNMOE_API int fnmoe_dequantize(const uint32_t *weight, const void *scales,
                     const void *biases, void *out, uint64_t rows,
                     uint32_t in_width, uint32_t group_size, void *stream);

/* Elementwise bf16 SwiGLU: out = (g*sigmoid(g))*u, one rounding per op. */
FNMOE_API int fnmoe_swiglu(const void *gate, const void *up, void *out, uint64_t n,
                 void *stream);

FNMOE_API int fnmoe_paged_decode_workspace_size(const FnPagedArgs *args, uint64_t *bytes);
FNMOE_API int fnmoe_paged_decode(const FnPagedArgs *args, void *stream);

/* Gather and dequantise table rows (see FnRowsArgs) on `stream`.  Replaces
 * StreamingQuantizedEmbedding.__call__ (ngram.py:62-69, rows read by
 * store.rows then mx.dequantize, ngram.py:49-60) and
 * StreamingShardedEmbedding._direct_rows (ngram.py:160-185); the input
 * embedding's streamed rows use the same class (loader.py:266-283). */
FNMOE_API int fnmoe_rows_dequantize(const FnRowsArgs *args, void *stream);

/* ---- Expert-parallel exchange over NVLink peer memory ----
 * No reference counterpart: the reference runs on one device.  One process
 * per GPU of a node; rank r owns routed experts [r*experts_per_rank,
 * (r+1)*experts_per_rank).  fnmoe_ep_create allocates this rank's exchange
 * window (once, at set-up: the only entry point besides the static-scratch
 * array that owns device memory); every rank passes its IPC handle to the
 * others (any host transport), then opens theirs.  A step is
 *   fnmoe_ep_dispatch        (x rows and owner-local expert ids of every
 *                             token to the ranks that own its slots; waits
 *                             for every rank's rows to arrive),
 *   fnmoe_moe_execute        on the window (FnEpWindow: world*capacity rows,
 *                             top_k + 1 slots, slot top_k = the shared
 *                             expert, the last local record; per-slot
 *                             outputs into window.slot_outputs),
 *   fnmoe_ep_return_combine  (per-slot outputs back to the tokens' ranks,
 *                             slot-ordered combine + gated shared expert).
 * Every rank takes every step (with 0 tokens if it has none), in the same
 * order, on one stream; nothing synchronises with the host, so a step can be
 * captured in a CUDA graph.  Waits on peers give up after about a second and
 * set bit 2 of the device error word; the exchange is then unusable (destroy
 * and recreate it on every rank).  Stores to peers are plain stores: no TMA
 * or multicast. */
#define FNMOE_EP_IPC_BYTES 64

typedef struct FnEpConfig {
  uint32_t abi_version;
  uint32_t world;              /* ranks, 1..8, one GPU each */
  uint32_t rank;
  uint32_t capacity_tokens;    /* most tokens a rank dispatches per step */
  uint32_t hidden_size;        /* multiple of 8, <= 4096 */
  uint32_t top_k;              /* 1..16 */
  uint32_t experts_per_rank;   /* routed experts per rank */
  uint32_t reserved;
} FnEpConfig;

typedef struct FnEpWindow {
  const void *rows;            /* [world * capacity][hidden] bf16 received rows */
  const uint32_t *ids;         /* [world * capacity][top_k + 1] local expert ids (FNMOE_ROUTE_NONE = empty) */
  void *slot_outputs;          /* [world * capacity][top_k + 1][hidden] bf16: per-slot outputs of the experts */
  uint32_t row_count;          /* world * capacity */
  uint32_t slots;              /* top_k + 1 */
  uint64_t bytes;              /* window size */
} FnEpWindow;

FNMOE_API int fnmoe_ep_create(const FnEpConfig *config, void **handle);
FNMOE_API int fnmoe_ep_ipc_handle(void *handle, void *out);          /* FNMOE_EP_IPC_BYTES bytes */
FNMOE_API int fnmoe_ep_open_peers(void *handle, const void *handles); /* world handles in rank order */
FNMOE_API int fnmoe_ep_window(void *handle, FnEpWindow *window);
FNMOE_API int fnmoe_ep_dispatch(void *handle, const void *x, const uint32_t *inds, uint32_t tokens,
                                void *stream);
FNMOE_API int fnmoe_ep_return_combine(void *handle, const void *scores, const void *shared_gate,
                                      uint32_t tokens, void *out, void *stream);
/* Synchronises the device, unmaps the peers' windows and frees this one;
 * call it on every rank after a barrier (no peer may still write here). */
FNMOE_API int fnmoe_ep_destroy(void *handle);

/* Device error word of the library: bit 0 = an out-of-range route was
 * skipped, bit 1 = a non-finite activation reached the fixed-point stage,
 * bit 2 = a bounded wait in a kernel gave up (its outputs are invalid),
 * bit 3 = an out-of-range prefill tile descriptor was skipped.
 * Reading synchronises the device; `clear` resets it. */
FNMOE_API int fnmoe_read_device_errors(uint32_t *flags, int clear);

/* Per-kernel device timing for benchmarks: while enabled, every kernel the
 * library launches is bracketed by CUDA events on its stream.
 * fnmoe_profile_read synchronises those events and writes
 * "name count total_ms\n" lines for each kernel into buf. */
FNMOE_API int fnmoe_profile_enable(int on);
FNMOE_API int fnmoe_profile_read(char *buf, uint32_t max_len, int reset);

#ifdef __cplusplus
}
#endif

#endif /* FNMOE_H */
