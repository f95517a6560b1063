// moe_kernels.cuh -- launch-side declarations shared by moe_kernels.cu and api.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fnmoe {

// Key assigned to the shared expert's bin in grouping.
constexpr uint32_t kSharedKey = 0xFFFFFFFFu;
// Pairs per grouped work item: up to two 4-token MMA tiles (N = 4 tokens x 2 limbs).
constexpr int kTokPerItem = 8;

// Pointers of one Q4 projection family.
struct ProjArrays {
  const uint32_t *w;   // [experts, rows, cols/8]
  const uint16_t *s;   // [experts, rows, cols/G]
  const uint16_t *b;
};

// HBM-resident expert table (device view of FnExpertTable).
struct TableView {
  const uint8_t *base;
  uint64_t header;
  uint64_t stride;
  uint64_t off[9];
  uint32_t records;
};

// Grouping results living in the workspace.
struct GroupView {
  int32_t *counts;     // [n_bins]
  int32_t *offsets;    // [n_bins + 1]
  int32_t *order;      // [n_total]   pair ids sorted by bin
  int4 *tiles;         // [3 * max_tiles] {route key, start, len, bin}, {pair ids 0-3}, {pair ids 4-7}
  int32_t *n_tiles;    // [4]: tile count (the rest is spare)
  uint32_t *bin_key;   // [n_bins]    route key of each bin
  int n_bins;
  int max_tiles;
};

struct DeviceInfo {
  int device;
  int sms;
};

DeviceInfo device_info();
cudaError_t ensure_exp_table(cudaStream_t stream);
// Device address of the bfloat16 exp table (initialised by ensure_exp_table).
cudaError_t exp_table_address(const uint16_t **table);
// Device address of the bfloat16 g*sigmoid(g) table (initialised with the exp table).
cudaError_t silu_table_address(const uint16_t **table);
uint32_t *device_error_word();

// Row fixed point of bf16 rows: limbs [rows][groups][2][G] fp16 (fragment
// order), meta [rows][meta_pitch(groups)] float (fl(SX) per group, then
// {A, B}; see meta_a_index).
// With skip_routes, row r < n_skip whose route skip_routes[r] is
// FNMOE_ROUTE_NONE (an empty slot) is skipped: its row is not read and its
// limbs are not written.
cudaError_t launch_prep_rows(const uint16_t *rows, int n_rows, int K, int G,
                             uint16_t *limbs, float *meta, cudaStream_t s,
                             const uint32_t *skip_routes = nullptr, int n_skip = 0);

// The same fixed point of float32 rows (K <= 4096).
cudaError_t launch_prep_rows_f32(const float *rows, int n_rows, int K, int G, uint16_t *limbs, float *meta,
                                 cudaStream_t s, const uint32_t *skip_routes = nullptr, int n_skip = 0);

// Softmax/top-k/renorm of <= 8 tokens followed by the grouping, one launch
// (cudaErrorNotSupported when T or E is too large for it).  tiles_only:
// write only the decode tiles (with the pair order), not the per-bin counts
// and offsets -- enough for the decode expert kernels.
cudaError_t launch_route_small(const uint16_t *logits, int T, int E, int k, float blend,
                               const uint32_t *route_map, int table_routes, uint32_t *inds,
                               uint32_t *routes, uint16_t *raw_scores, uint16_t *scores,
                               uint16_t *mass, const uint16_t *shared_logit, uint16_t *shared_gate,
                               int shared_tokens, int array_experts, int table_records, GroupView gv,
                               cudaStream_t s, double keep_threshold = 0.0, int min_keep = 0,
                               bool tiles_only = false);

// The same grouping over many CTAs for large pair counts: counts, offsets,
// bin keys and order only (no decode tiles; n_tiles = 0).  `hist` is scratch
// of chunks * n_bins ints (chunks = ceil(pairs / 4096)); cudaErrorNotSupported
// when it or the bins do not fit.
cudaError_t launch_group_large(const uint32_t *routes, int n_pairs, int shared_tokens, int array_experts,
                               int table_records, GroupView gv, int *hist, size_t hist_bytes, cudaStream_t s);

// Stable counting-sort grouping of routes (+ optional shared bin).
cudaError_t launch_group(const uint32_t *routes, int n_pairs, int shared_tokens,
                         int array_experts, int table_records, GroupView gv,
                         cudaStream_t s);

// Tiled expert tables (fnmoe_tile_experts): one kTileChunk-byte chunk per
// (row group, 128-byte block) -- 8 gate + 8 up rows for gate/up, 16 rows for
// down -- in MMA fragment order, scales and biases included.
constexpr int kTileChunk = 2560;
constexpr int kTileW = 2048;  // packed-word bytes at the start of a chunk

struct TiledView {
  const uint8_t *gate_up;   // [records][I/8 row groups][blocks][kTileChunk], or null
  const uint8_t *down;      // [records][H/16 row groups][blocks][kTileChunk], or null
  uint64_t gate_up_record;  // bytes per record
  uint64_t down_record;
  uint32_t records;         // routed experts (+1 when has_shared: the last record)
  int has_shared;
};

struct ExpertCallArgs {
  ProjArrays gate, up, down;          // routed arrays (may be null if table-only)
  ProjArrays sh_gate, sh_up, sh_down; // shared expert (bin key kSharedKey)
  TableView table;
  TableView stream;                   // records for routes without bit 31 (optional)
  int array_experts;                  // valid non-slot route range
  int tokens, slots, n_pairs;         // n_pairs = tokens*slots (routed)
  int H, I, I_shared, G;
  int sb_async;                       // scale/bias bases 4-byte aligned (rows too when the group count is even)
  int sb_bulk;                        // scale/bias bases 16-byte aligned
  TiledView tiled;                    // tiled tables replace the arrays when set
  int f32;                            // float32 activations: outputs float32, float32 SwiGLU
};

// gate/up + SwiGLU over all grouped tiles -> act [n_total, I] bf16.
cudaError_t launch_gate_up(const ExpertCallArgs &a, const GroupView &gv,
                           const uint16_t *x_limbs, const float *x_meta,
                           uint16_t *act, uint16_t *g_out, uint16_t *u_out,
                           cudaStream_t s);
// down projection -> d [n_total, H] bf16.
cudaError_t launch_down(const ExpertCallArgs &a, const GroupView &gv,
                        const uint16_t *act_limbs, const float *act_meta,
                        uint16_t *d, cudaStream_t s);

// Combine modes.
enum CombineMode { kCombineNone = 0, kCombineSharedY = 1, kCombineParts = 2 };
cudaError_t launch_combine(const uint16_t *d, const uint32_t *routes,
                           const void *scores, int scores_f32, int tokens,
                           int slots, int H, int mode, const uint16_t *shared_y,
                           const uint16_t *shared, const uint16_t *shared_gate,
                           int array_experts, int table_records,
                           uint16_t *out, cudaStream_t s);

// The combine with float32 per-slot rows, shared inputs and output.
cudaError_t launch_combine_f32(const float *d, const uint32_t *routes, const void *scores, int scores_f32,
                               int tokens, int slots, int H, int mode, const float *shared_y, const float *shared,
                               const float *shared_gate, int array_experts, int table_records, float *out,
                               cudaStream_t s);

// Router.
// With prep_limbs / prep_meta set, batches of <= 4 tokens also compute the
// row fixed point of x (launch_prep_rows' output) in extra CTAs of the same
// launch; *prep_done tells whether that happened (else call launch_prep_rows).
// Scratch of the many-token router: the byte-limb planes of the token rows'
// and router rows' fixed points and their row exponents (router_scratch_bytes).
struct RouterScratch {
  uint8_t *xq;  // [3][T][H]: bytes 0 and 1 (unsigned) and 2 (signed) of X
  uint8_t *wq;  // [2][R][H]: byte 0 (unsigned) and 1 (signed) of W
  int32_t *ex;  // [T]
  int32_t *ew;  // [R]
  unsigned long long *acc;  // [T][R] int64 partial sums (split-K only)
  int32_t *tickets;         // per 64 x 64 tile (split-K only)
  int ksplit;               // K slices per tile (router_ksplit)
};
// K slices of the tensor-core router for these sizes: enough (sequence of
// 128-byte k-chunks split evenly) that small token counts still fill the SMs.
int router_ksplit(int T, int R, int H);
// Output tiles of the tensor-core router (split-K tickets).
int router_tiles(int T, int R);
// Bytes of RouterScratch for T tokens and R router rows (0 when the tensor-
// core path does not apply: fewer than 64 tokens or H not a multiple of 128).
uint64_t router_scratch_bytes(int T, int R, int H);

// Router logits.  With `rs` (sized by router_scratch_bytes) and at least 64
// tokens, the integer tensor-core path; otherwise the exact integer GEMV.
cudaError_t launch_router_logits(const uint16_t *x, const uint16_t *W, int T,
                                 int H, int E, const uint16_t *w_shared_gate,
                                 uint16_t *logits, uint16_t *shared_logit,
                                 cudaStream_t s, uint16_t *prep_limbs = nullptr,
                                 float *prep_meta = nullptr, int prep_G = 32,
                                 bool *prep_done = nullptr, const RouterScratch *rs = nullptr);
cudaError_t launch_softmax_topk(const uint16_t *logits, int T, int E, int k,
                                float blend, const uint32_t *route_map,
                                int table_routes, uint32_t *inds,
                                uint32_t *routes, uint16_t *raw_scores,
                                uint16_t *scores, uint16_t *mass,
                                const uint16_t *shared_logit,
                                uint16_t *shared_gate, cudaStream_t s,
                                double keep_threshold = 0.0, int min_keep = 0);

// Repack `experts` experts' projections (reference layout) into tiled
// records: dual = gate (A) + up (B) rows, else down rows.
cudaError_t launch_tile_experts(const uint32_t *wA, const uint32_t *wB, const uint16_t *sA, const uint16_t *bA,
                                const uint16_t *sB, const uint16_t *bB, int experts, int O, int K, int G, bool dual,
                                uint8_t *dst, uint64_t record_bytes, cudaStream_t s);
uint64_t tiled_record_bytes(int O, int K, bool dual);

// Prefill (tcgen05) path: 128-pair tiles per expert bin, then grouped GEMMs
// on tiled tables with dequantised bf16 weights (G = 32, K % 256 == 0).
bool prefill_supported(const ExpertCallArgs &a);
int prefill_max_tiles(int n_total, int n_bins);
cudaError_t launch_prefill_tiles(const GroupView &gv, int4 *ptiles, int32_t *n_ptiles, int max_tiles,
                                 cudaStream_t s);
// Token rows of x gathered into bin order: dst [n_total][H], row p = x row of pair gv.order[p].
cudaError_t launch_prefill_gather(const ExpertCallArgs &a, const GroupView &gv, const uint16_t *x, uint16_t *dst,
                                  cudaStream_t s);
// Prefill grouped GEMM on tcgen05, inputs and activations in bin order:
// gate/up (dual) reads the gathered x rows ([in_rows = n_total][H]) and
// writes SwiGLU activations ([n_total][I]); down reads those ([in_rows =
// n_total][I]) and writes per-pair outputs ([n_total][H]).
cudaError_t launch_prefill_gemm(bool dual, const ExpertCallArgs &a, const GroupView &gv, const int4 *ptiles,
                                const int32_t *n_ptiles, int max_tiles, const uint16_t *in, int in_rows,
                                uint16_t *out, cudaStream_t s);

// Batch-1 layer as one persistent kernel (decode_layer.cuh): router,
// top-k, gate/up, down and combine of one token with two grid barriers.
struct FusedLayer {
  const uint16_t *x;        // [H] bf16
  const uint16_t *W;        // [E][H] bf16 router rows
  const uint16_t *wsg;      // [H] bf16 shared-expert gate row, or null (no shared expert)
  TiledView tiled;          // routed records [0, E) (+ the shared expert as the last record)
  int E, k, H, I;
  float blend;
  double keep_threshold;
  int min_keep;
  uint16_t *logits;         // [E] bf16
  uint16_t *shared_logit;   // [1] bf16
  uint32_t *inds;           // [k]
  uint16_t *scores;         // [k] bf16 (renormalised)
  uint16_t *mass;           // [1] bf16 (top-k mass)
  uint16_t *shared_gate;    // [1] bf16 sigmoid(shared logit)
  uint16_t *act;            // [k + 1][I] bf16: slot s at row s, the shared expert at row k
  uint32_t *bar;            // grid-barrier counter (grid_barrier_slot)
  uint32_t *amax;           // [k + 1] activation row maxima (bfloat16 magnitude bits), workspace
  uint16_t *out;            // [H] bf16
  // shared-memory carve (byte offsets into the dynamic allocation)
  int nslot;                // ring slots = most gate/up items a CTA can get
  int alias;                // 1: the down stage and activation limbs reuse the ring
  int off_x, off_xq, off_xl, off_xm, off_soft, off_d, off_ring, off_down, off_al, off_am;
};

// cudaErrorNotSupported when the sizes do not fit the fused kernel (the
// caller then runs the multi-launch layer).
cudaError_t launch_decode_layer(FusedLayer p, int G, cudaStream_t s);
// true when FNMOE_NO_FUSED is set: batch-1 layers run the multi-launch chain.
bool fused_disabled();
// The fused kernel's grid-barrier counter for workspace `key` (library-owned,
// zero-initialised, self-cleaning); reset_grid_barriers() after a timeout.
cudaError_t grid_barrier_slot(const void *key, uint32_t **bar);
cudaError_t reset_grid_barriers();

cudaError_t launch_dequant(const uint32_t *w, const uint16_t *sc,
                           const uint16_t *bi, uint16_t *out, uint64_t rows,
                           int K, int G, cudaStream_t s);
cudaError_t launch_swiglu(const uint16_t *g, const uint16_t *u, uint16_t *out,
                          uint64_t n, cudaStream_t s);
cudaError_t launch_weighted_combine(const float *outputs, const int32_t *routes,
                                    const float *scores, float *out, int T,
                                    int S, int E, int H, cudaStream_t s);

// Expert-parallel exchange (ep.cu); the FnEp* types come from fnmoe.h.
}  // namespace fnmoe
#include <string>
struct FnEpConfig;
struct FnEpWindow;
namespace fnmoe {
int ep_create(const FnEpConfig *cfg, void **out, std::string &err);
int ep_ipc_handle(void *handle, void *out64, std::string &err);
int ep_open_peers(void *handle, const void *handles, std::string &err);
int ep_destroy(void *handle, std::string &err);
int ep_window(void *handle, FnEpWindow *w, std::string &err);
int ep_dispatch(void *handle, const void *x, const uint32_t *inds, uint32_t tokens, cudaStream_t s, std::string &err);
int ep_return_combine(void *handle, const void *scores, const void *shared_gate, uint32_t tokens, void *out,
                      cudaStream_t s, std::string &err);
}  // namespace fnmoe
