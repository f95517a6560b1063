// prefill.cu -- grouped expert GEMMs on tcgen05 for prefill-sized batches.
//
// For thousands of tokens per layer (a prefill chunk) each expert sees ~100
// pairs and its projections become GEMMs.  A work item is a tile of up to 128
// pairs of one expert bin (MMA M) times 256 output rows (MMA N): 128 gate +
// 128 up rows (interleaved in groups of 8, as in the tiled tables) for
// gate/up, 256 rows for down.  One persistent CTA per SM runs the items with
// warp-specialised roles around mbarrier rings:
//
//   warp 0      producer: per 256-wide K block one bulk copy per row group
//               (the 2560-byte chunks of the tiled tables) into a raw ring;
//               per 64-wide k-step the tile's 128 input rows as one
//               128B-swizzled K-major TMA box -- the inputs are in bin order
//               (x rows gathered by k_gather_rows for gate/up, the bin-ordered
//               activations for down), so a tile's rows are contiguous;
//   warp 1      MMA issuer: 4 tcgen05.mma (kind::f16, bf16, M128 N256 K16)
//               per k-step into one of two 256-column fp32 accumulators in
//               TMEM, commits releasing the input stages;
//   warps 2-17  dequantise the raw ring into bf16 swizzled weight tiles,
//               bf16(s*q + b) with one rounding (fma.rn.bf16x2), the
//               reference's dequant rule;
//   warps 18-25 epilogue (two warps per TMEM lane quarter, half the columns
//               each): tcgen05.ld of the finished accumulator, then bf16
//               SwiGLU activations in bin order (gate/up) or bf16 per-pair
//               outputs (down), while the MMAs of the next item fill the
//               other accumulator.  g*sigmoid(g) comes from a shared-memory
//               slice of the bit-identical table for |g| in [2^-9, 2^7).
//
// Accumulation is float32 in the tensor core's order, so results match the
// exact decode path within float32 rounding, not bit for bit.  Every wait is
// bounded; a timeout sets the device error word, marks the CTA dead (later
// waits return at once) and the kernel runs to its end.

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "async.cuh"
#include "common.cuh"
#include "moe_kernels.cuh"
#include "umma.cuh"

namespace fnmoe {

namespace {

constexpr int kPM = 128;  // pairs per tile (MMA M)
constexpr int kPN = 256;  // output rows per item (MMA N)
constexpr int kDeqWarps = 16, kEpiWarps = 8;
constexpr int kDeqWarp0 = 2, kEpiWarp0 = kDeqWarp0 + kDeqWarps;
constexpr int kPThreads = 32 * (kEpiWarp0 + kEpiWarps);  // 832
constexpr int kAStages = 4, kBStages = 2, kRawStages = 2;
constexpr int kATile = kPM * 128;           // 128 rows x 64 bf16
constexpr int kBTile = kPN * 128;           // 256 rows x 64 bf16
constexpr int kRawTile = 16 * kTileChunk;   // 16 row groups x one 256-wide K block
constexpr int kSiluLo = 118, kSiluExps = 16;  // bf16 exponents 118..133: |g| in [2^-9, 2^7)
constexpr int kSiluEntries = 2 * kSiluExps * 128;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kAStages * kATile;
constexpr int kOffRaw = kOffB + kBStages * kBTile;
constexpr int kOffSilu = kOffRaw + kRawStages * kRawTile;
constexpr int kOffBar = kOffSilu + kSiluEntries * 2;
// barriers: a_full[4] a_empty[4] b_full[2] b_empty[2] raw_full[2] raw_empty[2] acc_full[2] acc_empty[2]
constexpr int kBarA = 0, kBarAE = kBarA + kAStages, kBarB = kBarAE + kAStages, kBarBE = kBarB + kBStages;
constexpr int kBarR = kBarBE + kBStages, kBarRE = kBarR + kRawStages, kBarC = kBarRE + kRawStages,
              kBarCE = kBarC + 2, kBars = kBarCE + 2;
constexpr int kOffMisc = kOffBar + kBars * 8;  // tmem base, dead flag
constexpr int kPSmem = kOffMisc + 16 + 1024;   // + slack for the 1024-byte alignment of the tiles
static_assert(kPSmem <= 227 * 1024, "prefill shared memory");
constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators
constexpr uint32_t kPSpinLimit = 1u << 22;

// Instruction descriptor: kind::f16, bf16 A and B (K-major), f32 D, M 128, N 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kPN >> 3) << 17) |
                            (static_cast<uint32_t>(kPM >> 4) << 24);

__device__ __forceinline__ void sts128(uint32_t s, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"r"(s), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s_u32(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
// Bounded wait on `bar` for the phase of parity `parity`.  A timeout (or a
// CTA already marked dead) returns false: the caller's role stops waiting.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile uint32_t *dead, uint32_t *err) {
  uint32_t spins = 0;
  while (!mbar_try_wait_u32(bar, parity)) {
    if (*dead) return false;
    if (++spins >= kPSpinLimit) {
      *dead = 1u;
      set_error(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_fma_q(uint32_t p, uint32_t ss, uint32_t bb) {
  // p holds bf16 (128 + q) pairs: subtract 128 exactly, then bf16(s*q + b) with one rounding.
  uint32_t q, d;
  asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(q) : "r"(p), "r"(0x43004300u));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(q), "r"(ss), "r"(bb));
  return d;
}
// 8 nibbles (inputs k..k+7, low nibble first) -> 8 dequantised bf16 in k order.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t ss, uint32_t bb) {
  const uint32_t t = w & 0x0F0F0F0Fu;          // nibbles 0, 2, 4, 6
  const uint32_t u = (w >> 4) & 0x0F0F0F0Fu;   // nibbles 1, 3, 5, 7
  const uint32_t lo = prmt(t, u, 0x5140u);     // nibbles 0 1 2 3 as bytes
  const uint32_t hi = prmt(t, u, 0x7362u);     // nibbles 4 5 6 7
  const uint32_t M = 0x43434343u;              // bf16 high byte of 128..143
  return make_uint4(bf16x2_fma_q(prmt(lo, M, 0x5140u), ss, bb), bf16x2_fma_q(prmt(lo, M, 0x5342u), ss, bb),
                    bf16x2_fma_q(prmt(hi, M, 0x5140u), ss, bb), bf16x2_fma_q(prmt(hi, M, 0x5342u), ss, bb));
}

__device__ __forceinline__ bool record_of(const ExpertCallArgs &a, uint32_t key, uint32_t &rec) {
  if (key == kSharedKey) {
    if (!a.tiled.has_shared) return false;
    rec = a.tiled.records - 1;
    return true;
  }
  if (key >= static_cast<uint32_t>(a.array_experts)) return false;
  rec = key;
  return true;
}

__device__ __forceinline__ int pair_row(int pair, int n_pairs, int slots) {
  return pair < n_pairs ? pair / slots : pair - n_pairs;
}

struct PItem {
  bool ok;
  int nt, start, len;
  uint32_t rec;
};

// Tile `item / NT`, checked against the pair count: a descriptor out of
// range is not ok (the producer reports it) and every role skips it.
__device__ __forceinline__ PItem item_of(const ExpertCallArgs &a, const int4 *ptiles, int item, int NT,
                                         int n_rows) {
  const int pt = item / NT;
  const int4 d0 = ptiles[pt];
  PItem it;
  it.nt = item - pt * NT;
  it.start = d0.y;
  it.len = d0.z;
  it.rec = 0;
  it.ok = record_of(a, static_cast<uint32_t>(d0.x), it.rec) && it.start >= 0 && it.len >= 1 && it.len <= kPM &&
          it.start <= n_rows - it.len;
  return it;
}

// Every role walks the same item sequence (blockIdx.x, + gridDim.x, ...) and
// skips the same bad items, so the rings stay in step.
template <bool DUAL>
__global__ void __launch_bounds__(kPThreads, 1) k_prefill_gemm(ExpertCallArgs a, GroupView gv,
                                                               const int4 *ptiles, const int32_t *n_ptiles,
                                                               int max_tiles, int n_rows,
                                                               const __grid_constant__ CUtensorMap in_map,
                                                               uint16_t *__restrict__ out,
                                                               const uint16_t *__restrict__ silu_tab,
                                                               uint32_t *err) {
  extern __shared__ uint8_t psmem_raw[];
  pdl_wait();
  pdl_trigger();
  const uint32_t raw0 = smem_u32(psmem_raw);
  const uint32_t sbase = (raw0 + 1023u) & ~1023u;
  uint8_t *sm = psmem_raw + (sbase - raw0);
  const uint32_t bars = sbase + kOffBar;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kOffMisc);
  volatile uint32_t *dead = reinterpret_cast<volatile uint32_t *>(sm + kOffMisc + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = DUAL ? a.H : a.I;
  const int O = DUAL ? a.I : a.H;
  const int NT = DUAL ? O / 128 : O / 256;
  const int nblk = K / 256;
  const uint64_t rec_bytes = DUAL ? a.tiled.gate_up_record : a.tiled.down_record;
  const uint8_t *tbase = DUAL ? a.tiled.gate_up : a.tiled.down;
  const int n_items = min(n_ptiles[0], max_tiles) * NT;
  if (static_cast<int>(blockIdx.x) >= n_items) return;

  if (tid == 0) {
    for (int i = 0; i < kBars; ++i) {
      uint32_t count = 1;
      if ((i >= kBarB && i < kBarB + kBStages) || (i >= kBarRE && i < kBarRE + kRawStages)) count = kDeqWarps;
      if (i >= kBarCE && i < kBarCE + 2) count = kEpiWarps;
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bars + 8 * i), "r"(count));
    }
    *dead = 0u;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  uint16_t *s_silu = reinterpret_cast<uint16_t *>(sm + kOffSilu);
  for (int i = tid; i < kSiluEntries; i += blockDim.x) {
    const int sign = i / (kSiluExps * 128), rest = i - sign * (kSiluExps * 128);
    s_silu[i] = silu_tab[(sign << 15) | ((kSiluLo + (rest >> 7)) << 7) | (rest & 127)];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    uint32_t a_st = 0, a_ph = 0, r_st = 0, r_ph = 0;
    bool live = true;
    for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
      const PItem it = item_of(a, ptiles, item, NT, n_rows);
      if (!it.ok) {
        if (lane == 0) set_error(err, kErrBadTile);
        continue;
      }
      const uint8_t *brg = tbase + it.rec * rec_bytes + static_cast<size_t>(it.nt * 16) * nblk * kTileChunk;
      for (int kb = 0; kb < nblk && live; ++kb) {
        if (lane == 0) {
          live = bar_wait(bars + 8 * (kBarRE + r_st), r_ph ^ 1u, dead, err);
          if (live) mbar_expect_tx_u32(bars + 8 * (kBarR + r_st), kRawTile);
        }
        live = __shfl_sync(0xFFFFFFFFu, live, 0);
        if (!live) break;
        if (lane < 16)
          bulk_g2s_u32(sbase + kOffRaw + r_st * kRawTile + lane * kTileChunk,
                       brg + (static_cast<size_t>(lane) * nblk + kb) * kTileChunk, kTileChunk,
                       bars + 8 * (kBarR + r_st));
        if (++r_st == kRawStages) {
          r_st = 0;
          r_ph ^= 1u;
        }
        for (int ks = 0; ks < 4; ++ks) {
          const int kt = kb * 4 + ks;
          if (lane == 0) {
            live = bar_wait(bars + 8 * (kBarAE + a_st), a_ph ^ 1u, dead, err);
            if (live) mbar_expect_tx_u32(bars + 8 * (kBarA + a_st), kATile);
          }
          live = __shfl_sync(0xFFFFFFFFu, live, 0);
          if (!live) break;
          if (lane == 0) tma_box2d(sbase + kOffA + a_st * kATile, &in_map, kt * 64, it.start, bars + 8 * (kBarA + a_st));
          if (++a_st == kAStages) {
            a_st = 0;
            a_ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t a_st = 0, a_ph = 0, b_st = 0, b_ph = 0;
      int n = 0;
      bool live = true;
      for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
        const PItem it = item_of(a, ptiles, item, NT, n_rows);
        if (!it.ok) continue;
        const uint32_t acc = n & 1, acc_ph = (n >> 1) & 1;
        ++n;
        if (!bar_wait(bars + 8 * (kBarCE + acc), acc_ph ^ 1u, dead, err)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * 256;
        for (int kt = 0; kt < 4 * nblk; ++kt) {
          live = bar_wait(bars + 8 * (kBarA + a_st), a_ph, dead, err) &&
                 bar_wait(bars + 8 * (kBarB + b_st), b_ph, dead, err);
          if (!live) break;
          tc_fence_after();
          const uint64_t ad = sw128_desc(sbase + kOffA + a_st * kATile);
          const uint64_t bd = sw128_desc(sbase + kOffB + b_st * kBTile);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(d, ad + 2 * kk, bd + 2 * kk, (kt | kk) != 0 ? 1u : 0u);
          umma_commit(bars + 8 * (kBarAE + a_st));
          umma_commit(bars + 8 * (kBarBE + b_st));
          if (++a_st == kAStages) {
            a_st = 0;
            a_ph ^= 1u;
          }
          if (++b_st == kBStages) {
            b_st = 0;
            b_ph ^= 1u;
          }
        }
        if (live) umma_commit(bars + 8 * (kBarC + acc));
      }
    }
  } else if (warp < kEpiWarp0) {
    // ---------------- dequantisation ----------------
    const int dw = warp - kDeqWarp0;
    const int r = lane >> 2, c = lane & 3;
    uint32_t b_st = 0, b_ph = 0, r_st = 0, r_ph = 0;
    bool live = true;
    for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
      const PItem it = item_of(a, ptiles, item, NT, n_rows);
      if (!it.ok) continue;
      for (int kb = 0; kb < nblk && live; ++kb) {
        live = bar_wait(bars + 8 * (kBarR + r_st), r_ph, dead, err);
        if (!live) break;
        const uint32_t raw = sbase + kOffRaw + r_st * kRawTile;
        for (int ks = 0; ks < 4; ++ks) {
          live = bar_wait(bars + 8 * (kBarBE + b_st), b_ph ^ 1u, dead, err);
          if (!live) break;
          const int h = ks >> 1, i0 = 2 * (ks & 1);
          const uint32_t bt = sbase + kOffB + b_st * kBTile;
#pragma unroll
          for (int task = 0; task < 32 / kDeqWarps; ++task) {
            const int wt = dw * (32 / kDeqWarps) + task;
            const int rg = wt >> 1, side = wt & 1;
            const uint32_t ch = raw + rg * kTileChunk;
            const uint2 w2 = lds64(ch + h * 1024 + side * 512 + (r * 4 + c) * 16 + i0 * 4);
            const uint32_t sbo = ch + kTileW + (side * 8 + r) * 32 + (4 * h + i0) * 2;
            const uint32_t sc = lds32(sbo), bi = lds32(sbo + 16);
            const int n = rg * 16 + side * 8 + r;
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
              const uint32_t ss = prmt(sc, 0u, gi ? 0x3232u : 0x1010u);
              const uint32_t bb = prmt(bi, 0u, gi ? 0x3232u : 0x1010u);
              const uint4 v = dequant_word(gi ? w2.y : w2.x, ss, bb);
              const int j = 4 * gi + c;
              sts128(bt + n * 128 + ((j ^ r) << 4), v);
            }
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(bars + 8 * (kBarB + b_st));
          if (++b_st == kBStages) {
            b_st = 0;
            b_ph ^= 1u;
          }
        }
        fence_proxy_async();  // generic reads of the raw stage before the next bulk copy into it
        __syncwarp();
        if (lane == 0) mbar_arrive(bars + 8 * (kBarRE + r_st));
        if (++r_st == kRawStages) {
          r_st = 0;
          r_ph ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 belong to this warp
    const int m = 32 * quarter + lane;
    const int cc0 = ((warp - kEpiWarp0) >> 2) * 4;  // this warp's four 32-column chunks
    int n = 0;
    bool live = true;
    for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
      const PItem it = item_of(a, ptiles, item, NT, n_rows);
      if (!it.ok) continue;
      const uint32_t acc = n & 1, acc_ph = (n >> 1) & 1;
      ++n;
      live = bar_wait(bars + 8 * (kBarC + acc), acc_ph, dead, err);
      if (!live) break;
      tc_fence_after();
      bool valid = m < it.len;
      int row_i = 0;
      if (valid) row_i = DUAL ? it.start + m : gv.order[it.start + m];
      if (valid && (row_i < 0 || row_i >= n_rows)) {
        set_error(err, kErrBadTile);
        valid = false;
      }
      const size_t row = static_cast<size_t>(row_i);
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + acc * 256;
#pragma unroll 1
      for (int cc = cc0; cc < cc0 + 4; ++cc) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(taddr + 32 * cc, v);
        if (valid && DUAL) {
          // columns: [gate rg 2cc, rows 0-7][up rg 2cc][gate rg 2cc+1][up rg 2cc+1]
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int base = (j < 4) ? 0 : 16;
            const int jj = 2 * (j & 3);
            float r2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint32_t g = f32_to_bf16(__uint_as_float(v[base + jj + e]));
              const float u = round_bf16(__uint_as_float(v[base + 8 + jj + e]));
              const uint32_t ex = ((g >> 7) & 0xFFu) - static_cast<uint32_t>(kSiluLo);
              const uint16_t sv = ex < static_cast<uint32_t>(kSiluExps)
                                      ? s_silu[((g >> 15) << 11) | (ex << 7) | (g & 127u)]
                                      : silu_tab[g];
              r2[e] = bmul(bf16_to_f32(sv), u);
            }
            o[j] = static_cast<uint32_t>(f32_to_bf16(r2[0])) | (static_cast<uint32_t>(f32_to_bf16(r2[1])) << 16);
          }
          uint4 *dst = reinterpret_cast<uint4 *>(out + row * O + it.nt * 128 + 16 * cc);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else if (valid) {
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            o[j] = static_cast<uint32_t>(f32_to_bf16(__uint_as_float(v[2 * j]))) |
                   (static_cast<uint32_t>(f32_to_bf16(__uint_as_float(v[2 * j + 1]))) << 16);
          uint4 *dst = reinterpret_cast<uint4 *>(out + row * O + it.nt * 256 + 32 * cc);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8 * (kBarCE + acc));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Input rows of the gate/up GEMM in bin order: row p of `dst` is the token
// row of pair order[p] (one warp per row, 16-byte copies).
__global__ void __launch_bounds__(256) k_gather_rows(const int32_t *order, const int32_t *grouped, int n_rows,
                                                     int n_pairs, int slots, int n_tokens, const uint16_t *x, int H,
                                                     uint16_t *dst, uint32_t *err) {
  pdl_wait();
  pdl_trigger();
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (p >= n_rows || p >= grouped[0]) return;  // grouped[0]: pairs placed by the grouping
  const int pair = order[p];
  int t = (pair >= 0 && pair < n_rows) ? pair_row(pair, n_pairs, slots) : -1;
  if (t < 0 || t >= n_tokens) {
    if (lane == 0) set_error(err, kErrBadTile);
    t = 0;
  }
  const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * H);
  uint4 *d = reinterpret_cast<uint4 *>(dst + static_cast<size_t>(p) * H);
  for (int i = lane; i < H / 8; i += 32) d[i] = src[i];
}

// 128-pair tiles of every bin from the grouping counts and offsets (one CTA).
__global__ void __launch_bounds__(1024) k_prefill_tiles(GroupView gv, int4 *ptiles, int32_t *n_ptiles,
                                                        int max_tiles) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_sums[32];
  __shared__ int total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (gv.n_bins + 1023) / 1024;
  const int b0 = min(tid * per, gv.n_bins), b1 = min(b0 + per, gv.n_bins);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += (gv.counts[b] + kPM - 1) / kPM;
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, wi, off);
      if (lane >= off) wi += v;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) total = wi;
  }
  __syncthreads();
  int t = incl - local + warp_sums[warp];
  for (int b = b0; b < b1; ++b) {
    const int c = gv.counts[b];
    for (int i = 0; i * kPM < c; ++i, ++t)
      if (t < max_tiles)
        ptiles[t] = make_int4(static_cast<int>(gv.bin_key[b]), gv.offsets[b] + i * kPM, min(kPM, c - i * kPM), b);
  }
  if (tid == 0) n_ptiles[0] = min(total, max_tiles);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 matrix [rows][cols] (row pitch cols), 128B swizzle, box 64 x box_rows.
cudaError_t make_map(CUtensorMap *map, const void *base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

bool prefill_supported(const ExpertCallArgs &a) {
  return a.tiled.gate_up != nullptr && a.tiled.down != nullptr && a.G == 32 && a.H % 256 == 0 && a.I % 256 == 0;
}

int prefill_max_tiles(int n_total, int n_bins) { return n_total / kPM + n_bins + 1; }

cudaError_t launch_prefill_tiles(const GroupView &gv, int4 *ptiles, int32_t *n_ptiles, int max_tiles,
                                 cudaStream_t s) {
  cudaError_t e = launch_pdl(k_prefill_tiles, 1, 1024, 0, s, gv, ptiles, n_ptiles, max_tiles);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_prefill_gather(const ExpertCallArgs &a, const GroupView &gv, const uint16_t *x, uint16_t *dst,
                                  cudaStream_t s) {
  const int n_rows = a.n_pairs + (a.tiled.has_shared ? a.tokens : 0);
  if (a.H % 8 != 0) return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl(k_gather_rows, (n_rows + 7) / 8, 256, 0, s, gv.order, gv.offsets + gv.n_bins, n_rows,
                             a.n_pairs, a.slots, a.tokens, x, a.H, dst, device_error_word());
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_prefill_gemm(bool dual, const ExpertCallArgs &a, const GroupView &gv, const int4 *ptiles,
                                const int32_t *n_ptiles, int max_tiles, const uint16_t *in, int in_rows,
                                uint16_t *out, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(in) % 16 != 0) return cudaErrorMisalignedAddress;
  const uint16_t *tab = nullptr;
  cudaError_t e = silu_table_address(&tab);
  if (e != cudaSuccess) return e;
  CUtensorMap map;
  e = make_map(&map, in, in_rows, dual ? a.H : a.I, kPM);
  if (e != cudaSuccess) return e;
  // pairs (grouped rows) of the layer: tokens * slots routed + one per token for the shared expert
  const int n_rows = a.n_pairs + (a.tiled.has_shared ? a.tokens : 0);
  const DeviceInfo di = device_info();
  const int nt = dual ? a.I / 128 : a.H / 256;
  const int grid = std::max(1, std::min(di.sms, max_tiles * nt));
  if (dual) {
    e = cudaFuncSetAttribute(k_prefill_gemm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_prefill_gemm<true>, grid, kPThreads, kPSmem, s, a, gv, ptiles, n_ptiles, max_tiles, n_rows, map,
                   out, tab, device_error_word());
  } else {
    e = cudaFuncSetAttribute(k_prefill_gemm<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_prefill_gemm<false>, grid, kPThreads, kPSmem, s, a, gv, ptiles, n_ptiles, max_tiles, n_rows,
                   map, out, tab, device_error_word());
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace fnmoe
