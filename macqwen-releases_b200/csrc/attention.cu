// attention.cu -- paged-KV decode attention for sm_100a.
//
// Semantics follow paged_attention (models/qwen27b/paged_kv.py:417-495) for
// one query token: scores in float32, online softmax with float32 running
// max / sum / weighted value sum, merged across chunks with
// exp(m_old - m) and exp(m_new - m), output o / l rounded to bfloat16.
//
// Layout: q [B, Hq, D]; K/V caches [pages, page_size, Hkv, D] (bf16);
// block_table [B, max_pages]; context_lens [B].
//
// Decomposition: one CTA per (sequence, kv head, split of `split_tokens`
// tokens).  A producer warp streams the split's K and V rows, 32 tokens per
// stage, into a ring of shared-memory stages with one bulk copy per row
// (cp.async.bulk completing on the stage's mbarrier; pages are looked up in
// the block table per row, so any page size works).  Two consumer warps each
// take 16 tokens of every stage and run tensor-core MMAs fed by ldmatrix:
//   S^T = K Q^T   (M = 16 tokens, N = 8 query heads of the GQA group, K = D)
//   O^T += V^T P^T (M = 16 head dims, N = 8 query heads, K = 16 tokens)
// with P^T moved into B-fragment order by movmatrix.  The two warps' online
// softmax states are merged in shared memory and one float32 partial
// (o, m, l) per split is written; a second kernel merges the splits of a
// sequence in split order.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "attention.cuh"
#include "async.cuh"
#include "common.cuh"
#include "moe_kernels.cuh"

namespace fnmoe {

namespace {

constexpr int kHeadsPerMma = 8;

__device__ __forceinline__ void mma_bf16_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct PagedView {
  const uint16_t *q, *k, *v;
  const int32_t *table, *ctx;
  int B, Hq, Hkv, page_size, max_pages, num_pages, split, splits_max, gq;
  float scale;
  float *part;  // [B][Hkv][splits_max][gq][D + 2]  (o[D], m, l)
};

// Shared-memory ring of k_paged_split for head dim D.  A stage holds the K
// and V rows of 32 tokens.
//  * TMA (page size and split multiples of 32): the 32 tokens of a stage lie
//    in one page, and their rows of this kv head are one 32-row box of the
//    cache viewed as [pages * page_size][Hkv * D]; the stage takes D / 64
//    boxes of 64 columns for K and as many for V (2D TMA, 128-byte swizzle:
//    16-byte chunk j of box row r sits at chunk j ^ (r & 7), so ldmatrix's
//    eight row addresses hit eight bank groups).  Boxes start 1 KiB aligned.
//  * Rows (any geometry): one bulk copy per token row into rows of 2D + 16
//    bytes: D/8 + 1 sixteen-byte chunks, odd modulo 8, which spreads the
//    eight rows of an ldmatrix phase over distinct bank groups.
template <int D, bool TMA>
struct PagedRing {
  static constexpr int kTok = 32;  // tokens per stage
  static constexpr int kStages = 3;
  static constexpr int kPitch = TMA ? 128 : 2 * D + 16;  // bytes per staged row (per box for TMA)
  static constexpr int kBoxBytes = kTok * 128;           // one 64-column box (TMA)
  static constexpr int kVOff = TMA ? (D / 64) * kBoxBytes : kTok * kPitch;
  static constexpr int kStageBytes = 2 * kVOff;
  static constexpr int kBarOff = kStages * kStageBytes;  // full[kStages], empty[kStages]
  static constexpr int kMaskOff = kBarOff + 16 * kStages;
  static constexpr int kAlign = TMA ? 1024 : 0;           // slack to align the ring to 1 KiB
  static constexpr int kSmem = kMaskOff + 4 * kStages + kAlign;
  static constexpr int kThreads = 96;  // producer warp + two consumer warps
};

constexpr uint32_t kPagedSpin = 1u << 22;  // mbarrier polls before a wait gives up

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(f32_to_bf16(lo)) | (static_cast<uint32_t>(f32_to_bf16(hi)) << 16);
}
// 2D TMA load of one box (no multicast) completing on mbarrier `bar`.
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Poll an mbarrier phase at most kPagedSpin times; false (and the timeout
// flag) when it never completes.
__device__ __forceinline__ bool paged_wait(uint64_t *bar, unsigned parity, uint32_t *err) {
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins >= kPagedSpin) {
      set_error(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// Byte offset, inside a stage's K (or V) half, of the 16 bytes at staged
// token row `row`, head dims [8 * chunk, 8 * chunk + 8).
template <int D, bool TMA>
__device__ __forceinline__ uint32_t staged_offset(int row, int chunk) {
  if (TMA) return (chunk >> 3) * PagedRing<D, TMA>::kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
  return row * PagedRing<D, TMA>::kPitch + chunk * 16;
}

template <int D, bool TMA>
__global__ void __launch_bounds__(PagedRing<D, TMA>::kThreads)
    k_paged_split(PagedView p, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  uint32_t *err) {
  using R = PagedRing<D, TMA>;
  constexpr int KT = D / 16;  // 16-wide tiles along D
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t *sm = sm_raw;
  if (TMA) sm += (1024u - (smem_u32(sm_raw) & 1023u)) & 1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_seq = p.Hkv * p.splits_max;
  const int b = blockIdx.x / per_seq;
  const int rem = blockIdx.x - b * per_seq;
  const int h = rem / p.splits_max;
  const int sp = rem - h * p.splits_max;
  const int ctx = p.ctx[b];
  const int t0 = sp * p.split;
  if (t0 >= ctx) return;
  const int t1 = min(ctx, t0 + p.split);
  const int n_st = (t1 - t0 + R::kTok - 1) / R::kTok;
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + R::kBarOff);
  uint64_t *empty = full + R::kStages;
  volatile uint32_t *mask = reinterpret_cast<volatile uint32_t *>(sm + R::kMaskOff);
  if (threadIdx.x == 0) {
    for (int s = 0; s < R::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 2);
    }
    mbar_init_fence();
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer ----
    // The block-table entry a stage needs is loaded one stage ahead, so its
    // latency overlaps the previous stage instead of delaying the copies.
    // TMA: lane 0 looks up the stage's page; rows: each lane its token's.
    auto page_of = [&](int st) -> int {
      const int t = t0 + st * R::kTok + (TMA ? 0 : lane);
      if (st >= n_st || t >= t1 || (TMA && lane != 0)) return -1;
      const int pi = t / p.page_size;
      return pi < p.max_pages ? p.table[static_cast<size_t>(b) * p.max_pages + pi] : -1;
    };
    bool dead = false;
    int page_next = page_of(0);
    for (int st = 0; st < n_st; ++st) {
      const int s = st % R::kStages;
      const int page = page_next;
      page_next = page_of(st + 1);
      if (st >= R::kStages && !dead) {
        dead = !paged_wait(empty + s, ((st / R::kStages) - 1) & 1, err);
        dead = __any_sync(0xFFFFFFFFu, dead);
      }
      const int ts = t0 + st * R::kTok;  // first token of the stage
      const bool page_ok = page >= 0 && page < p.num_pages && !dead;
      uint8_t *stg = sm + s * R::kStageBytes;
      if (TMA) {
        if (lane == 0) {
          const int n = min(R::kTok, t1 - ts);
          mask[s] = page_ok ? (n >= 32 ? 0xFFFFFFFFu : (1u << n) - 1u) : 0u;
          mbar_expect_tx(full + s, page_ok ? 4u * R::kTok * D : 0u);
          if (page_ok) {
            const int y = page * p.page_size + (ts - (ts / p.page_size) * p.page_size);
            const uint32_t bar = smem_u32(full + s);
#pragma unroll
            for (int c = 0; c < D / 64; ++c) {
              tma_box(smem_u32(stg + c * R::kBoxBytes), &kmap, h * D + 64 * c, y, bar);
              tma_box(smem_u32(stg + R::kVOff + c * R::kBoxBytes), &vmap, h * D + 64 * c, y, bar);
            }
          }
        }
        __syncwarp();
      } else {
        const uint16_t *kr = nullptr, *vr = nullptr;
        if (page_ok) {
          const int t = ts + lane;
          const int slot = t - (t / p.page_size) * p.page_size;
          const size_t row = (static_cast<size_t>(page) * p.page_size + slot) * p.Hkv + h;
          kr = p.k + row * D;
          vr = p.v + row * D;
        }
        const bool go = kr != nullptr;
        const unsigned valid = __ballot_sync(0xFFFFFFFFu, go);
        if (lane == 0) {
          mask[s] = valid;
          mbar_expect_tx(full + s, static_cast<unsigned>(__popc(valid)) * 4u * D);
        }
        __syncwarp();
        if (go) {
          bulk_g2s(stg + lane * R::kPitch, kr, 2 * D, full + s);
          bulk_g2s(stg + R::kVOff + lane * R::kPitch, vr, 2 * D, full + s);
        }
      }
    }
    // Every copy issued lands before this warp (and so the CTA) exits.
    for (int st = max(0, n_st - R::kStages); st < n_st; ++st)
      paged_wait(full + st % R::kStages, (st / R::kStages) & 1, err);
    return;
  }

  // ---- consumers: warp cw takes tokens [16 cw, 16 cw + 16) of each stage ----
  const int cw = warp - 1;
  const int g = lane >> 2, tq = lane & 3;
  // Q^T as the B operand: b0 = Q[head g][16k + 2tq, +1], b1 = Q[head g][16k + 2tq + 8, +9].
  uint32_t qb[KT][2];
  {
    const bool hv = g < p.gq;
    const uint16_t *qrow = p.q + (static_cast<size_t>(b) * p.Hq + h * p.gq + (hv ? g : 0)) * D;
#pragma unroll
    for (int k = 0; k < KT; ++k) {
      qb[k][0] = hv ? *reinterpret_cast<const uint32_t *>(qrow + 16 * k + 2 * tq) : 0u;
      qb[k][1] = hv ? *reinterpret_cast<const uint32_t *>(qrow + 16 * k + 2 * tq + 8) : 0u;
    }
  }
  float o[KT][4];
#pragma unroll
  for (int j = 0; j < KT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float mrun[2] = {-INFINITY, -INFINITY};
  float lrun[2] = {0.0f, 0.0f};
  const float sl2 = p.scale * 1.4426950408889634f;
  // ldmatrix row addresses: lane i serves row (i & 7) of matrix (i >> 3).
  // K (A operand): matrices = (tokens 0-7 | 8-15) x (dims +0 | +8);
  // V (A operand of V^T, transposed load): (dims +0 | +8) x (tokens 0-7 | 8-15).
  const int mi = lane >> 3, ri = lane & 7;
  const int k_row = 16 * cw + (mi & 1) * 8 + ri, k_half = mi >> 1;
  const int v_row = 16 * cw + (mi >> 1) * 8 + ri, v_half = mi & 1;
  const uint32_t sm_base = smem_u32(sm);
  bool dead = false;

  for (int st = 0; st < n_st; ++st) {
    const int s = st % R::kStages;
    if (!dead) {
      dead = !paged_wait(full + s, (st / R::kStages) & 1, err);
      dead = __any_sync(0xFFFFFFFFu, dead);
    }
    const uint32_t chunk = (mask[s] >> (16 * cw)) & 0xFFFFu;
    const uint32_t kst = sm_base + s * R::kStageBytes, vst = kst + R::kVOff;
    // ---- S^T = K Q^T, two accumulation chains ----
    float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k < KT; k += 2) {
      uint32_t a0[4], a1[4];
      ldsm_x4(kst + staged_offset<D, TMA>(k_row, 2 * k + k_half), a0);
      ldsm_x4(kst + staged_offset<D, TMA>(k_row, 2 * (k + 1) + k_half), a1);
      mma_bf16_16816(sa, a0[0], a0[1], a0[2], a0[3], qb[k][0], qb[k][1]);
      mma_bf16_16816(sb, a1[0], a1[1], a1[2], a1[3], qb[k + 1][0], qb[k + 1][1]);
    }
    // V^T fragments (issued before the softmax so their latency overlaps it).
    uint32_t va[KT][4];
#pragma unroll
    for (int j = 0; j < KT; ++j) ldsm_x4_t(vst + staged_offset<D, TMA>(v_row, 2 * j + v_half), va[j]);
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(empty + s)) : "memory");

    // s: (tok g, head 2tq) (tok g, head 2tq+1) (tok g+8, head 2tq) (tok g+8, head 2tq+1)
    const bool va_ok = (chunk >> g) & 1u, vb_ok = (chunk >> (g + 8)) & 1u;
    const float x0 = va_ok ? __fadd_rn(sa[0], sb[0]) * sl2 : -INFINITY;
    const float x1 = va_ok ? __fadd_rn(sa[1], sb[1]) * sl2 : -INFINITY;
    const float x2 = vb_ok ? __fadd_rn(sa[2], sb[2]) * sl2 : -INFINITY;
    const float x3 = vb_ok ? __fadd_rn(sa[3], sb[3]) * sl2 : -INFINITY;
    float cm0 = fmaxf(x0, x2), cm1 = fmaxf(x1, x3);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      cm0 = fmaxf(cm0, __shfl_xor_sync(0xFFFFFFFFu, cm0, off));
      cm1 = fmaxf(cm1, __shfl_xor_sync(0xFFFFFFFFu, cm1, off));
    }
    const float mn0 = fmaxf(mrun[0], cm0), mn1 = fmaxf(mrun[1], cm1);
    // A chunk with no valid token keeps -inf; a finite reference keeps
    // exp2 away from -inf - -inf.
    const float r0 = (mn0 == -INFINITY) ? 0.0f : mn0, r1 = (mn1 == -INFINITY) ? 0.0f : mn1;
    const float al0 = exp2f(mrun[0] - r0), al1 = exp2f(mrun[1] - r1);
    const float p0 = exp2f(x0 - r0), p1 = exp2f(x1 - r1);
    const float p2 = exp2f(x2 - r0), p3 = exp2f(x3 - r1);
    float ls0 = p0 + p2, ls1 = p1 + p3;
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      ls0 += __shfl_xor_sync(0xFFFFFFFFu, ls0, off);
      ls1 += __shfl_xor_sync(0xFFFFFFFFu, ls1, off);
    }
    lrun[0] = lrun[0] * al0 + ls0;
    lrun[1] = lrun[1] * al1 + ls1;
    mrun[0] = mn0;
    mrun[1] = mn1;
    // Rescale only when some running max moved (multiplying by 1 is exact).
    if (__any_sync(0xFFFFFFFFu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
      for (int j = 0; j < KT; ++j) {
        o[j][0] *= al0;
        o[j][1] *= al1;
        o[j][2] *= al0;
        o[j][3] *= al1;
      }
    }
    // P^T in B-fragment order: b0 = P[head g][tok 2tq, 2tq+1], b1 = tokens + 8.
    const uint32_t pb0 = movm_t(pack_bf16x2(p0, p1));
    const uint32_t pb1 = movm_t(pack_bf16x2(p2, p3));
    // Rows of tokens that were not loaded hold stale or uninitialised bytes:
    // zero them so that 0 * (inf or nan) never enters the sum.
    if (chunk != 0xFFFFu) {
      const uint32_t m01 = (((chunk >> (2 * tq)) & 1u) ? 0x0000FFFFu : 0u) |
                           (((chunk >> (2 * tq + 1)) & 1u) ? 0xFFFF0000u : 0u);
      const uint32_t m89 = (((chunk >> (2 * tq + 8)) & 1u) ? 0x0000FFFFu : 0u) |
                           (((chunk >> (2 * tq + 9)) & 1u) ? 0xFFFF0000u : 0u);
#pragma unroll
      for (int j = 0; j < KT; ++j) {
        va[j][0] &= m01;
        va[j][1] &= m01;
        va[j][2] &= m89;
        va[j][3] &= m89;
      }
    }
    // ---- O^T += V^T P^T ----
#pragma unroll
    for (int j = 0; j < KT; ++j) mma_bf16_16816(o[j], va[j][0], va[j][1], va[j][2], va[j][3], pb0, pb1);
  }

  // ---- merge the two consumer warps (through stage 0, idle by now) ----
  float *mb = reinterpret_cast<float *>(sm);
  asm volatile("bar.sync 1, 64;\n" ::: "memory");
  if (cw == 1) {
#pragma unroll
    for (int j = 0; j < KT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) mb[(4 * j + e) * 32 + lane] = o[j][e];
    mb[(4 * KT + 0) * 32 + lane] = mrun[0];
    mb[(4 * KT + 1) * 32 + lane] = mrun[1];
    mb[(4 * KT + 2) * 32 + lane] = lrun[0];
    mb[(4 * KT + 3) * 32 + lane] = lrun[1];
  }
  asm volatile("bar.sync 1, 64;\n" ::: "memory");
  if (cw == 1) return;
  float w0[2], w1[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float m2 = mb[(4 * KT + hh) * 32 + lane];
    const float l2 = mb[(4 * KT + 2 + hh) * 32 + lane];
    const float mm = fmaxf(mrun[hh], m2);
    const float ref = (mm == -INFINITY) ? 0.0f : mm;
    w0[hh] = exp2f(mrun[hh] - ref);
    w1[hh] = exp2f(m2 - ref);
    lrun[hh] = lrun[hh] * w0[hh] + l2 * w1[hh];
    mrun[hh] = mm;
  }
#pragma unroll
  for (int j = 0; j < KT; ++j) {
    o[j][0] = o[j][0] * w0[0] + mb[(4 * j + 0) * 32 + lane] * w1[0];
    o[j][1] = o[j][1] * w0[1] + mb[(4 * j + 1) * 32 + lane] * w1[1];
    o[j][2] = o[j][2] * w0[0] + mb[(4 * j + 2) * 32 + lane] * w1[0];
    o[j][3] = o[j][3] * w0[1] + mb[(4 * j + 3) * 32 + lane] * w1[1];
  }
  // o[j]: c0 (dim 16j+g, head 2tq) c1 (dim 16j+g, head 2tq+1) c2/c3 the same at dim 16j+g+8.
  const size_t seq_base = ((static_cast<size_t>(b) * p.Hkv + h) * p.splits_max + sp) * p.gq;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int head = 2 * tq + hh;
    if (head >= p.gq) continue;
    float *dst = p.part + (seq_base + head) * (D + 2);
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      dst[16 * j + g] = o[j][hh];
      dst[16 * j + g + 8] = o[j][2 + hh];
    }
    if (g == 0) {
      dst[D] = mrun[hh];
      dst[D + 1] = lrun[hh];
    }
  }
}

// Block-wide reduction over D threads (D / 32 warps); every thread gets the result.
template <int D, bool MAX>
__device__ __forceinline__ float block_reduce(float v, float *red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float o = __shfl_xor_sync(0xFFFFFFFFu, v, off);
    v = MAX ? fmaxf(v, o) : v + o;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < D / 32; ++w) v = MAX ? fmaxf(v, red[w]) : v + red[w];
  return v;
}

constexpr int kMergeChunk = 1024;  // split weights staged in shared memory per pass

// One CTA per (sequence, query head), one thread per head dim: the splits'
// running maxima give the common reference m, each split's weight
// exp2(m_s - m) is staged once in shared memory, and every thread sums its
// dimension over the splits with independent loads.
template <int D>
__global__ void __launch_bounds__(D) k_paged_merge(PagedView p, uint16_t *__restrict__ out) {
  __shared__ float red[D / 32];
  __shared__ float wsh[kMergeChunk];
  const int bh = blockIdx.x;  // b * Hq + head
  const int b = bh / p.Hq, head = bh - b * p.Hq;
  const int h = head / p.gq, hq = head - h * p.gq;
  const int d = threadIdx.x;
  const int ctx = p.ctx[b];
  const int ns = ctx > 0 ? (ctx + p.split - 1) / p.split : 0;
  const size_t sstride = static_cast<size_t>(p.gq) * (D + 2);
  const float *base = p.part + ((static_cast<size_t>(b) * p.Hkv + h) * p.splits_max * p.gq + hq) * (D + 2);
  float m = -INFINITY;
  for (int s = d; s < ns; s += D) m = fmaxf(m, base[s * sstride + D]);
  m = block_reduce<D, true>(m, red);
  float L = 0.0f, O = 0.0f;
  for (int c0 = 0; c0 < ns; c0 += kMergeChunk) {
    const int cn = min(kMergeChunk, ns - c0);
    float lp = 0.0f;
    for (int i = d; i < cn; i += D) {
      const float *src = base + (c0 + i) * sstride;
      const float ms = src[D];
      const float w = (ms == -INFINITY) ? 0.0f : exp2f(ms - m);
      wsh[i] = w;
      lp += src[D + 1] * w;
    }
    L += block_reduce<D, false>(lp, red);  // its barriers also publish wsh
    const float *col = base + c0 * sstride + d;
#pragma unroll 8
    for (int i = 0; i < cn; ++i) O += col[i * sstride] * wsh[i];
    __syncthreads();  // wsh is rewritten by the next pass
  }
  const float val = (ns > 0 && L > 0.0f) ? O / L : 0.0f;
  out[(static_cast<size_t>(b) * p.Hq + head) * D + d] = f32_to_bf16(val);
}

int check(const FnPagedArgs *a, std::string &err) {
  if (a == nullptr) { err = "args is NULL"; return FNMOE_ERR_NULL; }
  if (a->abi_version != FNMOE_ABI_VERSION) { err = "abi_version mismatch"; return FNMOE_ERR_ABI; }
  if (!a->q || !a->k_cache || !a->v_cache || !a->block_table || !a->context_lens || !a->out) {
    err = "q, k_cache, v_cache, block_table, context_lens and out are required";
    return FNMOE_ERR_NULL;
  }
  if (a->batch == 0 || a->q_heads == 0 || a->kv_heads == 0 || a->page_size == 0 || a->max_pages == 0 ||
      a->num_pages == 0) {
    err = "empty attention shape";
    return FNMOE_ERR_SHAPE;
  }
  if (a->q_heads % a->kv_heads) { err = "q_heads must be a multiple of kv_heads"; return FNMOE_ERR_SHAPE; }
  if (a->q_heads / a->kv_heads > kHeadsPerMma) { err = "at most 8 query heads per kv head"; return FNMOE_ERR_UNSUPPORTED; }
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) {
    err = "head_dim must be 64, 128 or 256";
    return FNMOE_ERR_UNSUPPORTED;
  }
  if (a->split_tokens == 0 || a->split_tokens % 16) { err = "split_tokens must be a positive multiple of 16"; return FNMOE_ERR_SHAPE; }
  // K/V rows move by bulk copies and q by 4-byte loads: 16-byte alignment.
  if ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k_cache) |
       reinterpret_cast<uintptr_t>(a->v_cache)) & 15u) {
    err = "q, k_cache and v_cache must be 16-byte aligned";
    return FNMOE_ERR_VALUE;
  }
  return FNMOE_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn paged_encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// A cache as a bf16 matrix [pages * page_size][Hkv * D]: 64-column x
// 32-row boxes, 128-byte swizzle.
bool make_cache_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols) {
  EncodeTiledFn fn = paged_encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, 32};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool TMA>
cudaError_t launch_split(const PagedView &p, const CUtensorMap &km, const CUtensorMap &vm, unsigned blocks,
                         uint32_t *derr, cudaStream_t s) {
  using R = PagedRing<D, TMA>;
  static const cudaError_t attr =
      cudaFuncSetAttribute(k_paged_split<D, TMA>, cudaFuncAttributeMaxDynamicSharedMemorySize, R::kSmem);
  if (attr != cudaSuccess) return attr;
  k_paged_split<D, TMA><<<blocks, R::kThreads, R::kSmem, s>>>(p, km, vm, derr);
  return cudaSuccess;
}

template <int D>
cudaError_t launch_paged(const PagedView &p, const FnPagedArgs *a, unsigned blocks, uint16_t *out, uint32_t *derr,
                         cudaStream_t s) {
  // TMA boxes need every 32-token stage inside one page.
  const bool tma = p.page_size % 32 == 0 && p.split % 32 == 0;
  CUtensorMap km{}, vm{};
  cudaError_t e;
  if (tma) {
    const uint64_t rows = static_cast<uint64_t>(p.num_pages) * p.page_size;
    const uint64_t cols = static_cast<uint64_t>(p.Hkv) * D;
    if (!make_cache_map(&km, a->k_cache, rows, cols) || !make_cache_map(&vm, a->v_cache, rows, cols))
      return cudaErrorInvalidValue;
    e = launch_split<D, true>(p, km, vm, blocks, derr, s);
  } else {
    e = launch_split<D, false>(p, km, vm, blocks, derr, s);
  }
  if (e != cudaSuccess) return e;
  k_paged_merge<D><<<p.B * p.Hq, D, 0, s>>>(p, out);
  return cudaSuccess;
}

uint64_t part_bytes(const FnPagedArgs *a) {
  const uint64_t max_tokens = static_cast<uint64_t>(a->max_pages) * a->page_size;
  const uint64_t splits = (max_tokens + a->split_tokens - 1) / a->split_tokens;
  const uint64_t gq = a->q_heads / a->kv_heads;
  return static_cast<uint64_t>(a->batch) * a->kv_heads * splits * gq * (a->head_dim + 2) * sizeof(float);
}

}  // namespace

int paged_workspace_size(const FnPagedArgs *a, uint64_t *bytes, std::string &err) {
  if (bytes == nullptr) { err = "bytes is NULL"; return FNMOE_ERR_NULL; }
  const int c = check(a, err);
  if (c != FNMOE_OK) return c;
  *bytes = part_bytes(a);
  return FNMOE_OK;
}

int paged_decode(const FnPagedArgs *a, cudaStream_t s, std::string &err) {
  const int c = check(a, err);
  if (c != FNMOE_OK) return c;
  const uint64_t need = part_bytes(a);
  if (a->workspace == nullptr || a->workspace_bytes < need) {
    err = "workspace needs " + std::to_string(need) + " bytes";
    return FNMOE_ERR_WORKSPACE;
  }
  PagedView p{};
  p.q = static_cast<const uint16_t *>(a->q);
  p.k = static_cast<const uint16_t *>(a->k_cache);
  p.v = static_cast<const uint16_t *>(a->v_cache);
  p.table = a->block_table;
  p.ctx = a->context_lens;
  p.B = a->batch;
  p.Hq = a->q_heads;
  p.Hkv = a->kv_heads;
  p.page_size = a->page_size;
  p.max_pages = a->max_pages;
  p.num_pages = a->num_pages;
  p.split = a->split_tokens;
  p.splits_max = static_cast<int>((static_cast<uint64_t>(a->max_pages) * a->page_size + a->split_tokens - 1) / a->split_tokens);
  p.gq = a->q_heads / a->kv_heads;
  p.scale = a->scale;
  p.part = static_cast<float *>(a->workspace);
  const uint64_t ctas = static_cast<uint64_t>(p.B) * p.Hkv * p.splits_max;
  if (ctas > 0x7FFFFFFFull) { err = "too many (sequence, kv head, split) items"; return FNMOE_ERR_SHAPE; }
  const unsigned blocks = static_cast<unsigned>(ctas);
  uint32_t *derr = device_error_word();
  cudaError_t e = cudaSuccess;
  switch (a->head_dim) {
    case 64:
      e = launch_paged<64>(p, a, blocks, static_cast<uint16_t *>(a->out), derr, s);
      break;
    case 128:
      e = launch_paged<128>(p, a, blocks, static_cast<uint16_t *>(a->out), derr, s);
      break;
    default:
      e = launch_paged<256>(p, a, blocks, static_cast<uint16_t *>(a->out), derr, s);
      break;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("paged decode: ") + cudaGetErrorString(e);
    return FNMOE_ERR_LAUNCH;
  }
  return FNMOE_OK;
}

}  // namespace fnmoe
