// prefill.cu -- grouped expert GEMMs on tcgen05 for prefill-sized batches.
//
// For thousands of tokens per layer (a prefill chunk) the experts see ~100
// pairs each and the projections become GEMMs.  Each work item is a tile of
// up to 128 pairs of one expert bin (MMA M) times 256 output rows (MMA N):
// 128 gate + 128 up rows (interleaved in groups of 8, as in the tiled tables)
// for gate/up, 256 rows for down.  Per 64-wide k-step the CTA
//   * gathers the tile's 128 input rows (bf16 x, or the bf16 SwiGLU output
//     for down) with cp.async into a 128B-swizzled K-major shared tile,
//   * stages the 256 weight rows' packed nibbles, scales and biases from the
//     tiled tables, and dequantises them to bf16 -- bf16(s*q + b), one
//     rounding (fma.rn.bf16x2), the reference's dequant rule -- into a second
//     swizzled tile,
//   * issues 4 tcgen05.mma (kind::f16, M128 N256 K16, fp32 accumulators in
//     256 TMEM columns) from one elected thread and commits them to an
//     mbarrier; the next k-step's copies and dequant overlap the MMAs.
// The epilogue reads TMEM (tcgen05.ld 32x32b) and writes bf16 SwiGLU
// activations (gate/up) or bf16 per-slot outputs (down).  Accumulation is
// float32 in the tensor core's order, so results match the exact decode path
// within float32 rounding, not bit for bit (the reference likewise switches
// kernels for large batches).

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "async.cuh"
#include "common.cuh"
#include "moe_kernels.cuh"

namespace fnmoe {

namespace {

constexpr int kPM = 128;                 // pairs per tile (MMA M)
constexpr int kPN = 256;                 // output rows per item (MMA N)
constexpr int kPThreads = 256;
constexpr int kARing = 4, kRawRing = 3, kBRing = 2;
constexpr int kATile = kPM * 128;        // 128 rows x 64 bf16
constexpr int kBTile = kPN * 128;        // 256 rows x 64 bf16
constexpr int kRawRow = 40;              // 32 packed bytes, 2 scales, 2 biases
constexpr int kRawTile = kPN * kRawRow;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kARing * kATile;
constexpr int kOffRaw = kOffB + kBRing * kBTile;
constexpr int kOffBar = kOffRaw + kRawRing * kRawTile;
constexpr int kPSmem = kOffBar + 64 + 1024;  // + slack for the 1024-byte alignment of the tiles
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kPSpinLimit = 1u << 22;

// Instruction descriptor: kind::f16, bf16 A and B (K-major), f32 D, M 128, N 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kPN >> 3) << 17) |
                            (static_cast<uint32_t>(kPM >> 4) << 24);

// Shared-memory matrix descriptor of a 128B-swizzled K-major tile: rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void cp16s(uint32_t s, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(g));
}
__device__ __forceinline__ void cp8s(uint32_t s, const void *g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(g));
}
__device__ __forceinline__ void cp4s(uint32_t s, const void *g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(g));
}
__device__ __forceinline__ void sts128(uint32_t s, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"r"(s), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Bounded wait for the next completion of `bar` (parity tracked in `phase`).
__device__ __forceinline__ void bar_wait(uint64_t *bar, uint32_t &phase, bool &dead, uint32_t *err) {
  if (!dead) {
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, phase)) {
      if (++spins >= kPSpinLimit) {
        dead = true;
        set_error(err, kErrTimeout);
        break;
      }
    }
  }
  phase ^= 1u;
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

template <bool DUAL>
__global__ void __launch_bounds__(kPThreads, 1) k_prefill_gemm(ExpertCallArgs a, GroupView gv,
                                                               const int4 *__restrict__ ptiles,
                                                               const int32_t *__restrict__ n_ptiles,
                                                               const uint16_t *__restrict__ in,
                                                               uint16_t *__restrict__ out,
                                                               const uint16_t *__restrict__ exp_tab,
                                                               uint32_t *err) {
  extern __shared__ uint8_t psmem_raw[];
  const uint32_t raw0 = smem_u32(psmem_raw);
  const uint32_t sbase = (raw0 + 1023u) & ~1023u;
  uint8_t *sm = psmem_raw + (sbase - raw0);
  uint64_t *done = reinterpret_cast<uint64_t *>(sm + kOffBar);  // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kOffBar + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = DUAL ? a.H : a.I;
  const int O = DUAL ? a.I : a.H;
  const int NT = DUAL ? O / 128 : O / 256;
  const int KT = K / 64;
  const int nblk = K / 256;
  const uint64_t rec_bytes = DUAL ? a.tiled.gate_up_record : a.tiled.down_record;
  const uint8_t *tbase = DUAL ? a.tiled.gate_up : a.tiled.down;
  pdl_trigger();
  pdl_wait();
  const int n_items = n_ptiles[0] * NT;
  if (static_cast<int>(blockIdx.x) >= n_items) return;

  if (tid == 0) {
    mbar_init(done + 0, 1);
    mbar_init(done + 1, 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint32_t phase[2] = {0u, 0u};
  bool dead = false;

  const int r = tid >> 1, half = tid & 1;  // A gather: row r, chunks 4*half .. 4*half+3
  const int n = tid, rg = n >> 4, side = (n >> 3) & 1, rr = n & 7;  // B row n of the item

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int pt = item / NT, nt = item - pt * NT;
    const int4 d0 = ptiles[pt];
    const int start = d0.y, len = d0.z;
    uint32_t rec = 0;
    if (!record_of(a, static_cast<uint32_t>(d0.x), rec)) {
      if (tid == 0) set_error(err, kErrBadRoute);
      continue;
    }
    const uint8_t *arow = nullptr;
    if (r < len) {
      const int pair = gv.order[start + r];
      const int row = DUAL ? pair_row(pair, a.n_pairs, a.slots) : pair;
      arow = reinterpret_cast<const uint8_t *>(in + static_cast<size_t>(row) * K);
    }
    const uint8_t *brg = tbase + rec * rec_bytes + static_cast<size_t>(nt * 16 + rg) * nblk * kTileChunk;
    auto issue = [&](int kt) {
      const uint32_t as = sbase + kOffA + (kt % kARing) * kATile + r * 128;
      if (arow != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = 4 * half + q;
          cp16s(as + ((j ^ (r & 7)) << 4), arow + kt * 128 + j * 16);
        }
      }
      const int blk = kt >> 2, h = (kt & 3) >> 1, i0 = 2 * (kt & 1);
      const uint8_t *ch = brg + static_cast<size_t>(blk) * kTileChunk;
      const uint32_t rs = sbase + kOffRaw + (kt % kRawRing) * kRawTile + n * kRawRow;
#pragma unroll
      for (int c = 0; c < 4; ++c) cp8s(rs + c * 8, ch + h * 1024 + side * 512 + (rr * 4 + c) * 16 + i0 * 4);
      cp4s(rs + 32, ch + kTileW + (side * 8 + rr) * 32 + (4 * h + i0) * 2);
      cp4s(rs + 36, ch + kTileW + (side * 8 + rr) * 32 + 16 + (4 * h + i0) * 2);
      cp_async_commit();
    };

    issue(0);
    if (KT > 1) issue(1);
    else cp_async_commit();  // two groups in flight before the first step, whatever KT
    for (int kt = 0; kt < KT; ++kt) {
      if (kt >= 2) bar_wait(done + (kt & 1), phase[kt & 1], dead, err);  // MMA(kt-2) is done
      if (kt + 2 < KT) issue(kt + 2);
      else cp_async_commit();  // keep one group per step
      cp_async_wait<2>();
      __syncthreads();  // the step's input rows and raw weights landed for every thread
      {
        const uint32_t rs = sbase + kOffRaw + (kt % kRawRing) * kRawTile + n * kRawRow;
        const uint2 w01 = lds64(rs), w23 = lds64(rs + 8), w45 = lds64(rs + 16), w67 = lds64(rs + 24);
        const uint2 sbw = lds64(rs + 32);
        const uint32_t wd[4][2] = {{w01.x, w01.y}, {w23.x, w23.y}, {w45.x, w45.y}, {w67.x, w67.y}};
        const uint32_t bs = sbase + kOffB + (kt & 1) * kBTile + n * 128;
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          const uint32_t s16 = gi ? (sbw.x >> 16) : (sbw.x & 0xFFFFu);
          const uint32_t b16 = gi ? (sbw.y >> 16) : (sbw.y & 0xFFFFu);
          const uint32_t ss = s16 | (s16 << 16), bb = b16 | (b16 << 16);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 v = dequant_word(wd[c][gi], ss, bb);
            const int j = 4 * gi + c;
            sts128(bs + ((j ^ (n & 7)) << 4), v.x, v.y, v.z, v.w);
          }
        }
      }
      fence_proxy_async();  // generic-proxy tile writes (cp.async, st.shared) -> tensor-core reads
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint64_t ad = sw128_desc(sbase + kOffA + (kt % kARing) * kATile);
        const uint64_t bd = sw128_desc(sbase + kOffB + (kt & 1) * kBTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, (kt | kk) != 0 ? 1u : 0u);
        umma_commit(done + (kt & 1));
      }
    }
    // all MMAs of the item complete (the last two commits)
    if (KT >= 2) bar_wait(done + (KT & 1), phase[KT & 1], dead, err);
    bar_wait(done + ((KT - 1) & 1), phase[(KT - 1) & 1], dead, err);
    tc_fence_after();
    {
      const int lb = 32 * (warp & 3);
      const int m = lb + lane;  // pair row of the tile
      int pair = -1;
      if (m < len) pair = gv.order[start + m];
#pragma unroll 1
      for (int qq = 0; qq < 4; ++qq) {
        const int q = (warp >> 2) * 4 + qq;  // 32-column chunk
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tmem + (static_cast<uint32_t>(lb) << 16) + 32 * q, v);
        if (pair >= 0 && DUAL) {
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // columns: [gate rg=2q r0-7][up rg=2q][gate rg=2q+1][up rg=2q+1]
            const int base = (j < 4) ? 0 : 16;
            const int jj = 2 * (j & 3);
            const float g0 = round_bf16(__uint_as_float(v[base + jj])), u0 = round_bf16(__uint_as_float(v[base + 8 + jj]));
            const float g1 = round_bf16(__uint_as_float(v[base + jj + 1]));
            const float u1 = round_bf16(__uint_as_float(v[base + 8 + jj + 1]));
            o[j] = static_cast<uint32_t>(f32_to_bf16(swiglu_bf16(exp_tab, g0, u0))) |
                   (static_cast<uint32_t>(f32_to_bf16(swiglu_bf16(exp_tab, g1, u1))) << 16);
          }
          uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(pair) * O + nt * 128 + 16 * q);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else if (pair >= 0) {
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            o[j] = static_cast<uint32_t>(f32_to_bf16(__uint_as_float(v[2 * j]))) |
                   (static_cast<uint32_t>(f32_to_bf16(__uint_as_float(v[2 * j + 1]))) << 16);
          uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(pair) * O + nt * 256 + 32 * q);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM reads are done before the next item's MMAs overwrite the accumulators
    tc_fence_after();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// 128-pair tiles of every bin from the grouping counts and offsets (one CTA).
__global__ void __launch_bounds__(1024) k_prefill_tiles(GroupView gv, int4 *ptiles, int32_t *n_ptiles,
                                                        int max_tiles) {
  pdl_trigger();
  pdl_wait();
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

cudaError_t launch_prefill_gemm(bool dual, const ExpertCallArgs &a, const GroupView &gv, const int4 *ptiles,
                                const int32_t *n_ptiles, int max_tiles, const uint16_t *in, uint16_t *out,
                                cudaStream_t s) {
  const uint16_t *tab = nullptr;
  cudaError_t e = exp_table_address(&tab);
  if (e != cudaSuccess) return e;
  const DeviceInfo di = device_info();
  const int nt = dual ? a.I / 128 : a.H / 256;
  const int grid = std::max(1, std::min(di.sms, max_tiles * nt));
  if (dual) {
    e = cudaFuncSetAttribute(k_prefill_gemm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_prefill_gemm<true>, grid, kPThreads, kPSmem, s, a, gv, ptiles, n_ptiles, in, out, tab,
                   device_error_word());
    if (e != cudaSuccess) return e;
  } else {
    e = cudaFuncSetAttribute(k_prefill_gemm<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_prefill_gemm<false>, grid, kPThreads, kPSmem, s, a, gv, ptiles, n_ptiles, in, out, tab,
                   device_error_word());
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

}  // namespace fnmoe
