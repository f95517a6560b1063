// moe_kernels.cu -- sm_100a kernels of the Flash-Next sparse-MoE decode path.
//
// Pipeline of one executor call (metal_runtime.py:764-932 semantics):
//   prep_rows(x)      bf16 activations -> block fixed point, two fp16 limbs
//   group             stable counting sort of (token, slot) pairs by expert
//   gate_up           grouped Q4 gate+up projections + bf16 SwiGLU epilogue
//   prep_rows(act)    limbs of the SwiGLU output
//   down              grouped Q4 down projection (per-slot bf16 rows)
//   combine           slot-ordered fp32 combine + shared epilogue
//
// Exactness: each Q4 group dot product sum_i X_i*q_i is formed from two
// 12-bit limbs of the fixed-point activations and the 4-bit codes on the
// tensor cores (m16n8k16 fp16 -> fp32).  Every operand and partial sum is an
// integer below 2^21, so the accumulation is exact and order-free; the
// epilogue rounds exactly where the CPU oracle does (oracle/moe.py).
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <mutex>

#include "common.cuh"
#include "moe_kernels.cuh"

namespace fnmoe {

__device__ uint16_t g_exp_bf16[65536];
__device__ uint32_t g_device_errors;

// ---------------------------------------------------------------------------
// init: exp table
// ---------------------------------------------------------------------------

__global__ void k_init_exp_table() {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536) return;
  const float v = bf16_to_f32(static_cast<uint16_t>(i));
  g_exp_bf16[i] = f64_to_bf16_once(exp(static_cast<double>(v)));
}

namespace {
std::mutex g_init_mutex;
bool g_exp_ready[64] = {false};
int g_sms[64] = {0};
}  // namespace

DeviceInfo device_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return {dev, 148};
  std::lock_guard<std::mutex> lock(g_init_mutex);
  if (g_sms[dev] == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = sms > 0 ? sms : 148;
  }
  return {dev, g_sms[dev]};
}

cudaError_t ensure_exp_table(cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_init_mutex);
  if (g_exp_ready[dev]) return cudaSuccess;
  k_init_exp_table<<<256, 256, 0, stream>>>();
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return e;
  g_exp_ready[dev] = true;
  return cudaSuccess;
}

uint32_t *device_error_word() {
  void *p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_errors) != cudaSuccess) return nullptr;
  return static_cast<uint32_t *>(p);
}

// ---------------------------------------------------------------------------
// prep_rows: block fixed point of bf16 rows, fp16 limbs in fragment order
// ---------------------------------------------------------------------------

constexpr int kNoExp = -100000;

template <int G>
__global__ void __launch_bounds__(256) k_prep_rows(const uint16_t *__restrict__ rows,
                                                   int n_rows, int K,
                                                   uint16_t *__restrict__ limbs,
                                                   float4 *__restrict__ meta,
                                                   uint32_t *err) {
  constexpr int PER = G / 32;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int Gc = K / G;
  if (gw >= n_rows * Gc) return;
  const int row = gw / Gc;
  const int g = gw - row * Gc;
  const uint16_t *src = rows + static_cast<size_t>(row) * K + static_cast<size_t>(g) * G;
  uint32_t xb[PER];
  int ex[PER];
  int emax = kNoExp;
  bool bad = false;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    xb[p] = src[p * 32 + lane];
    const uint32_t ef = (xb[p] >> 7) & 0xFFu;
    const uint32_t mf = xb[p] & 0x7Fu;
    int e;
    if ((xb[p] & 0x7FFFu) == 0) {
      e = kNoExp;
    } else if (ef == 0) {
      e = (31 - __clz(static_cast<int>(mf))) - 133;
    } else if (ef == 255) {
      e = 128;
      bad = true;
    } else {
      e = static_cast<int>(ef) - 127;
    }
    ex[p] = e;
    emax = max(emax, e);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) emax = max(emax, __shfl_xor_sync(0xFFFFFFFFu, emax, off));
  if (emax == kNoExp) emax = 0;
  if (bad) set_error(err, kErrNonFinite);
  int sx = 0;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    int X = 0;
    if (ex[p] != kNoExp && !(((xb[p] >> 7) & 0xFFu) == 255u)) {
      const uint32_t ef = (xb[p] >> 7) & 0xFFu;
      const uint32_t mf = xb[p] & 0x7Fu;
      const uint32_t M = ef ? (mf | 0x80u) : mf;
      const int sh = ef ? (static_cast<int>(ef) - 112 - emax) : (-111 - emax);
      uint32_t mag;
      if (sh >= 0) mag = M << sh;
      else mag = (-sh >= 31) ? 0u : (M >> (-sh));
      X = (xb[p] & 0x8000u) ? -static_cast<int>(mag) : static_cast<int>(mag);
    }
    sx += X;
    const int l1 = ((X + 2048) & 4095) - 2048;
    const int l0 = (X - l1) >> 12;
    const int i = p * 32 + lane;
    const int i32 = i & 31;
    const int pos = (i >> 5) * 32 + (i32 >> 3) * 8 + ((i32 & 7) & 3) * 2 + ((i32 & 7) >> 2);
    const size_t base = (static_cast<size_t>(row) * Gc + g) * 2 * G;
    limbs[base + pos] = __half_as_ushort(__int2half_rn(l0));
    limbs[base + G + pos] = __half_as_ushort(__int2half_rn(l1));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) sx += __shfl_xor_sync(0xFFFFFFFFu, sx, off);
  if (lane == 0) {
    const int k = emax - 22;
    const float scale = (k >= -126) ? __int_as_float((k + 127) << 23) : 0.0f;
    meta[static_cast<size_t>(row) * Gc + g] =
        make_float4(__int2float_rn(sx), scale, static_cast<float>(k), 0.0f);
  }
}

cudaError_t launch_prep_rows(const uint16_t *rows, int n_rows, int K, int G,
                             uint16_t *limbs, float4 *meta, cudaStream_t s) {
  const long long warps = static_cast<long long>(n_rows) * (K / G);
  if (warps <= 0) return cudaSuccess;
  const int blocks = static_cast<int>((warps + 7) / 8);
  uint32_t *err = device_error_word();
  if (G == 32)
    k_prep_rows<32><<<blocks, 256, 0, s>>>(rows, n_rows, K, limbs, meta, err);
  else
    k_prep_rows<64><<<blocks, 256, 0, s>>>(rows, n_rows, K, limbs, meta, err);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// group: stable counting sort of pairs by expert bin (one CTA)
// ---------------------------------------------------------------------------

__device__ __forceinline__ int block_exclusive_scan_1024(int v, int *warp_sums, int *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_sums[lane];
    int winc = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, winc, off);
      if (lane >= off) winc += n;
    }
    warp_sums[lane] = winc - w;
    if (lane == 31) *total = winc;
  }
  __syncthreads();
  const int r = incl - v + warp_sums[warp];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int bin_of_pair(const uint32_t *routes, int i, int n_pairs,
                                           int E_arr, int records, int n_bins) {
  if (i >= n_pairs) return n_bins - 1;  // shared expert bin
  const uint32_t r = routes[i];
  if (r & kSlotBit) {
    const uint32_t slot = r & 0x7FFFFFFFu;
    return slot < static_cast<uint32_t>(records) ? E_arr + static_cast<int>(slot) : -1;
  }
  return r < static_cast<uint32_t>(E_arr) ? static_cast<int>(r) : -1;
}

__global__ void __launch_bounds__(1024) k_group(const uint32_t *__restrict__ routes, int n_pairs,
                                                int shared_tokens, int E_arr, int records,
                                                GroupView gv, uint32_t *err) {
  extern __shared__ int sm[];
  int *cnt = sm;                 // [n_bins]
  int *run = sm + gv.n_bins;     // [n_bins]
  __shared__ int warp_sums[32];
  __shared__ int total_pairs, total_tiles;
  const int tid = threadIdx.x;
  const int n_bins = gv.n_bins;
  const int n_total = n_pairs + shared_tokens;
  for (int b = tid; b < n_bins; b += blockDim.x) {
    cnt[b] = 0;
    run[b] = 0;
  }
  __syncthreads();
  for (int i = tid; i < n_total; i += blockDim.x) {
    const int b = bin_of_pair(routes, i, n_pairs, E_arr, records, n_bins);
    if (b >= 0) atomicAdd(&cnt[b], 1);
    else set_error(err, kErrBadRoute);
  }
  __syncthreads();
  // Exclusive scans of counts and tile counts over contiguous bin segments.
  const int per = (n_bins + 1023) / 1024;
  const int b0 = min(tid * per, n_bins), b1 = min(b0 + per, n_bins);
  int local_c = 0, local_t = 0;
  for (int b = b0; b < b1; ++b) {
    local_c += cnt[b];
    local_t += (cnt[b] + kTokPerItem - 1) / kTokPerItem;
  }
  int pre_c = block_exclusive_scan_1024(local_c, warp_sums, &total_pairs);
  int pre_t = block_exclusive_scan_1024(local_t, warp_sums, &total_tiles);
  for (int b = b0; b < b1; ++b) {
    const int c = cnt[b];
    gv.counts[b] = c;
    gv.offsets[b] = pre_c;
    gv.bin_key[b] = (b < E_arr) ? static_cast<uint32_t>(b)
                    : (b < E_arr + records) ? (kSlotBit | static_cast<uint32_t>(b - E_arr))
                                            : kSharedKey;
    const int nt = (c + kTokPerItem - 1) / kTokPerItem;
    for (int t = 0; t < nt && pre_t + t < gv.max_tiles; ++t) {
      gv.tiles[pre_t + t] = make_int4(b, pre_c + t * kTokPerItem, min(kTokPerItem, c - t * kTokPerItem), 0);
    }
    run[b] = pre_c;  // running write position
    pre_c += c;
    pre_t += nt;
  }
  __syncthreads();
  if (tid == 0) {
    gv.offsets[n_bins] = total_pairs;
    gv.n_tiles[0] = min(total_tiles, gv.max_tiles);
  }
  // Stable scatter: warp 0 walks pairs in index order, 32 at a time.
  if (tid < 32) {
    const int lane = tid;
    const unsigned lt = (1u << lane) - 1u;
    for (int base = 0; base < n_total; base += 32) {
      const int i = base + lane;
      const int b = (i < n_total) ? bin_of_pair(routes, i, n_pairs, E_arr, records, n_bins) : -2;
      const unsigned m = __match_any_sync(0xFFFFFFFFu, b);
      const int rank = __popc(m & lt);
      int pos = 0;
      if (b >= 0) pos = run[b] + rank;
      __syncwarp();
      if (b >= 0) {
        gv.order[pos] = i;
        if ((m >> lane) == 1u) run[b] += __popc(m);  // highest lane of the group
      }
      __syncwarp();
    }
  }
}

cudaError_t launch_group(const uint32_t *routes, int n_pairs, int shared_tokens,
                         int array_experts, int table_records, GroupView gv,
                         cudaStream_t s) {
  const size_t smem = static_cast<size_t>(gv.n_bins) * 2 * sizeof(int);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_group, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  k_group<<<1, 1024, smem, s>>>(routes, n_pairs, shared_tokens, array_experts, table_records,
                                gv, device_error_word());
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// expert pointer resolution
// ---------------------------------------------------------------------------

struct Ptrs {
  const uint32_t *w;
  const uint16_t *s;
  const uint16_t *b;
};

// part: 0 gate, 1 up, 2 down.  rows/cols of the projection matrix.
__device__ __forceinline__ bool resolve(const ExpertCallArgs &a, uint32_t key, int part,
                                        int rows, int cols, Ptrs &p) {
  if (key == kSharedKey) {
    const ProjArrays &pa = part == 0 ? a.sh_gate : (part == 1 ? a.sh_up : a.sh_down);
    p = {pa.w, pa.s, pa.b};
    return pa.w != nullptr;
  }
  if (key & kSlotBit) {
    const uint32_t slot = key & 0x7FFFFFFFu;
    if (a.table.base == nullptr || slot >= a.table.records) return false;
    const uint8_t *rec = a.table.base + a.table.header + static_cast<uint64_t>(slot) * a.table.stride;
    p.w = reinterpret_cast<const uint32_t *>(rec + a.table.off[3 * part + 0]);
    p.s = reinterpret_cast<const uint16_t *>(rec + a.table.off[3 * part + 1]);
    p.b = reinterpret_cast<const uint16_t *>(rec + a.table.off[3 * part + 2]);
    return true;
  }
  if (a.stream.base != nullptr) {
    if (key >= a.stream.records) return false;
    const uint8_t *rec = a.stream.base + a.stream.header + static_cast<uint64_t>(key) * a.stream.stride;
    p.w = reinterpret_cast<const uint32_t *>(rec + a.stream.off[3 * part + 0]);
    p.s = reinterpret_cast<const uint16_t *>(rec + a.stream.off[3 * part + 1]);
    p.b = reinterpret_cast<const uint16_t *>(rec + a.stream.off[3 * part + 2]);
    return true;
  }
  const ProjArrays &pa = part == 0 ? a.gate : (part == 1 ? a.up : a.down);
  if (pa.w == nullptr || key >= static_cast<uint32_t>(a.array_experts)) return false;
  const size_t wstride = static_cast<size_t>(rows) * (cols / 8);
  const size_t mstride = static_cast<size_t>(rows) * (cols / a.G);
  p.w = pa.w + key * wstride;
  p.s = pa.s + key * mstride;
  p.b = pa.b + key * mstride;
  return true;
}

__device__ __forceinline__ int token_of_pair(int pair, int n_pairs, int slots) {
  return pair < n_pairs ? pair / slots : pair - n_pairs;
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU
// ---------------------------------------------------------------------------
// CTA = WR row-warps x 4 chain-warps.  A row-warp owns 8 intermediate rows;
// its MMA A operand stacks 8 gate rows (M 0-7) over the same 8 up rows
// (M 8-15).  B = fixed-point limbs of 4 tokens (N = 2 limbs x 4 tokens), so
// thread (r, c) ends up holding gate and up results of row r, token c.

template <int G, int WR>
__global__ void __launch_bounds__(WR * 128) k_gate_up(ExpertCallArgs a, GroupView gv,
                                                      const uint16_t *__restrict__ xl,
                                                      const float4 *__restrict__ xm,
                                                      uint16_t *__restrict__ act,
                                                      uint16_t *__restrict__ g_out,
                                                      uint16_t *__restrict__ u_out,
                                                      uint32_t *err) {
  constexpr int WPG = G / 8;     // packed words per group per row
  constexpr int WB = G / 32;     // 32-value word blocks per group
  constexpr int KSTEPS = G / 16;
  constexpr int ROWS = 8 * WR;
  constexpr int MT = kTokPerItem / 4;
  extern __shared__ float part[];  // [WR][4][16][kTokPerItem]
  const int H = a.H, I = a.I;
  const int Gh = H / G;
  const int P = chain_count(Gh);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wr = warp >> 2, ch = warp & 3;
  const int r = lane >> 2, c = lane & 3;
  const int row_tiles = (I + ROWS - 1) / ROWS;
  const int n_items = gv.n_tiles[0] * row_tiles;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int tile = item / row_tiles, rt = item - tile * row_tiles;
    const int4 td = gv.tiles[tile];
    const int start = td.y, len = td.z;
    const uint32_t key = gv.bin_key[td.x];
    Ptrs pg, pu;
    const bool ok = resolve(a, key, 0, I, H, pg) && resolve(a, key, 1, I, H, pu);
    if (!ok && threadIdx.x == 0) set_error(err, kErrBadRoute);
    if (ok && ch < P) {
      const int o = rt * ROWS + wr * 8 + r;
      const bool row_ok = o < I;
      const int oc = row_ok ? o : 0;
      const int nmt = (len + 3) >> 2;
      int tokB[MT], tokE[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int qb = 4 * mt + (r >> 1);
        const int qe = 4 * mt + c;
        tokB[mt] = (qb < len) ? token_of_pair(gv.order[start + qb], a.n_pairs, a.slots) : -1;
        tokE[mt] = (qe < len) ? token_of_pair(gv.order[start + qe], a.n_pairs, a.slots) : -1;
      }
      float acc[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = -0.0f;
      const uint32_t *wg_row = pg.w + static_cast<size_t>(oc) * (H / 8);
      const uint32_t *wu_row = pu.w + static_cast<size_t>(oc) * (H / 8);
      const uint16_t *sg_row = pg.s + static_cast<size_t>(oc) * Gh;
      const uint16_t *bg_row = pg.b + static_cast<size_t>(oc) * Gh;
      const uint16_t *su_row = pu.s + static_cast<size_t>(oc) * Gh;
      const uint16_t *bu_row = pu.b + static_cast<size_t>(oc) * Gh;
      const int g0 = chain_begin(ch, P, Gh), g1 = chain_begin(ch + 1, P, Gh);
      for (int g = g0; g < g1; ++g) {
        uint32_t wg[WB], wu[WB];
#pragma unroll
        for (int wb = 0; wb < WB; ++wb) {
          wg[wb] = row_ok ? ldg_u32(wg_row + g * WPG + wb * 4 + c) : 0u;
          wu[wb] = row_ok ? ldg_u32(wu_row + g * WPG + wb * 4 + c) : 0u;
        }
        const float sg = row_ok ? bf16_to_f32(ldg_u16(sg_row + g)) : 0.0f;
        const float bg = row_ok ? bf16_to_f32(ldg_u16(bg_row + g)) : 0.0f;
        const float su = row_ok ? bf16_to_f32(ldg_u16(su_row + g)) : 0.0f;
        const float bu = row_ok ? bf16_to_f32(ldg_u16(bu_row + g)) : 0.0f;
        uint32_t A[KSTEPS][4];
#pragma unroll
        for (int st = 0; st < KSTEPS; ++st) {
          const int wb = st >> 1, j = (st & 1) * 2;
          A[st][0] = nibble_pair(wg[wb], j);
          A[st][1] = nibble_pair(wu[wb], j);
          A[st][2] = nibble_pair(wg[wb], j + 1);
          A[st][3] = nibble_pair(wu[wb], j + 1);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (mt < nmt) {
            float C[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint4 v[WB];
            if (tokB[mt] >= 0) {
              const uint16_t *base = xl + (static_cast<size_t>(tokB[mt]) * Gh + g) * 2 * G + (r & 1) * G;
#pragma unroll
              for (int wb = 0; wb < WB; ++wb)
                v[wb] = ldg_u128(reinterpret_cast<const uint4 *>(base + wb * 32 + c * 8));
            } else {
#pragma unroll
              for (int wb = 0; wb < WB; ++wb) v[wb] = make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int st = 0; st < KSTEPS; ++st) {
              const uint4 &vv = v[st >> 1];
              if (st & 1) mma_16816(C, A[st], vv.z, vv.w);
              else mma_16816(C, A[st], vv.x, vv.y);
            }
            if (tokE[mt] >= 0) {
              const float4 m = xm[static_cast<size_t>(tokE[mt]) * Gh + g];
              const int k = static_cast<int>(m.z);
              const float Sg = __fmaf_rn(C[0], 4096.0f, C[1]);
              const float tg = __fadd_rn(__fmul_rn(sg, Sg), __fmul_rn(bg, m.x));
              acc[mt][0] = __fadd_rn(acc[mt][0], scale_pow2(tg, m.y, k));
              const float Su = __fmaf_rn(C[2], 4096.0f, C[3]);
              const float tu = __fadd_rn(__fmul_rn(su, Su), __fmul_rn(bu, m.x));
              acc[mt][1] = __fadd_rn(acc[mt][1], scale_pow2(tu, m.y, k));
            }
          }
        }
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int qe = 4 * mt + c;
        if (qe < len) {
          part[((wr * 4 + ch) * 16 + r) * kTokPerItem + qe] = acc[mt][0];
          part[((wr * 4 + ch) * 16 + r + 8) * kTokPerItem + qe] = acc[mt][1];
        }
      }
    }
    __syncthreads();
    if (ok) {
      for (int idx = threadIdx.x; idx < len * ROWS; idx += blockDim.x) {
        const int q = idx / ROWS, ol = idx - q * ROWS;
        const int o = rt * ROWS + ol;
        if (o >= I) continue;
        const int wr2 = ol >> 3, r2 = ol & 7;
        float cg[4] = {-0.0f, -0.0f, -0.0f, -0.0f}, cu[4] = {-0.0f, -0.0f, -0.0f, -0.0f};
        for (int k = 0; k < P; ++k) {
          cg[k] = part[((wr2 * 4 + k) * 16 + r2) * kTokPerItem + q];
          cu[k] = part[((wr2 * 4 + k) * 16 + r2 + 8) * kTokPerItem + q];
        }
        const float gvv = round_bf16(chain_tree(cg, P));
        const float uvv = round_bf16(chain_tree(cu, P));
        const float av = swiglu_bf16(g_exp_bf16, gvv, uvv);
        const int pair = gv.order[start + q];
        act[static_cast<size_t>(pair) * I + o] = f32_to_bf16(av);
        if (g_out != nullptr && pair < a.n_pairs) {
          g_out[static_cast<size_t>(pair) * I + o] = f32_to_bf16(gvv);
          u_out[static_cast<size_t>(pair) * I + o] = f32_to_bf16(uvv);
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// down projection
// ---------------------------------------------------------------------------
// CTA = WR row-warps x 4 chain-warps; a row-warp owns 16 hidden rows
// (M 0-7 = rows r, M 8-15 = rows r+8).  B = limbs of 4 pairs' SwiGLU rows.

template <int G, int WR>
__global__ void __launch_bounds__(WR * 128) k_down(ExpertCallArgs a, GroupView gv,
                                                   const uint16_t *__restrict__ al,
                                                   const float4 *__restrict__ am,
                                                   uint16_t *__restrict__ d, uint32_t *err) {
  constexpr int WPG = G / 8;
  constexpr int WB = G / 32;
  constexpr int KSTEPS = G / 16;
  constexpr int ROWS = 16 * WR;
  constexpr int MT = kTokPerItem / 4;
  extern __shared__ float part[];  // [WR][4][16][kTokPerItem]
  const int H = a.H, I = a.I;
  const int Gi = I / G;
  const int P = chain_count(Gi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wr = warp >> 2, ch = warp & 3;
  const int r = lane >> 2, c = lane & 3;
  const int row_tiles = (H + ROWS - 1) / ROWS;
  const int n_items = gv.n_tiles[0] * row_tiles;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int tile = item / row_tiles, rt = item - tile * row_tiles;
    const int4 td = gv.tiles[tile];
    const int start = td.y, len = td.z;
    const uint32_t key = gv.bin_key[td.x];
    Ptrs pd;
    const bool ok = resolve(a, key, 2, H, I, pd);
    if (!ok && threadIdx.x == 0) set_error(err, kErrBadRoute);
    if (ok && ch < P) {
      const int h0 = rt * ROWS + wr * 16 + r;
      const int h1 = h0 + 8;
      const bool ok0 = h0 < H, ok1 = h1 < H;
      const int hc0 = ok0 ? h0 : 0, hc1 = ok1 ? h1 : 0;
      const int nmt = (len + 3) >> 2;
      int pB[MT], pE[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int qb = 4 * mt + (r >> 1);
        const int qe = 4 * mt + c;
        pB[mt] = (qb < len) ? gv.order[start + qb] : -1;
        pE[mt] = (qe < len) ? gv.order[start + qe] : -1;
      }
      float acc[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = -0.0f;
      const uint32_t *w0 = pd.w + static_cast<size_t>(hc0) * (I / 8);
      const uint32_t *w1 = pd.w + static_cast<size_t>(hc1) * (I / 8);
      const uint16_t *s0 = pd.s + static_cast<size_t>(hc0) * Gi;
      const uint16_t *b0 = pd.b + static_cast<size_t>(hc0) * Gi;
      const uint16_t *s1 = pd.s + static_cast<size_t>(hc1) * Gi;
      const uint16_t *b1 = pd.b + static_cast<size_t>(hc1) * Gi;
      const int g0 = chain_begin(ch, P, Gi), g1 = chain_begin(ch + 1, P, Gi);
      for (int g = g0; g < g1; ++g) {
        uint32_t wa[WB], wb_[WB];
#pragma unroll
        for (int wb = 0; wb < WB; ++wb) {
          wa[wb] = ok0 ? ldg_u32(w0 + g * WPG + wb * 4 + c) : 0u;
          wb_[wb] = ok1 ? ldg_u32(w1 + g * WPG + wb * 4 + c) : 0u;
        }
        const float sa = ok0 ? bf16_to_f32(ldg_u16(s0 + g)) : 0.0f;
        const float ba = ok0 ? bf16_to_f32(ldg_u16(b0 + g)) : 0.0f;
        const float sb = ok1 ? bf16_to_f32(ldg_u16(s1 + g)) : 0.0f;
        const float bb = ok1 ? bf16_to_f32(ldg_u16(b1 + g)) : 0.0f;
        uint32_t A[KSTEPS][4];
#pragma unroll
        for (int st = 0; st < KSTEPS; ++st) {
          const int wb = st >> 1, j = (st & 1) * 2;
          A[st][0] = nibble_pair(wa[wb], j);
          A[st][1] = nibble_pair(wb_[wb], j);
          A[st][2] = nibble_pair(wa[wb], j + 1);
          A[st][3] = nibble_pair(wb_[wb], j + 1);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (mt < nmt) {
            float C[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint4 v[WB];
            if (pB[mt] >= 0) {
              const uint16_t *base = al + (static_cast<size_t>(pB[mt]) * Gi + g) * 2 * G + (r & 1) * G;
#pragma unroll
              for (int wb = 0; wb < WB; ++wb)
                v[wb] = ldg_u128(reinterpret_cast<const uint4 *>(base + wb * 32 + c * 8));
            } else {
#pragma unroll
              for (int wb = 0; wb < WB; ++wb) v[wb] = make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int st = 0; st < KSTEPS; ++st) {
              const uint4 &vv = v[st >> 1];
              if (st & 1) mma_16816(C, A[st], vv.z, vv.w);
              else mma_16816(C, A[st], vv.x, vv.y);
            }
            if (pE[mt] >= 0) {
              const float4 m = am[static_cast<size_t>(pE[mt]) * Gi + g];
              const int k = static_cast<int>(m.z);
              const float S0 = __fmaf_rn(C[0], 4096.0f, C[1]);
              const float t0 = __fadd_rn(__fmul_rn(sa, S0), __fmul_rn(ba, m.x));
              acc[mt][0] = __fadd_rn(acc[mt][0], scale_pow2(t0, m.y, k));
              const float S1 = __fmaf_rn(C[2], 4096.0f, C[3]);
              const float t1 = __fadd_rn(__fmul_rn(sb, S1), __fmul_rn(bb, m.x));
              acc[mt][1] = __fadd_rn(acc[mt][1], scale_pow2(t1, m.y, k));
            }
          }
        }
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int qe = 4 * mt + c;
        if (qe < len) {
          part[((wr * 4 + ch) * 16 + r) * kTokPerItem + qe] = acc[mt][0];
          part[((wr * 4 + ch) * 16 + r + 8) * kTokPerItem + qe] = acc[mt][1];
        }
      }
    }
    __syncthreads();
    if (ok) {
      for (int idx = threadIdx.x; idx < len * ROWS; idx += blockDim.x) {
        const int q = idx / ROWS, ol = idx - q * ROWS;
        const int h = rt * ROWS + ol;
        if (h >= H) continue;
        const int wr2 = ol >> 4, rr = ol & 15;
        float cc[4] = {-0.0f, -0.0f, -0.0f, -0.0f};
        for (int k = 0; k < P; ++k) cc[k] = part[((wr2 * 4 + k) * 16 + rr) * kTokPerItem + q];
        const int pair = gv.order[start + q];
        d[static_cast<size_t>(pair) * H + h] = f32_to_bf16(chain_tree(cc, P));
      }
    }
    __syncthreads();
  }
}

namespace {
constexpr int kWR = 2;
template <typename K>
int persistent_grid(K kernel, int threads, size_t smem) {
  const DeviceInfo di = device_info();
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 1;
  return di.sms * per_sm;
}
}  // namespace

cudaError_t launch_gate_up(const ExpertCallArgs &a, const GroupView &gv,
                           const uint16_t *x_limbs, const float4 *x_meta,
                           uint16_t *act, uint16_t *g_out, uint16_t *u_out,
                           cudaStream_t s) {
  const int threads = kWR * 128;
  const size_t smem = static_cast<size_t>(kWR) * 4 * 16 * kTokPerItem * sizeof(float);
  uint32_t *err = device_error_word();
  if (a.G == 32) {
    const int grid = persistent_grid(k_gate_up<32, kWR>, threads, smem);
    k_gate_up<32, kWR><<<grid, threads, smem, s>>>(a, gv, x_limbs, x_meta, act, g_out, u_out, err);
  } else {
    const int grid = persistent_grid(k_gate_up<64, kWR>, threads, smem);
    k_gate_up<64, kWR><<<grid, threads, smem, s>>>(a, gv, x_limbs, x_meta, act, g_out, u_out, err);
  }
  return cudaGetLastError();
}

cudaError_t launch_down(const ExpertCallArgs &a, const GroupView &gv,
                        const uint16_t *act_limbs, const float4 *act_meta,
                        uint16_t *d, cudaStream_t s) {
  const int threads = kWR * 128;
  const size_t smem = static_cast<size_t>(kWR) * 4 * 16 * kTokPerItem * sizeof(float);
  uint32_t *err = device_error_word();
  if (a.G == 32) {
    const int grid = persistent_grid(k_down<32, kWR>, threads, smem);
    k_down<32, kWR><<<grid, threads, smem, s>>>(a, gv, act_limbs, act_meta, d, err);
  } else {
    const int grid = persistent_grid(k_down<64, kWR>, threads, smem);
    k_down<64, kWR><<<grid, threads, smem, s>>>(a, gv, act_limbs, act_meta, d, err);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// combine (metal_runtime.py:301-333)
// ---------------------------------------------------------------------------

__global__ void k_combine(const uint16_t *__restrict__ d, const uint32_t *__restrict__ routes,
                          const void *__restrict__ scores, int sf32, int T, int S, int H,
                          int mode, const uint16_t *__restrict__ sy,
                          const uint16_t *__restrict__ sh, const uint16_t *__restrict__ sg,
                          int E_arr, int records, uint16_t *__restrict__ out) {
  const int t = blockIdx.y;
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H || t >= T) return;
  float acc = 0.0f;
  for (int s = 0; s < S; ++s) {
    const uint32_t r = routes[t * S + s];
    const bool valid = (r & kSlotBit) ? ((r & 0x7FFFFFFFu) < static_cast<uint32_t>(records))
                                      : (r < static_cast<uint32_t>(E_arr));
    if (!valid) continue;
    const float dv = bf16_to_f32(d[(static_cast<size_t>(t) * S + s) * H + h]);
    const float sc = sf32 ? static_cast<const float *>(scores)[t * S + s]
                          : bf16_to_f32(static_cast<const uint16_t *>(scores)[t * S + s]);
    acc = __fadd_rn(acc, __fmul_rn(dv, sc));
  }
  const float routed = round_bf16(acc);
  float res;
  if (mode == kCombineSharedY) {
    res = __fadd_rn(routed, bf16_to_f32(sy[static_cast<size_t>(t) * H + h]));
  } else if (mode == kCombineParts) {
    const float comp = bmul(bf16_to_f32(sh[static_cast<size_t>(t) * H + h]), bf16_to_f32(sg[t]));
    res = __fadd_rn(routed, comp);
  } else {
    res = routed;
  }
  out[static_cast<size_t>(t) * H + h] = f32_to_bf16(res);
}

cudaError_t launch_combine(const uint16_t *d, const uint32_t *routes, const void *scores,
                           int scores_f32, int tokens, int slots, int H, int mode,
                           const uint16_t *shared_y, const uint16_t *shared,
                           const uint16_t *shared_gate, int array_experts, int table_records,
                           uint16_t *out, cudaStream_t s) {
  dim3 grid((H + 255) / 256, tokens);
  k_combine<<<grid, 256, 0, s>>>(d, routes, scores, scores_f32, tokens, slots, H, mode, shared_y,
                                 shared, shared_gate, array_experts, table_records, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// router logits: bf16 GEMV with the canonical 32-lane order
// ---------------------------------------------------------------------------

constexpr int kRouterWarps = 4;
constexpr int kRouterTokBlock = 8;

template <int CH>
__global__ void __launch_bounds__(kRouterWarps * 32) k_router_logits(
    const uint16_t *__restrict__ x, const uint16_t *__restrict__ W, int T, int H, int E,
    const uint16_t *__restrict__ wsg, uint16_t *__restrict__ logits,
    uint16_t *__restrict__ shared_logit) {
  extern __shared__ float xs[];  // [kRouterTokBlock][H]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRouterWarps + warp;
  const int rows = E + (wsg != nullptr ? 1 : 0);
  const int nchunks = H / 8;
  const uint16_t *wrow = nullptr;
  if (row < E) wrow = W + static_cast<size_t>(row) * H;
  else if (row < rows) wrow = wsg;
  float w[CH * 8];
#pragma unroll
  for (int m = 0; m < CH; ++m) {
    const int cidx = lane + 32 * m;
    if (wrow != nullptr && cidx < nchunks) {
      const uint4 v = ldg_u128(reinterpret_cast<const uint4 *>(wrow + cidx * 8));
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w[m * 8 + 2 * i] = __uint_as_float(u[i] << 16);
        w[m * 8 + 2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[m * 8 + i] = 0.0f;
    }
  }
  for (int t0 = 0; t0 < T; t0 += kRouterTokBlock) {
    const int tb = min(kRouterTokBlock, T - t0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < tb * H; idx += blockDim.x) {
      xs[idx] = bf16_to_f32(x[static_cast<size_t>(t0) * H + idx]);
    }
    __syncthreads();
    if (wrow == nullptr) continue;
    for (int tt = 0; tt < tb; ++tt) {
      float acc = -0.0f;
#pragma unroll
      for (int m = 0; m < CH; ++m) {
        const int cidx = lane + 32 * m;
        if (cidx < nchunks) {
          const float *xp = xs + tt * H + cidx * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) acc = __fmaf_rn(w[m * 8 + i], xp[i], acc);
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, off));
      if (lane == 0) {
        if (row < E) logits[static_cast<size_t>(t0 + tt) * E + row] = f32_to_bf16(acc);
        else shared_logit[t0 + tt] = f32_to_bf16(acc);
      }
    }
  }
}

cudaError_t launch_router_logits(const uint16_t *x, const uint16_t *W, int T, int H, int E,
                                 const uint16_t *w_shared_gate, uint16_t *logits,
                                 uint16_t *shared_logit, cudaStream_t s) {
  const int rows = E + (w_shared_gate ? 1 : 0);
  const int blocks = (rows + kRouterWarps - 1) / kRouterWarps;
  const size_t smem = static_cast<size_t>(kRouterTokBlock) * H * sizeof(float);
  const int nchunks = H / 8;
  const int ch = (nchunks + 31) / 32;
#define FNMOE_ROUTER_CASE(N)                                                                 \
  if (ch <= N) {                                                                            \
    if (smem > 48 * 1024) {                                                                 \
      cudaError_t e = cudaFuncSetAttribute(k_router_logits<N>,                              \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                                           static_cast<int>(smem));                         \
      if (e != cudaSuccess) return e;                                                       \
    }                                                                                       \
    k_router_logits<N><<<blocks, kRouterWarps * 32, smem, s>>>(x, W, T, H, E, w_shared_gate, \
                                                               logits, shared_logit);       \
    return cudaGetLastError();                                                              \
  }
  FNMOE_ROUTER_CASE(4)
  FNMOE_ROUTER_CASE(8)
  FNMOE_ROUTER_CASE(12)
  FNMOE_ROUTER_CASE(16)
#undef FNMOE_ROUTER_CASE
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// softmax (precise) + top-k + renorm, one warp per token
// ---------------------------------------------------------------------------

constexpr int kMaxPerLane = 32;  // experts <= 1024

__global__ void __launch_bounds__(128) k_softmax_topk(
    const uint16_t *__restrict__ logits, int T, int E, int k, float blend,
    const uint32_t *__restrict__ route_map, int table_routes, uint32_t *__restrict__ inds,
    uint32_t *__restrict__ routes, uint16_t *__restrict__ raw_scores,
    uint16_t *__restrict__ scores, uint16_t *__restrict__ mass,
    const uint16_t *__restrict__ shl, uint16_t *__restrict__ shg) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= T) return;
  const int per = (E + 31) / 32;
  float l[kMaxPerLane];
  float mx = -INFINITY;
  const uint16_t *lrow = logits + static_cast<size_t>(t) * E;
#pragma unroll
  for (int m = 0; m < kMaxPerLane; ++m) {
    const int i = lane + 32 * m;
    l[m] = (m < per && i < E) ? bf16_to_f32(lrow[i]) : -INFINITY;
    mx = fmaxf(mx, l[m]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  float sum = -0.0f;
#pragma unroll
  for (int m = 0; m < kMaxPerLane; ++m) {
    const int i = lane + 32 * m;
    if (m < per && i < E) {
      l[m] = __double2float_rn(exp(static_cast<double>(__fsub_rn(l[m], mx))));
      sum = __fadd_rn(sum, l[m]);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, off));
  uint32_t key[kMaxPerLane];
#pragma unroll
  for (int m = 0; m < kMaxPerLane; ++m) {
    const int i = lane + 32 * m;
    if (m < per && i < E) {
      const uint32_t pb = f32_to_bf16(__fdiv_rn(l[m], sum));
      key[m] = (pb << 16) | (0xFFFFu - static_cast<uint32_t>(i));
    } else {
      key[m] = 0u;
    }
  }
  float acc = 0.0f;
  float sel[16];
  uint32_t idx[16];
  for (int s = 0; s < k; ++s) {
    uint32_t best = 0u;
#pragma unroll
    for (int m = 0; m < kMaxPerLane; ++m) best = max(best, key[m]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, off));
#pragma unroll
    for (int m = 0; m < kMaxPerLane; ++m)
      if (key[m] == best) key[m] = 0u;
    const uint32_t i = 0xFFFFu - (best & 0xFFFFu);
    const float p = bf16_to_f32(static_cast<uint16_t>(best >> 16));
    sel[s] = p;
    idx[s] = i;
    acc = __fadd_rn(acc, p);
  }
  if (lane == 0) {
    const float topm = round_bf16(acc);
    const float selected = topm;  // threshold 1.0 keeps every selected slot
    const float bl = round_bf16(blend);
    const float normalizer = badd(topm, bmul(bl, bsub(selected, topm)));
    for (int s = 0; s < k; ++s) {
      const uint32_t e = idx[s];
      inds[static_cast<size_t>(t) * k + s] = e;
      routes[static_cast<size_t>(t) * k + s] =
          route_map ? route_map[e] : (table_routes ? (kSlotBit | e) : e);
      if (raw_scores) raw_scores[static_cast<size_t>(t) * k + s] = f32_to_bf16(sel[s]);
      if (scores) scores[static_cast<size_t>(t) * k + s] = f32_to_bf16(__fdiv_rn(sel[s], normalizer));
    }
    if (mass) mass[t] = f32_to_bf16(topm);
    if (shl && shg) shg[t] = f32_to_bf16(sigmoid_bf16(g_exp_bf16, bf16_to_f32(shl[t])));
  }
}

cudaError_t launch_softmax_topk(const uint16_t *logits, int T, int E, int k, float blend,
                                const uint32_t *route_map, int table_routes, uint32_t *inds,
                                uint32_t *routes, uint16_t *raw_scores, uint16_t *scores,
                                uint16_t *mass, const uint16_t *shared_logit,
                                uint16_t *shared_gate, cudaStream_t s) {
  k_softmax_topk<<<(T + 3) / 4, 128, 0, s>>>(logits, T, E, k, blend, route_map, table_routes,
                                            inds, routes, raw_scores, scores, mass, shared_logit,
                                            shared_gate);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// elementwise helpers
// ---------------------------------------------------------------------------

__global__ void k_dequant(const uint32_t *__restrict__ w, const uint16_t *__restrict__ sc,
                          const uint16_t *__restrict__ bi, uint16_t *__restrict__ out,
                          uint64_t words, int K, int G) {
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const int wpr = K / 8;
  const uint64_t row = i / wpr;
  const int wcol = static_cast<int>(i - row * wpr);
  const int g = (wcol * 8) / G;
  const double s = bf16_to_f32(sc[row * (K / G) + g]);
  const double b = bf16_to_f32(bi[row * (K / G) + g]);
  const uint32_t word = w[i];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const double q = static_cast<double>((word >> (4 * j)) & 15u);
    out[row * K + wcol * 8 + j] = f64_to_bf16_once(s * q + b);
  }
}

cudaError_t launch_dequant(const uint32_t *w, const uint16_t *sc, const uint16_t *bi,
                           uint16_t *out, uint64_t rows, int K, int G, cudaStream_t s) {
  const uint64_t words = rows * (K / 8);
  if (words == 0) return cudaSuccess;
  k_dequant<<<static_cast<unsigned>((words + 255) / 256), 256, 0, s>>>(w, sc, bi, out, words, K, G);
  return cudaGetLastError();
}

__global__ void k_swiglu(const uint16_t *__restrict__ g, const uint16_t *__restrict__ u,
                         uint16_t *__restrict__ out, uint64_t n) {
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = f32_to_bf16(swiglu_bf16(g_exp_bf16, bf16_to_f32(g[i]), bf16_to_f32(u[i])));
}

cudaError_t launch_swiglu(const uint16_t *g, const uint16_t *u, uint16_t *out, uint64_t n,
                          cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_swiglu<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(g, u, out, n);
  return cudaGetLastError();
}

// weighted_combine (metal_runtime.py:145-191): products then a sequential sum
// over slots starting from the first product (NumPy add.reduce on axis -2).
__global__ void k_weighted_combine(const float *__restrict__ outputs, const int32_t *__restrict__ routes,
                                   const float *__restrict__ scores, float *__restrict__ out,
                                   int T, int S, int E, int H) {
  const int t = blockIdx.y;
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  float acc = 0.0f;
  for (int s = 0; s < S; ++s) {
    const float v = (E > 0)
        ? outputs[(static_cast<size_t>(t) * E + routes[t * S + s]) * H + h]
        : outputs[(static_cast<size_t>(t) * S + s) * H + h];
    const float p = __fmul_rn(v, scores[t * S + s]);
    acc = (s == 0) ? p : __fadd_rn(acc, p);
  }
  out[static_cast<size_t>(t) * H + h] = acc;
}

cudaError_t launch_weighted_combine(const float *outputs, const int32_t *routes,
                                    const float *scores, float *out, int T, int S, int E, int H,
                                    cudaStream_t s) {
  dim3 grid((H + 255) / 256, T);
  k_weighted_combine<<<grid, 256, 0, s>>>(outputs, routes, scores, out, T, S, E, H);
  return cudaGetLastError();
}

}  // namespace fnmoe
