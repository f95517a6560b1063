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

#include <algorithm>
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
    const int ka = max(k, -126);
    const float A = __int_as_float((ka + 127) << 23);       // 2^ka, normal
    const float B = __int_as_float((k - ka + 127) << 23);   // 2^(k-ka) in [2^-29, 1]
    meta[static_cast<size_t>(row) * Gc + g] = make_float4(__int2float_rn(sx), A, B, 0.0f);
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
    cnt[b] = pre_t;  // first tile of the bin (counts now live in gv.counts)
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
  __syncthreads();
  // Self-contained tile descriptors: {route key, start, len, bin} and the pair ids.
  for (int b = b0; b < b1; ++b) {
    const int c = gv.counts[b];
    const int nt = (c + kTokPerItem - 1) / kTokPerItem;
    const int first = cnt[b];
    const int start_b = gv.offsets[b];
    const uint32_t key = gv.bin_key[b];
    for (int t = 0; t < nt && first + t < gv.max_tiles; ++t) {
      const int st = start_b + t * kTokPerItem;
      const int len = min(kTokPerItem, c - t * kTokPerItem);
      int p[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) p[q] = q < len ? gv.order[st + q] : -1;
      gv.tiles[3 * (first + t)] = make_int4(static_cast<int>(key), st, len, b);
      gv.tiles[3 * (first + t) + 1] = make_int4(p[0], p[1], p[2], p[3]);
      gv.tiles[3 * (first + t) + 2] = make_int4(p[4], p[5], p[6], p[7]);
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
// grouped Q4 expert projections (gate/up + SwiGLU, and down)
// ---------------------------------------------------------------------------
// Work item = (expert bin, WARPS x RPW output rows, up to kTokPerItem pairs).
// Each warp owns RPW rows over the full contraction width and keeps all P
// summation chains in registers, so no cross-warp reduction is needed.  The
// packed rows and their scales/biases stream straight from HBM into
// registers, PF groups ahead of use; the item's activation limbs and
// fixed-point metadata (shared by every warp of the CTA) are staged in
// shared memory with cp.async, double-buffered across items.
//
// MMA row mapping: DUAL (gate/up) -- M rows 0-7 are 8 gate rows and M rows
// 8-15 the same 8 up rows, so a thread ends with gate and up of the same
// (row, token) and applies SwiGLU in registers.  Single (down) -- M rows
// 0-7 and 8-15 are 16 consecutive hidden rows.

struct XStage {
  int Gc;      // groups along the contraction width
  int Xrow;    // limb bytes per pair
  int Mp;      // padded metadata pitch per pair
  int m_off;   // metadata offset in the stage
  int bytes;   // stage size
};

__host__ __device__ inline XStage xstage_geom(int K, int G) {
  XStage s{};
  s.Gc = K / G;
  s.Xrow = s.Gc * 4 * G;
  s.Mp = s.Gc * 16 + 16;
  s.m_off = kTokPerItem * s.Xrow;
  s.bytes = ((s.m_off + kTokPerItem * s.Mp + 127) / 128) * 128;
  return s;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::); }

struct RawDesc {
  int4 d0, d1, d2;
};

struct ItemInfo {
  bool valid;   // item index in range
  bool ok;      // expert pointers resolved
  int len, rt;
  int pair[kTokPerItem];  // pair ids of the token slots (-1 beyond len)
  Ptrs p[2];
};

__device__ __forceinline__ RawDesc load_desc(const GroupView &gv, int item, int n_items, int row_tiles) {
  RawDesc r{};
  if (item < n_items) {
    const int tile = item / row_tiles;
    r.d0 = gv.tiles[3 * tile];
    r.d1 = gv.tiles[3 * tile + 1];
    r.d2 = gv.tiles[3 * tile + 2];
  }
  return r;
}

template <bool DUAL>
__device__ __forceinline__ ItemInfo item_info(const ExpertCallArgs &a, const RawDesc &rd, int item,
                                              int n_items, int row_tiles, int out_rows, int in_cols) {
  ItemInfo it{};
  it.valid = item < n_items;
  if (!it.valid) return it;
  it.rt = item - (item / row_tiles) * row_tiles;
  it.len = rd.d0.z;
  it.pair[0] = rd.d1.x;
  it.pair[1] = rd.d1.y;
  it.pair[2] = rd.d1.z;
  it.pair[3] = rd.d1.w;
  it.pair[4] = rd.d2.x;
  it.pair[5] = rd.d2.y;
  it.pair[6] = rd.d2.z;
  it.pair[7] = rd.d2.w;
  const uint32_t key = static_cast<uint32_t>(rd.d0.x);
  if (DUAL) {
    it.ok = resolve(a, key, 0, out_rows, in_cols, it.p[0]) && resolve(a, key, 1, out_rows, in_cols, it.p[1]);
  } else {
    it.ok = resolve(a, key, 2, out_rows, in_cols, it.p[0]);
  }
  return it;
}

// Stage the activation limbs and metadata of an item's pairs (all threads).
__device__ __forceinline__ void load_xstage(uint8_t *st, const XStage &xs, const ItemInfo &it,
                                            const uint16_t *__restrict__ xl, const float4 *__restrict__ xm,
                                            int n_pairs, int slots, bool by_token) {
  if (!it.valid || !it.ok) return;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int cpx = xs.Xrow / 16;
#pragma unroll
  for (int q = 0; q < kTokPerItem; ++q) {
    uint8_t *dst = st + q * xs.Xrow;
    uint8_t *mdst = st + xs.m_off + q * xs.Mp;
    if (q < it.len) {
      const int pair = it.pair[q];
      const int row = by_token ? token_of_pair(pair, n_pairs, slots) : pair;
      const uint8_t *src = reinterpret_cast<const uint8_t *>(xl) + static_cast<size_t>(row) * xs.Xrow;
      for (int cc = tid; cc < cpx; cc += nt) cp_async16(dst + cc * 16, src + cc * 16);
      const float4 *msrc = xm + static_cast<size_t>(row) * xs.Gc;
      for (int g = tid; g < xs.Gc; g += nt) cp_async16(mdst + g * 16, msrc + g);
    } else {
      // empty slot: zero limbs (the MMA adds nothing) and a neutral scale
      for (int cc = tid; cc < cpx; cc += nt) *reinterpret_cast<uint4 *>(dst + cc * 16) = make_uint4(0u, 0u, 0u, 0u);
      for (int g = tid; g < xs.Gc; g += nt) *reinterpret_cast<float4 *>(mdst + g * 16) = make_float4(0.0f, 1.0f, 1.0f, 0.0f);
    }
  }
}

// Fold one group into a chain: fS = fl(S); t = fma(s, fS, fl(b*fl(SX)));
// acc = fma(fl(t*A), B, acc).  m = {fl(SX), A, B, -}.
__device__ __forceinline__ float group_fold(float acc, float c_hi, float c_lo, float s, float b, const float4 &m) {
  const float S = __fmaf_rn(c_hi, 4096.0f, c_lo);
  const float t = __fmaf_rn(s, S, __fmul_rn(b, m.x));
  return __fmaf_rn(__fmul_rn(t, m.y), m.z, acc);
}

// PF consecutive bfloat16 scales (or biases) loaded as one vector.
template <int PF>
struct Vec16 {
  uint32_t w[(PF + 1) / 2];
  __device__ __forceinline__ void load(const uint16_t *p) {
    if constexpr (PF == 8) {
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (PF == 4) {
      const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p));
      w[0] = v.x; w[1] = v.y;
    } else if constexpr (PF == 2) {
      w[0] = __ldg(reinterpret_cast<const uint32_t *>(p));
    } else {
      w[0] = __ldg(p);
    }
  }
  __device__ __forceinline__ float get(int j) const {  // j is a compile-time constant after unrolling
    const uint32_t word = w[j >> 1];
    return __uint_as_float((j & 1) ? (word & 0xFFFF0000u) : (word << 16));
  }
};

// Pair id of token slot 4t + c without dynamic register-array indexing.
__device__ __forceinline__ int item_pair(const ItemInfo &it, int t, int c) {
  if (t == 0) return c == 0 ? it.pair[0] : c == 1 ? it.pair[1] : c == 2 ? it.pair[2] : it.pair[3];
  return c == 0 ? it.pair[4] : c == 1 ? it.pair[5] : c == 2 ? it.pair[6] : it.pair[7];
}

// Multiply one item's rows for NT token tiles (4 pairs each) and write the
// results.  The packed words of the two MMA rows stream through a PF-deep
// register ring; scales/biases arrive as PF-wide vectors one block ahead.
template <int G, int WARPS, bool DUAL, int PF, int NT>
__device__ __forceinline__ void run_item(const ExpertCallArgs &a, const ItemInfo &cur, const uint8_t *st,
                                         const XStage &xs, int O, int K, uint16_t *__restrict__ out,
                                         uint16_t *__restrict__ g_out, uint16_t *__restrict__ u_out) {
  constexpr int WB = G / 32;
  constexpr int WPG = G / 8;
  constexpr int RPW = DUAL ? 8 : 16;
  constexpr int ROWS = RPW * WARPS;
  const int Gc = xs.Gc;
  const int P = chain_count(Gc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int wpr = K / 8;
  const int o0 = cur.rt * ROWS + warp * RPW + r;
  const int oA = o0;
  const int oB = DUAL ? o0 : o0 + 8;
  const int cA = min(oA, O - 1), cB = min(oB, O - 1);
  const Ptrs &pA = cur.p[0];
  const Ptrs &pB = DUAL ? cur.p[1] : cur.p[0];
  const uint32_t *wA = pA.w + static_cast<size_t>(cA) * wpr + c;
  const uint32_t *wB = pB.w + static_cast<size_t>(cB) * wpr + c;
  const uint16_t *sA = pA.s + static_cast<size_t>(cA) * Gc;
  const uint16_t *bA = pA.b + static_cast<size_t>(cA) * Gc;
  const uint16_t *sB = pB.s + static_cast<size_t>(cB) * Gc;
  const uint16_t *bB = pB.b + static_cast<size_t>(cB) * Gc;
  uint32_t qa[PF][WB], qb[PF][WB];
#pragma unroll
  for (int j = 0; j < PF; ++j) {
#pragma unroll
    for (int wb = 0; wb < WB; ++wb) {
      qa[j][wb] = ldg_u32(wA + j * WPG + wb * 4);
      qb[j][wb] = ldg_u32(wB + j * WPG + wb * 4);
    }
  }
  Vec16<PF> vsA, vbA, vsB, vbB;
  vsA.load(sA);
  vbA.load(bA);
  vsB.load(sB);
  vbB.load(bB);
  const uint8_t *xb = st + (r >> 1) * xs.Xrow + (r & 1) * (G * 2) + c * 16;
  const float4 *mrow = reinterpret_cast<const float4 *>(st + xs.m_off + c * xs.Mp);
  // Chain tree folded as chains complete: h0 = c0 (+ c2), h1 = c1 (+ c3).
  float hA0[NT], hA1[NT], hB0[NT], hB1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) hA0[t] = hA1[t] = hB0[t] = hB1[t] = -0.0f;
  for (int ch = 0; ch < P; ++ch) {
    float accA[NT], accB[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) accA[t] = accB[t] = -0.0f;
    const int gend = chain_begin(ch + 1, P, Gc);
    for (int g0 = chain_begin(ch, P, Gc); g0 < gend; g0 += PF) {
      const int gn0 = (g0 + PF < Gc) ? g0 + PF : g0;  // next block (the last one is re-read)
      Vec16<PF> nsA, nbA, nsB, nbB;
      nsA.load(sA + gn0);
      nbA.load(bA + gn0);
      nsB.load(sB + gn0);
      nbB.load(bB + gn0);
      const uint32_t *nwA = wA + gn0 * WPG;
      const uint32_t *nwB = wB + gn0 * WPG;
      const uint8_t *xg = xb + g0 * (4 * G);
      const float4 *mg = mrow + g0;
#pragma unroll
      for (int j = 0; j < PF; ++j) {
        uint32_t A0[WB][4], A1[WB][4];
#pragma unroll
        for (int wb = 0; wb < WB; ++wb) {
          nibble_operands(qa[j][wb], qb[j][wb], A0[wb], A1[wb]);
          qa[j][wb] = ldg_u32(nwA + j * WPG + wb * 4);
          qb[j][wb] = ldg_u32(nwB + j * WPG + wb * 4);
        }
        const float s0 = vsA.get(j), b0 = vbA.get(j), s1 = vsB.get(j), b1 = vbB.get(j);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float C[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int wb = 0; wb < WB; ++wb) {
            const uint4 v = *reinterpret_cast<const uint4 *>(xg + t * 4 * xs.Xrow + j * (4 * G) + wb * 64);
            mma_16816(C, A0[wb], v.x, v.y);
            mma_16816(C, A1[wb], v.z, v.w);
          }
          const float4 m = *reinterpret_cast<const float4 *>(
              reinterpret_cast<const uint8_t *>(mg + j) + t * 4 * xs.Mp);
          accA[t] = group_fold(accA[t], C[0], C[1], s0, b0, m);
          accB[t] = group_fold(accB[t], C[2], C[3], s1, b1, m);
        }
      }
      vsA = nsA;
      vbA = nbA;
      vsB = nsB;
      vbB = nbB;
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (ch == 0) { hA0[t] = accA[t]; hB0[t] = accB[t]; }
      else if (ch == 1) { hA1[t] = accA[t]; hB1[t] = accB[t]; }
      else if (ch == 2) { hA0[t] = __fadd_rn(hA0[t], accA[t]); hB0[t] = __fadd_rn(hB0[t], accB[t]); }
      else { hA1[t] = __fadd_rn(hA1[t], accA[t]); hB1[t] = __fadd_rn(hB1[t], accB[t]); }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int q = 4 * t + c;
    if (q < cur.len) {
      const int pair = item_pair(cur, t, c);
      const float yA = P == 1 ? hA0[t] : __fadd_rn(hA0[t], hA1[t]);
      const float yB = P == 1 ? hB0[t] : __fadd_rn(hB0[t], hB1[t]);
      if (DUAL) {
        if (oA < O) {
          const float gvv = round_bf16(yA), uvv = round_bf16(yB);
          out[static_cast<size_t>(pair) * O + oA] = f32_to_bf16(swiglu_bf16(g_exp_bf16, gvv, uvv));
          if (g_out != nullptr && pair < a.n_pairs) {
            g_out[static_cast<size_t>(pair) * O + oA] = f32_to_bf16(gvv);
            u_out[static_cast<size_t>(pair) * O + oA] = f32_to_bf16(uvv);
          }
        }
      } else {
        if (oA < O) out[static_cast<size_t>(pair) * O + oA] = f32_to_bf16(yA);
        if (oB < O) out[static_cast<size_t>(pair) * O + oB] = f32_to_bf16(yB);
      }
    }
  }
}

template <int G, int WARPS, bool DUAL, int PF>
__global__ void __launch_bounds__(WARPS * 32) k_expert_rows(ExpertCallArgs a, GroupView gv,
                                                            const uint16_t *__restrict__ xl,
                                                            const float4 *__restrict__ xm,
                                                            uint16_t *__restrict__ out,
                                                            uint16_t *__restrict__ g_out,
                                                            uint16_t *__restrict__ u_out, uint32_t *err) {
  constexpr int RPW = DUAL ? 8 : 16;
  constexpr int ROWS = RPW * WARPS;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = DUAL ? a.H : a.I;
  const int O = DUAL ? a.I : a.H;
  const XStage xs = xstage_geom(K, G);
  const int row_tiles = (O + ROWS - 1) / ROWS;
  const int n_items = gv.n_tiles[0] * row_tiles;

  int item = blockIdx.x;
  ItemInfo cur = item_info<DUAL>(a, load_desc(gv, item, n_items, row_tiles), item, n_items, row_tiles, O, K);
  RawDesc raw_next = load_desc(gv, item + gridDim.x, n_items, row_tiles);
  load_xstage(smem, xs, cur, xl, xm, a.n_pairs, a.slots, DUAL);
  cp_async_commit();
  for (int k = 0; cur.valid; ++k) {
    const uint8_t *st = smem + (k & 1) * xs.bytes;
    const int nitem = item + gridDim.x;
    const ItemInfo nxt = item_info<DUAL>(a, raw_next, nitem, n_items, row_tiles, O, K);
    raw_next = load_desc(gv, nitem + gridDim.x, n_items, row_tiles);
    load_xstage(smem + ((k + 1) & 1) * xs.bytes, xs, nxt, xl, xm, a.n_pairs, a.slots, DUAL);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();  // activation stage of this item is visible
    if (!cur.ok) {
      if (threadIdx.x == 0) set_error(err, kErrBadRoute);
    } else if (cur.len > 4) {
      run_item<G, WARPS, DUAL, PF, 2>(a, cur, st, xs, O, K, out, g_out, u_out);
    } else {
      run_item<G, WARPS, DUAL, PF, 1>(a, cur, st, xs, O, K, out, g_out, u_out);
    }
    __syncthreads();  // the stage is refilled two items later
    item = nitem;
    cur = nxt;
  }
  asm volatile("cp.async.wait_all;\n" ::);
}

namespace {

template <typename Kern>
cudaError_t launch_rows(Kern kernel, int threads, size_t smem, const ExpertCallArgs &a, const GroupView &gv,
                        const uint16_t *xl, const float4 *xm, uint16_t *out, uint16_t *g_out,
                        uint16_t *u_out, cudaStream_t s) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const DeviceInfo di = device_info();
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm <= 0)
    per_sm = 1;
  kernel<<<di.sms * per_sm, threads, smem, s>>>(a, gv, xl, xm, out, g_out, u_out, device_error_word());
  return cudaGetLastError();
}

constexpr size_t kSmemBudget = 200 * 1024;

}  // namespace

// Prefetch block: the largest of 8/4/2/1 that divides every chain length and
// keeps the scales/biases vector loads aligned.
int pick_pf(int K, int G) {
  const int Gc = K / G;
  const int P = chain_count(Gc);
  for (int pf : {8, 4, 2}) {
    bool ok = (Gc * 2) % (pf * 2) == 0;
    for (int ch = 0; ch < P && ok; ++ch) ok = ((chain_begin(ch + 1, P, Gc) - chain_begin(ch, P, Gc)) % pf) == 0;
    for (int ch = 0; ch < P && ok; ++ch) ok = (chain_begin(ch, P, Gc) % pf) == 0;
    if (ok) return pf;
  }
  return 1;
}

template <int G, int WARPS, bool DUAL>
cudaError_t launch_rows_pf(int pf, size_t smem, const ExpertCallArgs &a, const GroupView &gv, const uint16_t *xl,
                           const float4 *xm, uint16_t *out, uint16_t *g_out, uint16_t *u_out, cudaStream_t s) {
  const int threads = WARPS * 32;
  switch (pf) {
    case 8: return launch_rows(k_expert_rows<G, WARPS, DUAL, 8>, threads, smem, a, gv, xl, xm, out, g_out, u_out, s);
    case 4: return launch_rows(k_expert_rows<G, WARPS, DUAL, 4>, threads, smem, a, gv, xl, xm, out, g_out, u_out, s);
    case 2: return launch_rows(k_expert_rows<G, WARPS, DUAL, 2>, threads, smem, a, gv, xl, xm, out, g_out, u_out, s);
    default: return launch_rows(k_expert_rows<G, WARPS, DUAL, 1>, threads, smem, a, gv, xl, xm, out, g_out, u_out, s);
  }
}

// Expected pairs per launch decide the CTA width: many pairs -> 8 warps,
// few pairs (batch-1 decode) -> 4 warps so that the handful of experts still
// spreads over every SM.
cudaError_t launch_gate_up(const ExpertCallArgs &a, const GroupView &gv,
                           const uint16_t *x_limbs, const float4 *x_meta,
                           uint16_t *act, uint16_t *g_out, uint16_t *u_out,
                           cudaStream_t s) {
  const XStage xs = xstage_geom(a.H, a.G);
  const size_t smem = 2 * static_cast<size_t>(xs.bytes);
  if (smem > kSmemBudget) return cudaErrorInvalidValue;
  const bool wide = (a.n_pairs + a.tokens) >= 64;
  const int pf = std::min(4, pick_pf(a.H, a.G));
  if (a.G == 32) {
    if (wide) return launch_rows_pf<32, 16, true>(pf, smem, a, gv, x_limbs, x_meta, act, g_out, u_out, s);
    return launch_rows_pf<32, 4, true>(pf, smem, a, gv, x_limbs, x_meta, act, g_out, u_out, s);
  }
  if (wide) return launch_rows_pf<64, 16, true>(pf, smem, a, gv, x_limbs, x_meta, act, g_out, u_out, s);
  return launch_rows_pf<64, 4, true>(pf, smem, a, gv, x_limbs, x_meta, act, g_out, u_out, s);
}

cudaError_t launch_down(const ExpertCallArgs &a, const GroupView &gv,
                        const uint16_t *act_limbs, const float4 *act_meta,
                        uint16_t *d, cudaStream_t s) {
  const XStage xs = xstage_geom(a.I, a.G);
  const size_t smem = 2 * static_cast<size_t>(xs.bytes);
  if (smem > kSmemBudget) return cudaErrorInvalidValue;
  const bool wide = (a.n_pairs + a.tokens) >= 64;
  const int pf = pick_pf(a.I, a.G);
  if (a.G == 32) {
    if (wide) return launch_rows_pf<32, 16, false>(pf, smem, a, gv, act_limbs, act_meta, d, nullptr, nullptr, s);
    return launch_rows_pf<32, 4, false>(pf, smem, a, gv, act_limbs, act_meta, d, nullptr, nullptr, s);
  }
  if (wide) return launch_rows_pf<64, 16, false>(pf, smem, a, gv, act_limbs, act_meta, d, nullptr, nullptr, s);
  return launch_rows_pf<64, 4, false>(pf, smem, a, gv, act_limbs, act_meta, d, nullptr, nullptr, s);
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
  extern __shared__ __align__(16) float xs[];  // [kRouterTokBlock][H]
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
    // 8 bf16 per 16-byte load -> two float4 stores (rows are contiguous)
    const uint4 *xsrc = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t0) * H);
    float4 *xdst = reinterpret_cast<float4 *>(xs);
    for (int idx = threadIdx.x; idx < tb * H / 8; idx += blockDim.x) {
      const uint4 v = ldg_u128(xsrc + idx);
      xdst[2 * idx] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                  __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
      xdst[2 * idx + 1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                                      __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
    }
    __syncthreads();
    if (wrow == nullptr) continue;
    for (int tt = 0; tt < tb; ++tt) {
      float acc = -0.0f;
#pragma unroll
      for (int m = 0; m < CH; ++m) {
        const int cidx = lane + 32 * m;
        if (cidx < nchunks) {
          const float4 *xp = reinterpret_cast<const float4 *>(xs + tt * H + cidx * 8);
          const float4 p0 = xp[0], p1 = xp[1];
          acc = __fmaf_rn(w[m * 8 + 0], p0.x, acc);
          acc = __fmaf_rn(w[m * 8 + 1], p0.y, acc);
          acc = __fmaf_rn(w[m * 8 + 2], p0.z, acc);
          acc = __fmaf_rn(w[m * 8 + 3], p0.w, acc);
          acc = __fmaf_rn(w[m * 8 + 4], p1.x, acc);
          acc = __fmaf_rn(w[m * 8 + 5], p1.y, acc);
          acc = __fmaf_rn(w[m * 8 + 6], p1.z, acc);
          acc = __fmaf_rn(w[m * 8 + 7], p1.w, acc);
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
