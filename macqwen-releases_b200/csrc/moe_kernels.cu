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
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <map>
#include <mutex>

#include "async.cuh"
#include "common.cuh"
#include "umma.cuh"
#include "moe_kernels.cuh"

namespace fnmoe {

__device__ uint16_t g_exp_bf16[65536];
__device__ uint16_t g_silu_bf16[65536];  // bf16 bits of bmul(g, sigmoid_bf16(g)) for every bf16 g
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

// g * sigmoid(g) with the SwiGLU's own bf16 operations (swiglu_bf16 without
// the final multiply by u), so a lookup gives bit-identical activations.
__global__ void k_init_silu_table() {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536) return;
  const float g = bf16_to_f32(static_cast<uint16_t>(i));
  g_silu_bf16[i] = f32_to_bf16(bmul(g, sigmoid_bf16(g_exp_bf16, g)));
}

namespace {
std::mutex g_init_mutex;
bool g_exp_ready[64] = {false};
int g_sms[64] = {0};
}  // namespace

bool pdl_enabled() {
  static const bool on = std::getenv("FNMOE_NO_PDL") == nullptr;
  return on;
}

// FNMOE_NO_GEMV=1 runs small batches through k_expert_rows' 4-warp CTAs
// instead of the K-split GEMV (same results; for comparisons).
bool gemv_disabled() {
  static const bool off = std::getenv("FNMOE_NO_GEMV") != nullptr;
  return off;
}

// FNMOE_NO_FUSED=1 runs batch-1 layers through the multi-launch chain
// instead of the persistent kernel (same results; for comparisons).
bool fused_disabled() {
  static const bool off = std::getenv("FNMOE_NO_FUSED") != nullptr;
  return off;
}

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

cudaError_t exp_table_address(const uint16_t **table) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_exp_bf16);
  *table = static_cast<const uint16_t *>(p);
  return e;
}

cudaError_t silu_table_address(const uint16_t **table) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_silu_bf16);
  *table = static_cast<const uint16_t *>(p);
  return e;
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
  k_init_silu_table<<<256, 256, 0, stream>>>();
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

// Fixed-point value of one bfloat16 input for the row exponent E:
// trunc(x * 2^(22-E)); non-finite inputs give 0 (and are flagged).
__device__ __forceinline__ int fixed_x(uint32_t h, int E) {
  const uint32_t ef = (h >> 7) & 0xFFu, mf = h & 0x7Fu;
  if ((h & 0x7FFFu) == 0 || ef == 255u) return 0;
  const uint32_t M = ef ? (mf | 0x80u) : mf;
  const int sh = ef ? (static_cast<int>(ef) - 112 - E) : (-111 - E);
  const uint32_t mag = sh >= 0 ? (M << sh) : ((-sh >= 31) ? 0u : (M >> (-sh)));
  return (h & 0x8000u) ? -static_cast<int>(mag) : static_cast<int>(mag);
}

// Router fixed points (see k_router_prep): token rows keep 22 fraction bits
// below the row's top exponent, router rows 14; a logit is the exact integer
// dot product scaled by 2^(Ex - 22 + Ew - 14), rounded once to bfloat16.
constexpr int kRouterXBits = 22, kRouterWBits = 14;

// floor(log2) of a row's largest finite magnitude from its bfloat16
// magnitude bits (magnitudes order like their bit patterns); 0 for a zero row.
__device__ __forceinline__ int row_exponent(uint32_t mx) {
  if (mx == 0) return 0;
  return (mx >> 7) ? static_cast<int>(mx >> 7) - 127 : (31 - __clz(static_cast<int>(mx))) - 133;
}
// trunc(x * 2^(bits - E)) of one bfloat16 input x (bits h), E the row
// exponent (fixed_x is the integer form for bits = 22), through float32: the
// scale 2^(bits - E) = s1 * s2 (each a power of two), the product exact
// (|x * 2^(bits - E)| < 2^(bits + 1); a product that would drop below
// 2^-126 truncates to 0 either way), cvt.rzi truncates.  Non-finite inputs
// give 0.
struct FixScale {
  float s1, s2;
};
__device__ __forceinline__ FixScale fix_scale(int E, int bits) {
  const int k = bits - E;  // >= -113 for bfloat16 rows
  const int k1 = min(k, 127);
  return FixScale{__int_as_float((k1 + 127) << 23), __int_as_float((k - k1 + 127) << 23)};
}
__device__ __forceinline__ int fixed_qf(uint32_t h, FixScale sc) {
  if ((h & 0x7F80u) == 0x7F80u) return 0;
  return __float2int_rz(__fmul_rn(__fmul_rn(__uint_as_float(h << 16), sc.s1), sc.s2));
}

// Largest finite magnitude bits of 8 bfloat16 values; `bad` when one is not finite.
__device__ __forceinline__ uint32_t max_mag8(const uint4 v, bool &bad) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t mx = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t a = (w[e >> 1] >> (16 * (e & 1))) & 0x7FFFu;
    if (a >= 0x7F80u) bad = true;
    else mx = max(mx, a);
  }
  return mx;
}
// Router logit bits from the exact dot product S of the fixed points.
__device__ __forceinline__ uint16_t router_logit_bits(long long S, int ex, int ew) {
  return f64_to_bf16_once(ldexp(static_cast<double>(S), ex + ew - kRouterXBits - kRouterWBits));
}

// The same for one float32 input (bits), E the row exponent.
__device__ __forceinline__ int fixed_x32(uint32_t bits, int E) {
  const uint32_t ef = (bits >> 23) & 0xFFu, mf = bits & 0x7FFFFFu;
  if ((bits & 0x7FFFFFFFu) == 0 || ef == 255u) return 0;
  const uint32_t M = ef ? (mf | 0x800000u) : mf;
  const int sh = ef ? (static_cast<int>(ef) - 128 - E) : (-127 - E);
  const uint32_t mag = sh >= 0 ? (M << sh) : ((-sh >= 32) ? 0u : (M >> (-sh)));
  return (bits & 0x80000000u) ? -static_cast<int>(mag) : static_cast<int>(mag);
}

__device__ __forceinline__ uint32_t half_pair(int lo, int hi) {
  return static_cast<uint32_t>(__half_as_ushort(__int2half_rn(lo))) |
         (static_cast<uint32_t>(__half_as_ushort(__int2half_rn(hi))) << 16);
}

// TPR threads (a multiple of 32, <= 256) per row, RPC rows per CTA.  Thread
// tr of a row handles the 8-input slices tr, tr + TPR, ... (SPT of them;
// slice i covers inputs 8i..8i+7), all loaded up front.  The row's largest
// finite magnitude (bfloat16 magnitudes order like their bit patterns) is
// reduced over its warps through shared memory; then each slice's limbs go
// out as one 16-byte store per limb in fragment order
// [e0,e4,e1,e5,e2,e6,e3,e7], and each group's sum fl(SX) (G/8 consecutive
// slices = consecutive lanes) from a shuffle reduction.
// Body of the row fixed point for CTA `block` (TPR threads per row,
// blockDim.x / TPR rows per CTA); shared by k_prep_rows and the small-batch
// router launch, which runs it in extra CTAs.
template <int G, int SPT>
__device__ __forceinline__ void prep_rows_body(const uint16_t *rows, int n_rows, int K, int TPR, uint16_t *limbs,
                                               float *meta, uint32_t *err, int block,
                                               const uint32_t *skip_routes = nullptr, int n_skip = 0) {
  constexpr int LPG = G / 8;  // lanes per group
  __shared__ uint32_t s_mx[8][8];
  const int lane = threadIdx.x & 31;
  const int rl = threadIdx.x / TPR;  // row within the CTA
  const int tr = threadIdx.x - rl * TPR;
  const int wr = tr >> 5;            // warp within the row
  const int row = block * (blockDim.x / TPR) + rl;
  // rows of empty slots (route FNMOE_ROUTE_NONE; rows past n_skip have no
  // route) are neither read nor written: no kernel reads their limbs
  const bool live = row < n_rows && !(row < n_skip && __ldcg(skip_routes + row) == kRouteNone);
  const int Gc = K / G;
  const int slices = K / 8;
  const int mp = meta_pitch(Gc);
  const uint4 *src = reinterpret_cast<const uint4 *>(rows + static_cast<size_t>(live ? row : 0) * K);
  uint4 v[SPT];
#pragma unroll
  for (int k = 0; k < SPT; ++k) {
    const int i = tr + k * TPR;
    v[k] = (live && i < slices) ? src[i] : make_uint4(0u, 0u, 0u, 0u);
  }
  uint32_t mx = 0;
  bool bad = false;
#pragma unroll
  for (int k = 0; k < SPT; ++k) {
    const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t m = (w[e >> 1] >> (16 * (e & 1))) & 0x7FFFu;
      if (m >= 0x7F80u) bad = true;
      else mx = max(mx, m);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) set_error(err, kErrNonFinite);
  if (TPR > 32) {
    if (lane == 0) s_mx[rl][wr] = mx;
    __syncthreads();
    for (int q = 0; q < TPR / 32; ++q) mx = max(mx, s_mx[rl][q]);
  }
  if (!live) return;
  int E = 0;
  if (mx != 0) E = (mx >> 7) ? static_cast<int>(mx >> 7) - 127 : (31 - __clz(static_cast<int>(mx))) - 133;
  float *mrow = meta + static_cast<size_t>(row) * mp;
#pragma unroll
  for (int k = 0; k < SPT; ++k) {
    const int i = tr + k * TPR;
    int sx = 0;
    if (i < slices) {
      const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      int X[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        X[e] = fixed_x((w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu, E);
        sx += X[e];
      }
      int l0[8], l1[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        l1[e] = ((X[e] + 2048) & 4095) - 2048;
        l0[e] = (X[e] - l1[e]) >> 12;
      }
      const int g = (8 * i) / G;
      const int within = (8 * i) - g * G;
      uint16_t *dst = limbs + (static_cast<size_t>(row) * Gc + g) * 2 * G + within;
      *reinterpret_cast<uint4 *>(dst) = make_uint4(half_pair(l0[0], l0[4]), half_pair(l0[1], l0[5]),
                                                   half_pair(l0[2], l0[6]), half_pair(l0[3], l0[7]));
      *reinterpret_cast<uint4 *>(dst + G) = make_uint4(half_pair(l1[0], l1[4]), half_pair(l1[1], l1[5]),
                                                       half_pair(l1[2], l1[6]), half_pair(l1[3], l1[7]));
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) sx += __shfl_xor_sync(0xFFFFFFFFu, sx, off);
    if (i < slices && (lane & (LPG - 1)) == 0) mrow[(8 * i) / G] = __int2float_rn(sx);
  }
  if (tr == 0) {
    const int ai = meta_a_index(Gc);
    for (int g = Gc; g < ai; ++g) mrow[g] = 0.0f;
    const int k = E - 22;
    const int ka = max(k, -126);
    mrow[ai] = __int_as_float((ka + 127) << 23);          // A = 2^ka, normal
    mrow[ai + 1] = __int_as_float((k - ka + 127) << 23);  // B = 2^(k-ka) in [2^-29, 1]
    mrow[ai + 2] = 0.0f;
    mrow[ai + 3] = 0.0f;
  }
}

template <int G, int SPT>
__global__ void __launch_bounds__(256) k_prep_rows(const uint16_t *rows, int n_rows, int K, int TPR,
                                                   uint16_t *__restrict__ limbs, float *__restrict__ meta,
                                                   uint32_t *err, const uint32_t *skip_routes, int n_skip) {
  pdl_wait();
  pdl_trigger();
  prep_rows_body<G, SPT>(rows, n_rows, K, TPR, limbs, meta, err, blockIdx.x, skip_routes, n_skip);
}

// prep_rows_body for float32 rows: the same fixed point (trunc(x*2^(22-E)),
// E = floor(log2 max|x|) over the row's finite values), limbs and metadata.
// One thread per row slice of 8 inputs (TPR threads per row, as above).
template <int G, int SPT>
__global__ void __launch_bounds__(256) k_prep_rows_f32(const float *rows, int n_rows, int K, int TPR,
                                                       uint16_t *__restrict__ limbs, float *__restrict__ meta,
                                                       uint32_t *err, const uint32_t *skip_routes, int n_skip) {
  constexpr int LPG = G / 8;
  __shared__ uint32_t s_mx[8][8];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int rl = threadIdx.x / TPR;
  const int tr = threadIdx.x - rl * TPR;
  const int wr = tr >> 5;
  const int row = blockIdx.x * (blockDim.x / TPR) + rl;
  const bool live = row < n_rows && !(row < n_skip && __ldcg(skip_routes + row) == kRouteNone);
  const int Gc = K / G;
  const int slices = K / 8;
  const int mp = meta_pitch(Gc);
  const uint4 *src = reinterpret_cast<const uint4 *>(rows + static_cast<size_t>(live ? row : 0) * K);
  uint4 v[SPT][2];
#pragma unroll
  for (int q = 0; q < SPT; ++q) {
    const int i = tr + q * TPR;
    const bool ok = live && i < slices;
    v[q][0] = ok ? src[2 * i] : make_uint4(0u, 0u, 0u, 0u);
    v[q][1] = ok ? src[2 * i + 1] : make_uint4(0u, 0u, 0u, 0u);
  }
  uint32_t mx = 0;
  bool bad = false;
#pragma unroll
  for (int q = 0; q < SPT; ++q) {
    const uint32_t w[8] = {v[q][0].x, v[q][0].y, v[q][0].z, v[q][0].w, v[q][1].x, v[q][1].y, v[q][1].z, v[q][1].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t a = w[e] & 0x7FFFFFFFu;
      if (a >= 0x7F800000u) bad = true;
      else mx = max(mx, a);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) set_error(err, kErrNonFinite);
  if (TPR > 32) {
    if (lane == 0) s_mx[rl][wr] = mx;
    __syncthreads();
    for (int q = 0; q < TPR / 32; ++q) mx = max(mx, s_mx[rl][q]);
  }
  if (!live) return;
  int E = 0;
  if (mx != 0) E = (mx >> 23) ? static_cast<int>(mx >> 23) - 127 : (31 - __clz(static_cast<int>(mx))) - 149;
  float *mrow = meta + static_cast<size_t>(row) * mp;
#pragma unroll
  for (int q = 0; q < SPT; ++q) {
    const int i = tr + q * TPR;
    int sx = 0;
    if (i < slices) {
      const uint32_t w[8] = {v[q][0].x, v[q][0].y, v[q][0].z, v[q][0].w, v[q][1].x, v[q][1].y, v[q][1].z, v[q][1].w};
      int X[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        X[e] = fixed_x32(w[e], E);
        sx += X[e];
      }
      int l0[8], l1[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        l1[e] = ((X[e] + 2048) & 4095) - 2048;
        l0[e] = (X[e] - l1[e]) >> 12;
      }
      const int g = (8 * i) / G;
      const int within = (8 * i) - g * G;
      uint16_t *dst = limbs + (static_cast<size_t>(row) * Gc + g) * 2 * G + within;
      *reinterpret_cast<uint4 *>(dst) = make_uint4(half_pair(l0[0], l0[4]), half_pair(l0[1], l0[5]),
                                                   half_pair(l0[2], l0[6]), half_pair(l0[3], l0[7]));
      *reinterpret_cast<uint4 *>(dst + G) = make_uint4(half_pair(l1[0], l1[4]), half_pair(l1[1], l1[5]),
                                                       half_pair(l1[2], l1[6]), half_pair(l1[3], l1[7]));
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) sx += __shfl_xor_sync(0xFFFFFFFFu, sx, off);
    if (i < slices && (lane & (LPG - 1)) == 0) mrow[(8 * i) / G] = __int2float_rn(sx);
  }
  if (tr == 0) {
    const int ai = meta_a_index(Gc);
    for (int g = Gc; g < ai; ++g) mrow[g] = 0.0f;
    const int k = E - 22;
    const int ka = max(k, -126);
    mrow[ai] = __int_as_float((ka + 127) << 23);
    mrow[ai + 1] = __int_as_float((k - ka + 127) << 23);
    mrow[ai + 2] = 0.0f;
    mrow[ai + 3] = 0.0f;
  }
}

template <int G>
cudaError_t launch_prep_f32_g(const float *rows, int n_rows, int K, uint16_t *limbs, float *meta, cudaStream_t s,
                              const uint32_t *skip_routes, int n_skip) {
  const int slices = K / 8;
  const int tpr = std::min(256, ((slices + 31) / 32) * 32);
  const int spt = (slices + tpr - 1) / tpr;
  const int rpc = std::min(8, 256 / tpr);
  const int blocks = (n_rows + rpc - 1) / rpc;
  const int threads = rpc * tpr;
  uint32_t *err = device_error_word();
  cudaError_t e = cudaSuccess;
  if (spt == 1) e = launch_pdl(k_prep_rows_f32<G, 1>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else if (spt == 2) e = launch_pdl(k_prep_rows_f32<G, 2>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_prep_rows_f32(const float *rows, int n_rows, int K, int G, uint16_t *limbs, float *meta,
                                 cudaStream_t s, const uint32_t *skip_routes, int n_skip) {
  if (n_rows <= 0) return cudaSuccess;
  if (skip_routes == nullptr) n_skip = 0;
  return G == 32 ? launch_prep_f32_g<32>(rows, n_rows, K, limbs, meta, s, skip_routes, n_skip)
                 : launch_prep_f32_g<64>(rows, n_rows, K, limbs, meta, s, skip_routes, n_skip);
}

template <int G>
cudaError_t launch_prep_g(const uint16_t *rows, int n_rows, int K, uint16_t *limbs, float *meta, cudaStream_t s,
                          const uint32_t *skip_routes, int n_skip) {
  const int slices = K / 8;
  const int tpr = std::min(256, ((slices + 31) / 32) * 32);
  const int spt = (slices + tpr - 1) / tpr;
  const int rpc = std::min(8, 256 / tpr);
  const int blocks = (n_rows + rpc - 1) / rpc;
  const int threads = rpc * tpr;
  uint32_t *err = device_error_word();
  cudaError_t e = cudaSuccess;
  if (spt == 1) e = launch_pdl(k_prep_rows<G, 1>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else if (spt == 2) e = launch_pdl(k_prep_rows<G, 2>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else if (spt <= 4) e = launch_pdl(k_prep_rows<G, 4>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else if (spt <= 8) e = launch_pdl(k_prep_rows<G, 8>, blocks, threads, 0, s, rows, n_rows, K, tpr, limbs, meta, err, skip_routes, n_skip);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_prep_rows(const uint16_t *rows, int n_rows, int K, int G,
                             uint16_t *limbs, float *meta, cudaStream_t s, const uint32_t *skip_routes, int n_skip) {
  if (n_rows <= 0) return cudaSuccess;
  if (skip_routes == nullptr) n_skip = 0;
  return G == 32 ? launch_prep_g<32>(rows, n_rows, K, limbs, meta, s, skip_routes, n_skip)
                 : launch_prep_g<64>(rows, n_rows, K, limbs, meta, s, skip_routes, n_skip);
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

// Bin of a route value (see bin_of_pair): -3 empty slot, -1 bad route.
__device__ __forceinline__ int bin_of_route(uint32_t r, int E_arr, int records) {
  if (r == kRouteNone) return -3;
  if (r & kSlotBit) {
    const uint32_t slot = r & 0x7FFFFFFFu;
    return slot < static_cast<uint32_t>(records) ? E_arr + static_cast<int>(slot) : -1;
  }
  return r < static_cast<uint32_t>(E_arr) ? static_cast<int>(r) : -1;
}

__device__ __forceinline__ int bin_of_pair(const uint32_t *routes, int i, int n_pairs,
                                           int E_arr, int records, int n_bins) {
  if (i >= n_pairs) return n_bins - 1;  // shared expert bin
  const uint32_t r = __ldcg(routes + i);  // L2 load: routes may come from this same kernel
  if (r == kRouteNone) return -3;         // an empty slot: no bin, no error
  if (r & kSlotBit) {
    const uint32_t slot = r & 0x7FFFFFFFu;
    return slot < static_cast<uint32_t>(records) ? E_arr + static_cast<int>(slot) : -1;
  }
  return r < static_cast<uint32_t>(E_arr) ? static_cast<int>(r) : -1;
}

// Stable counting sort of the pairs by bin in one CTA.  The first `seg_warps`
// warps each own a contiguous segment of pair ids; a table of per-warp bin
// counts ([seg_warps][n_bins] in shared memory) turns into each
// warp's first write position inside every bin, so the segments scatter in
// parallel and pair order inside a bin is kept.  The 8-pair decode tiles are
// then written one per thread (bin found by binary search over the tile
// prefix), so a large bin is not left to one thread.
constexpr int kGroupUnroll = 4;

// Lanes holding the same key (0 <= key < 2^nbits): a ballot per key bit.
__device__ __forceinline__ unsigned match_key(int key, int nbits) {
  unsigned m = 0xFFFFFFFFu;
  for (int k = 0; k < nbits; ++k) {
    const bool bit = (key >> k) & 1;
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, bit);
    m &= bit ? bal : ~bal;
  }
  return m;
}

// One warp's segment [i0, i1): with order == nullptr, count pairs per bin into
// `row`; otherwise scatter them stably, `row` holding the warp's next write
// position inside each bin (relative to off[bin]).
__device__ __forceinline__ void group_walk(const uint32_t *routes, int n_pairs, int E_arr,
                                           int records, int n_bins, int i0, int i1, int *row,
                                           const int *off, int32_t *order, uint32_t *err) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  const int nbits = 32 - __clz(n_bins + 2);  // keys b + 3 for b in [-3, n_bins)
  for (int base = i0; base < i1; base += 32 * kGroupUnroll) {
    int b[kGroupUnroll];
#pragma unroll
    for (int u = 0; u < kGroupUnroll; ++u) {
      const int i = base + 32 * u + lane;
      b[u] = i < i1 ? bin_of_pair(routes, i, n_pairs, E_arr, records, n_bins) : -3;
    }
    if (order == nullptr) {
#pragma unroll
      for (int u = 0; u < kGroupUnroll; ++u) {
        if (b[u] >= 0) atomicAdd(&row[b[u]], 1);
        else if (b[u] == -1) set_error(err, kErrBadRoute);
      }
      continue;
    }
#pragma unroll
    for (int u = 0; u < kGroupUnroll; ++u) {
      const unsigned m = match_key(b[u] + 3, nbits);
      const bool leader = (m >> lane) == 1u;  // highest lane of its bin group
      int pos = 0;
      if (b[u] >= 0) pos = off[b[u]] + row[b[u]] + __popc(m & lt);
      __syncwarp();
      if (b[u] >= 0) {
        order[pos] = base + 32 * u + lane;
        if (leader) row[b[u]] += __popc(m);
      }
      __syncwarp();
    }
  }
}

// Body of the grouping (1024 threads); `sm` is group_smem_bytes() of shared memory.
__device__ __forceinline__ void group_body(const uint32_t *routes, int n_pairs,
                                           int shared_tokens, int E_arr, int records,
                                           const GroupView &gv, int seg_warps, uint32_t *err, int *sm) {
  const int n_bins = gv.n_bins;
  int *off = sm;                  // [n_bins + 1] first pair position of each bin
  int *first = sm + n_bins + 1;   // [n_bins + 1] first decode tile of each bin
  int *tbl = sm + 2 * (n_bins + 1);  // [seg_warps][n_bins]
  __shared__ int warp_sums[32];
  __shared__ int total_pairs, total_tiles;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int n_total = n_pairs + shared_tokens;
  const int seg = ((n_total + seg_warps - 1) / seg_warps + 31) & ~31;
  const int i0 = min(warp * seg, n_total), i1 = min(i0 + seg, n_total);
  for (int j = tid; j < seg_warps * n_bins; j += blockDim.x) tbl[j] = 0;
  __syncthreads();
  if (warp < seg_warps)
    group_walk(routes, n_pairs, E_arr, records, n_bins, i0, i1, tbl + warp * n_bins, nullptr, nullptr, err);
  __syncthreads();
  // per bin: total count, and each warp's exclusive prefix inside the bin
  for (int b = tid; b < n_bins; b += blockDim.x) {
    int c = 0;
    for (int w = 0; w < seg_warps; ++w) {
      const int v = tbl[w * n_bins + b];
      tbl[w * n_bins + b] = c;
      c += v;
    }
    off[b] = c;  // count for now
  }
  __syncthreads();
  // exclusive scans of counts and decode-tile counts over contiguous bin segments
  const int per = (n_bins + 1023) / 1024;
  const int b0 = min(tid * per, n_bins), b1 = min(b0 + per, n_bins);
  int local_c = 0, local_t = 0;
  for (int b = b0; b < b1; ++b) {
    local_c += off[b];
    local_t += (off[b] + kTokPerItem - 1) / kTokPerItem;
  }
  int pre_c = block_exclusive_scan_1024(local_c, warp_sums, &total_pairs);
  int pre_t = block_exclusive_scan_1024(local_t, warp_sums, &total_tiles);
  for (int b = b0; b < b1; ++b) {
    const int c = off[b];
    gv.counts[b] = c;
    gv.offsets[b] = pre_c;
    gv.bin_key[b] = (b < E_arr) ? static_cast<uint32_t>(b)
                    : (b < E_arr + records) ? (kSlotBit | static_cast<uint32_t>(b - E_arr))
                                            : kSharedKey;
    off[b] = pre_c;
    first[b] = pre_t;
    pre_c += c;
    pre_t += (c + kTokPerItem - 1) / kTokPerItem;
  }
  if (tid == 0) {
    off[n_bins] = total_pairs;
    first[n_bins] = total_tiles;
    gv.offsets[n_bins] = total_pairs;
    gv.n_tiles[0] = min(total_tiles, gv.max_tiles);
  }
  __syncthreads();
  if (warp < seg_warps)
    group_walk(routes, n_pairs, E_arr, records, n_bins, i0, i1, tbl + warp * n_bins, off, gv.order, err);
  __syncthreads();
  // self-contained decode tile descriptors: {route key, start, len, bin} and the pair ids
  const int n_tiles = min(total_tiles, gv.max_tiles);
  for (int t = tid; t < n_tiles; t += blockDim.x) {
    int lo = 0, hi = n_bins - 1;  // last bin with first[b] <= t (empty bins share their successor's start)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (first[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int b = lo;
    const int st = off[b] + (t - first[b]) * kTokPerItem;
    const int len = min(kTokPerItem, off[b + 1] - st);
    int p[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) p[q] = q < len ? gv.order[st + q] : -1;
    gv.tiles[3 * t] = make_int4(static_cast<int>(gv.bin_key[b]), st, len, b);
    gv.tiles[3 * t + 1] = make_int4(p[0], p[1], p[2], p[3]);
    gv.tiles[3 * t + 2] = make_int4(p[4], p[5], p[6], p[7]);
  }
}

__global__ void __launch_bounds__(1024) k_group(const uint32_t *routes, int n_pairs,
                                                int shared_tokens, int E_arr, int records,
                                                GroupView gv, int seg_warps, uint32_t *err) {
  extern __shared__ int sm[];
  pdl_wait();
  pdl_trigger();
  group_body(routes, n_pairs, shared_tokens, E_arr, records, gv, seg_warps, err, sm);
}

// Segment warps and shared-memory bytes of the grouping for n_total pairs.
size_t group_smem_bytes(int n_total, int n_bins, int *seg_warps_out) {
  constexpr size_t kBudget = 200 * 1024;
  const size_t fixed = static_cast<size_t>(n_bins + 1) * 2 * sizeof(int);
  const size_t per_warp = static_cast<size_t>(n_bins) * sizeof(int);
  int seg_warps = static_cast<int>(std::min<size_t>(32, (kBudget - std::min(fixed, kBudget)) / per_warp));
  seg_warps = std::max(1, std::min(seg_warps, (n_total + 31) / 32));
  *seg_warps_out = seg_warps;
  return fixed + static_cast<size_t>(seg_warps) * per_warp;
}

cudaError_t launch_group(const uint32_t *routes, int n_pairs, int shared_tokens,
                         int array_experts, int table_records, GroupView gv,
                         cudaStream_t s) {
  int seg_warps = 1;
  const size_t smem = group_smem_bytes(n_pairs + shared_tokens, gv.n_bins, &seg_warps);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_group, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = launch_pdl(k_group, 1, 1024, smem, s, routes, n_pairs, shared_tokens, array_experts,
                             table_records, gv, seg_warps, device_error_word());
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Grouping of many pairs over many CTAs (prefill-sized batches, no decode
// tiles): chunks of kGroupChunk pairs are counted per bin in parallel
// (k_group_count), one CTA turns the per-chunk counts into each chunk's first
// position inside every bin plus the bin counts and offsets (k_group_scan),
// and every chunk scatters its pairs stably with the per-warp segments of the
// single-CTA grouping (k_group_scatter).  Same order as k_group: by bin, then
// pair index.
constexpr int kGroupChunk = 4096;

__global__ void __launch_bounds__(1024) k_group_count(const uint32_t *routes, int n_pairs, int shared_tokens,
                                                      int E_arr, int records, int n_bins, int *hist, uint32_t *err) {
  extern __shared__ int cnt[];  // [n_bins]
  pdl_wait();
  pdl_trigger();
  const int n_total = n_pairs + shared_tokens;
  const int i0 = blockIdx.x * kGroupChunk, i1 = min(i0 + kGroupChunk, n_total);
  for (int b = threadIdx.x; b < n_bins; b += blockDim.x) cnt[b] = 0;
  __syncthreads();
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int b = bin_of_pair(routes, i, n_pairs, E_arr, records, n_bins);
    if (b >= 0) atomicAdd(&cnt[b], 1);
    else if (b == -1) set_error(err, kErrBadRoute);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < n_bins; b += blockDim.x) hist[static_cast<size_t>(blockIdx.x) * n_bins + b] = cnt[b];
}

__global__ void __launch_bounds__(1024) k_group_scan(int *hist, int chunks, int E_arr, int records, GroupView gv) {
  extern __shared__ int tot[];  // [n_bins]
  __shared__ int warp_sums[32];
  __shared__ int total_pairs;
  pdl_wait();
  pdl_trigger();
  const int n_bins = gv.n_bins, tid = threadIdx.x;
  for (int b = tid; b < n_bins; b += blockDim.x) {  // per bin: each chunk's exclusive prefix
    int run = 0;
    for (int c = 0; c < chunks; ++c) {
      const int v = hist[static_cast<size_t>(c) * n_bins + b];
      hist[static_cast<size_t>(c) * n_bins + b] = run;
      run += v;
    }
    tot[b] = run;
  }
  __syncthreads();
  const int per = (n_bins + 1023) / 1024;
  const int b0 = min(tid * per, n_bins), b1 = min(b0 + per, n_bins);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += tot[b];
  int pre = block_exclusive_scan_1024(local, warp_sums, &total_pairs);
  for (int b = b0; b < b1; ++b) {
    const int c = tot[b];
    gv.counts[b] = c;
    gv.offsets[b] = pre;
    gv.bin_key[b] = (b < E_arr) ? static_cast<uint32_t>(b)
                    : (b < E_arr + records) ? (kSlotBit | static_cast<uint32_t>(b - E_arr))
                                            : kSharedKey;
    tot[b] = pre;  // first position of the bin
    pre += c;
  }
  if (tid == 0) {
    gv.offsets[n_bins] = total_pairs;
    gv.n_tiles[0] = 0;  // no decode tiles from this grouping
  }
  __syncthreads();
  for (int b = tid; b < n_bins; b += blockDim.x)
    for (int c = 0; c < chunks; ++c) hist[static_cast<size_t>(c) * n_bins + b] += tot[b];
}

__global__ void __launch_bounds__(1024) k_group_scatter(const uint32_t *routes, int n_pairs, int shared_tokens,
                                                        int E_arr, int records, int n_bins, const int *hist,
                                                        int seg_warps, int32_t *order, uint32_t *err) {
  extern __shared__ int sm[];
  int *base = sm;            // [n_bins] this chunk's first position inside each bin
  int *tbl = sm + n_bins;    // [seg_warps][n_bins]
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5;
  const int n_total = n_pairs + shared_tokens;
  const int c0 = blockIdx.x * kGroupChunk, c1 = min(c0 + kGroupChunk, n_total);
  const int seg = ((c1 - c0 + seg_warps - 1) / seg_warps + 31) & ~31;
  const int i0 = min(c0 + warp * seg, c1), i1 = min(i0 + seg, c1);
  for (int b = tid; b < n_bins; b += blockDim.x) base[b] = hist[static_cast<size_t>(blockIdx.x) * n_bins + b];
  for (int j = tid; j < seg_warps * n_bins; j += blockDim.x) tbl[j] = 0;
  __syncthreads();
  if (warp < seg_warps)
    group_walk(routes, n_pairs, E_arr, records, n_bins, i0, i1, tbl + warp * n_bins, nullptr, nullptr, err);
  __syncthreads();
  for (int b = tid; b < n_bins; b += blockDim.x) {
    int run = 0;
    for (int w = 0; w < seg_warps; ++w) {
      const int v = tbl[w * n_bins + b];
      tbl[w * n_bins + b] = run;
      run += v;
    }
  }
  __syncthreads();
  if (warp < seg_warps)
    group_walk(routes, n_pairs, E_arr, records, n_bins, i0, i1, tbl + warp * n_bins, base, order, err);
}

cudaError_t launch_group_large(const uint32_t *routes, int n_pairs, int shared_tokens, int array_experts,
                               int table_records, GroupView gv, int *hist, size_t hist_bytes, cudaStream_t s) {
  const int n_total = n_pairs + shared_tokens;
  const int chunks = (n_total + kGroupChunk - 1) / kGroupChunk;
  const int n_bins = gv.n_bins;
  if (chunks == 0 || hist == nullptr) return cudaErrorNotSupported;
  if (static_cast<size_t>(chunks) * n_bins * sizeof(int) > hist_bytes) return cudaErrorNotSupported;
  constexpr size_t kBudget = 200 * 1024;
  const size_t per_bins = static_cast<size_t>(n_bins) * sizeof(int);
  if (per_bins * 2 > kBudget) return cudaErrorNotSupported;
  const int seg_warps = static_cast<int>(std::min<size_t>(32, (kBudget - per_bins) / per_bins));
  const size_t scatter_smem = per_bins * (1 + seg_warps);
  cudaError_t e;
  if (per_bins > 48 * 1024) {
    e = cudaFuncSetAttribute(k_group_count, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(per_bins));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_group_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(per_bins));
    if (e != cudaSuccess) return e;
  }
  if (scatter_smem > 48 * 1024) {
    e = cudaFuncSetAttribute(k_group_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(scatter_smem));
    if (e != cudaSuccess) return e;
  }
  uint32_t *err = device_error_word();
  e = launch_pdl(k_group_count, chunks, 1024, per_bins, s, routes, n_pairs, shared_tokens, array_experts,
                 table_records, n_bins, hist, err);
  if (e != cudaSuccess) return e;
  e = launch_pdl(k_group_scan, 1, 1024, per_bins, s, hist, chunks, array_experts, table_records, gv);
  if (e != cudaSuccess) return e;
  e = launch_pdl(k_group_scatter, chunks, 1024, scatter_smem, s, routes, n_pairs, shared_tokens, array_experts,
                 table_records, n_bins, static_cast<const int *>(hist), seg_warps, gv.order, err);
  if (e != cudaSuccess) return e;
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
// Work item = (expert bin tile of up to kTokPerItem pairs, ROWS output rows).
// A CTA takes a contiguous range of items, so consecutive items usually share
// their tile and its staged activations (limbs + metadata, one shared-memory
// stage reloaded only when the tile changes).  Each warp owns RPW output rows
// over the full contraction width, one float32 accumulator per (row, token),
// and streams its packed rows, scales and biases through a private R-stage
// shared-memory ring, up to R-1 blocks ahead and across item boundaries.  A
// block is 128 bytes (256 inputs) of each of the warp's 16 MMA rows plus
// their scales and biases.
//
// Two weight layouts feed the ring:
//  * arrays / table records in the reference layout (packed rows
//    [rows][K/8] uint32, scales/biases [rows][K/G] bf16): every lane copies
//    its share with 16-byte cp.async (per-lane copy groups);
//  * tiled tables (fnmoe_tile_experts): each (16-row group, block) is one
//    contiguous 2560-byte chunk, already in fragment order, which lane 0
//    moves with one bulk copy (cp.async.bulk, no multicast) completing on the
//    stage's mbarrier.
//
// MMA row mapping: DUAL (gate/up) -- M rows 0-7 are 8 gate rows and M rows
// 8-15 the same 8 up rows, so a thread ends with gate and up of the same
// (row, token) and applies SwiGLU in registers.  Single (down) -- M rows
// 0-7 and 8-15 are 16 consecutive output rows.  N = 4 tokens x 2 limbs.

constexpr int kBlkBytes = 128;                // packed bytes per row per block
constexpr int kRowPitch = kBlkBytes + 16;     // generic layout: padded rows, conflict-free reads
constexpr int kSBOff = 16 * kRowPitch;        // generic layout: [16 rows][scales 16 B | biases 16 B]
constexpr int kStageBytes = kSBOff + 16 * 32;
constexpr uint32_t kSpinLimit = 1u << 20;     // mbarrier polls before a wait gives up

struct XStage {
  int Gc;      // groups along the contraction width
  int Xrow;    // limb bytes per pair
  int Mp;      // metadata bytes per pair: fl(SX) per group, then {A, B}
  int a_off;   // byte offset of {A, B} in a metadata row
  int m_off;   // metadata offset in the stage
  int bytes;   // stage size
};

__host__ __device__ inline XStage xstage_geom(int K, int G) {
  XStage s{};
  s.Gc = K / G;
  s.Xrow = s.Gc * 4 * G;
  s.Mp = meta_pitch(s.Gc) * 4;
  s.a_off = meta_a_index(s.Gc) * 4;
  s.m_off = kTokPerItem * s.Xrow;
  s.bytes = ((s.m_off + kTokPerItem * s.Mp + 127) / 128) * 128;
  return s;
}

struct RawDesc {
  int4 d0, d1, d2;
};

__device__ __forceinline__ RawDesc load_desc(const GroupView &gv, int tile) {
  RawDesc r{};
  if (tile >= 0) {
    r.d0 = gv.tiles[3 * tile];
    r.d1 = gv.tiles[3 * tile + 1];
    r.d2 = gv.tiles[3 * tile + 2];
  }
  return r;
}

struct ItemInfo {
  bool ok;      // expert data resolved and this warp's rows exist
  int len, rt;  // pairs in the tile, row tile
};

// This lane's copy sources for one item.  Generic layout: the packed row of
// MMA row lane % 16 and the scale (lanes 0-15) or bias (lanes 16-31) row of
// MMA row lane % 16.  Tiled layout: w is the warp's first chunk.
struct Src {
  const uint8_t *w, *sb;
};

// Record of a tiled route key: routed experts map to their index, the shared
// expert to the last record.
__device__ __forceinline__ bool tiled_record(const ExpertCallArgs &a, uint32_t key, uint32_t &rec) {
  if (key == kSharedKey) {
    if (!a.tiled.has_shared) return false;
    rec = a.tiled.records - 1;
    return true;
  }
  if (key >= static_cast<uint32_t>(a.array_experts)) return false;
  rec = key;
  return true;
}

// Resolve item `item` (tile descriptor rd) into its info and this lane's
// copy sources.
template <bool DUAL, bool TILED>
__device__ __forceinline__ ItemInfo item_setup(const ExpertCallArgs &a, const RawDesc &rd, int rt, int rows_per_tile,
                                               int wbase, int O, int K, int Gc, int nblk, int lane, Src &src) {
  ItemInfo it{};
  src = Src{nullptr, nullptr};
  it.rt = rt;
  it.len = rd.d0.z;
  const uint32_t key = static_cast<uint32_t>(rd.d0.x);
  const int o_base = it.rt * rows_per_tile + wbase;
  if (TILED) {
    uint32_t rec = 0;
    it.ok = tiled_record(a, key, rec);
    if (!it.ok) return it;
    const int rg = DUAL ? o_base / 8 : o_base / 16;
    const uint8_t *base = DUAL ? a.tiled.gate_up + rec * a.tiled.gate_up_record
                               : a.tiled.down + rec * a.tiled.down_record;
    src.w = base + static_cast<size_t>(rg) * nblk * kTileChunk;
    return it;
  }
  Ptrs p[2];
  if (DUAL) {
    it.ok = resolve(a, key, 0, O, K, p[0]) && resolve(a, key, 1, O, K, p[1]);
  } else {
    it.ok = resolve(a, key, 2, O, K, p[0]);
    p[1] = p[0];
  }
  if (!it.ok) return it;
  const int mrow = lane & 15;
  const int row = DUAL ? min(o_base + (mrow & 7), O - 1) : min(o_base + mrow, O - 1);
  const Ptrs &pp = (DUAL && mrow >= 8) ? p[1] : p[0];
  src.w = reinterpret_cast<const uint8_t *>(pp.w) + static_cast<size_t>(row) * (K / 2);
  const uint16_t *base = (lane >> 4) ? pp.b : pp.s;
  src.sb = reinterpret_cast<const uint8_t *>(base + static_cast<size_t>(row) * Gc);
  return it;
}

// Per-warp ring state.  Blocks are numbered in consumption order across
// items; block n lives in stage n % R.
struct Ring {
  uint8_t *base;
  uint64_t *bars;  // R mbarriers (tiled layout)
  int fetched;     // blocks issued
  int consumed;    // blocks computed
  int f_next;      // 0: the fetch cursor is in the current item, 1: in the next
  int f_blk;       // next block of that item to fetch
  int f_stage;     // fetched % R
  int c_stage;     // consumed % R
  uint32_t phase;  // bit s: parity of stage s's next completion
  bool dead;       // a wait gave up: skip waits, results are void
};

// Scale/bias copy modes of the generic layout.
enum SBMode { kSB16 = 0, kSB4 = 1, kSBSync = 2 };

// Issue the copies of block fb of an item into stage st.
template <int G, bool TILED>
__device__ __forceinline__ void issue_block(uint8_t *st, uint64_t *bar, const Src &src, int fb, int lane,
                                            int rowbytes, int Gc, int sb_mode) {
  if (TILED) {
    if (lane == 0) {
      fence_proxy_async();
      mbar_expect_tx(bar, kTileChunk);
      bulk_g2s(st, src.w + static_cast<size_t>(fb) * kTileChunk, kTileChunk, bar);
    }
    return;
  }
  constexpr int GPB = 2 * kBlkBytes / G;
  // packed rows: lane copies 64 bytes (half h) of MMA row lane % 16
  const int row = lane & 15, h = lane >> 4;
  const int off = fb * kBlkBytes + h * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (off + 16 * i < rowbytes) cp_async16(st + row * kRowPitch + h * 64 + 16 * i, src.w + off + 16 * i);
  uint8_t *d = st + kSBOff + row * 32 + h * 16;
  const int g0 = fb * GPB;
  if (sb_mode == kSB16) {
    cp_async16(d, src.sb + 2 * g0);  // GPB == 8: one piece, always full
  } else if (sb_mode == kSB4) {
#pragma unroll
    for (int p = 0; p < GPB / 2; ++p)
      if (g0 + 2 * p < Gc) cp_async4(d + 4 * p, src.sb + 2 * (g0 + 2 * p));
  } else {
#pragma unroll
    for (int j = 0; j < GPB; ++j)
      if (g0 + j < Gc)
        *reinterpret_cast<uint16_t *>(d + 2 * j) = ldg_u16(reinterpret_cast<const uint16_t *>(src.sb) + g0 + j);
  }
  cp_async_commit();
}

// Keep up to R blocks (the one being computed included) in the ring.
template <int G, int R, bool TILED>
__device__ __forceinline__ void ring_fill(Ring &rg, const Src &sc, const Src &sn, int nb_cur, int nb_nxt,
                                          int lane, int rowbytes, int Gc, int sb_mode) {
  while (rg.fetched - rg.consumed < R) {
    if (rg.f_next == 0 && rg.f_blk >= nb_cur) {
      rg.f_next = 1;
      rg.f_blk = 0;
    }
    if (rg.f_next == 1 && rg.f_blk >= nb_nxt) break;
    issue_block<G, TILED>(rg.base + rg.f_stage * kStageBytes, rg.bars + rg.f_stage, rg.f_next ? sn : sc, rg.f_blk,
                          lane, rowbytes, Gc, sb_mode);
    ++rg.f_blk;
    ++rg.fetched;
    if (++rg.f_stage == R) rg.f_stage = 0;
  }
}

// Wait for block rg.consumed (stage rg.c_stage).  A wait that gives up sets
// the timeout flag and marks the warp dead: later waits return at once.
template <bool TILED>
__device__ __forceinline__ void ring_wait(Ring &rg, uint32_t *err) {
  if (!TILED) {
    cp_async_wait_dyn(rg.fetched - rg.consumed - 1);
  } else if (!rg.dead) {
    const unsigned parity = (rg.phase >> rg.c_stage) & 1u;
    uint32_t spins = 0;
    while (!mbar_try_wait(rg.bars + rg.c_stage, parity)) {
      if (++spins >= kSpinLimit) {
        rg.dead = true;
        set_error(err, kErrTimeout);
        break;
      }
    }
    rg.phase ^= 1u << rg.c_stage;
  }
  __syncwarp();
}

// Stage the activation limbs and metadata of a tile's pairs (all threads) and
// its pair ids.  Slots past the tile's length keep stale data: they only feed
// MMA columns (and accumulators) whose results are never stored.
__device__ __forceinline__ void load_xstage(uint8_t *st, int *s_pairs, const XStage &xs, const RawDesc &rd, bool ok,
                                            const uint16_t *xl, const float *xm,
                                            int n_pairs, int slots, bool by_token) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int cpx = xs.Xrow / 16, cpm = xs.Mp / 16;
  const int len = rd.d0.z;
  const int pairs[kTokPerItem] = {rd.d1.x, rd.d1.y, rd.d1.z, rd.d1.w, rd.d2.x, rd.d2.y, rd.d2.z, rd.d2.w};
#pragma unroll
  for (int q = 0; q < kTokPerItem; ++q) {
    if (tid == q) s_pairs[q] = pairs[q];
    uint8_t *dst = st + q * xs.Xrow;
    uint8_t *mdst = st + xs.m_off + q * xs.Mp;
    if (ok && q < len) {
      const int pair = pairs[q];
      const int row = by_token ? token_of_pair(pair, n_pairs, slots) : pair;
      const uint8_t *src = reinterpret_cast<const uint8_t *>(xl) + static_cast<size_t>(row) * xs.Xrow;
      const uint8_t *msrc = reinterpret_cast<const uint8_t *>(xm) + static_cast<size_t>(row) * xs.Mp;
      for (int cc = tid; cc < cpx; cc += nt) cp_async16(dst + cc * 16, src + cc * 16);
      for (int cc = tid; cc < cpm; cc += nt) cp_async16(mdst + cc * 16, msrc + cc * 16);
    }
  }
}

// bfloat16 j (0-3) of two packed words as float32.
__device__ __forceinline__ float bf16_at(const uint2 &v, int j) {
  const uint32_t w = j < 2 ? v.x : v.y;
  return __uint_as_float((j & 1) ? (w & 0xFFFF0000u) : (w << 16));
}

__device__ __forceinline__ uint32_t word_at(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ float f_at(const float4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One group against NT token tiles: MMA the two rows' nibbles with the
// token limbs, fold S and SX into the accumulators.
template <int G, int NT>
__device__ __forceinline__ void group_step(const uint32_t (&qa)[G / 32], const uint32_t (&qb)[G / 32], float sA,
                                           float bA, float sB, float bB, uint32_t xgj, int xstep,
                                           const float (&fs)[NT], float (&accA)[NT], float (&accB)[NT]) {
  constexpr int WB = G / 32;
  uint32_t A0[WB][4], A1[WB][4];
#pragma unroll
  for (int wb = 0; wb < WB; ++wb) nibble_operands(qa[wb], qb[wb], A0[wb], A1[wb]);
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float C[4];
#pragma unroll
    for (int wb = 0; wb < WB; ++wb) {
      const uint4 v = lds128(xgj + t * xstep + wb * 64);
      if (wb == 0) mma_16816_z(C, A0[wb], v.x, v.y);
      else mma_16816(C, A0[wb], v.x, v.y);
      mma_16816(C, A1[wb], v.z, v.w);
    }
    const float SA = __fmaf_rn(C[0], 4096.0f, C[1]);
    const float SB = __fmaf_rn(C[2], 4096.0f, C[3]);
    accA[t] = __fmaf_rn(bA, fs[t], __fmaf_rn(sA, SA, accA[t]));
    accB[t] = __fmaf_rn(bB, fs[t], __fmaf_rn(sB, SB, accB[t]));
  }
}

// One ring block: GPB groups of the warp's 16 MMA rows against NT token
// tiles, in halves (scales, biases and group sums of one half live in
// registers at a time).  TAIL blocks stop at the last group.
template <int G, int NT, bool TAIL, bool TILED>
__device__ __forceinline__ void compute_block(uint32_t st, uint32_t xg, uint32_t mg, int xstep, int mstep, int g0,
                                              int Gc, int r, int c, float (&accA)[NT], float (&accB)[NT]) {
  constexpr int WB = G / 32;
  constexpr int GPB = 2 * kBlkBytes / G;
  constexpr int QG = GPB / 2;  // groups per half
  const uint32_t sbA = st + (TILED ? kTileW : kSBOff) + r * 32;
  const uint32_t sbB = sbA + 8 * 32;
  const uint32_t wq = TILED ? st + (r * 4 + c) * 16 : st + r * kRowPitch + c * 4;
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const int gh = h * QG;
    if (TAIL && g0 + gh >= Gc) break;
    uint2 sA2, bA2, sB2, bB2;
    if (QG == 4) {
      sA2 = lds64(sbA + 2 * gh);
      bA2 = lds64(sbA + 16 + 2 * gh);
      sB2 = lds64(sbB + 2 * gh);
      bB2 = lds64(sbB + 16 + 2 * gh);
    } else {
      sA2 = make_uint2(lds32(sbA + 2 * gh), 0u);
      bA2 = make_uint2(lds32(sbA + 16 + 2 * gh), 0u);
      sB2 = make_uint2(lds32(sbB + 2 * gh), 0u);
      bB2 = make_uint2(lds32(sbB + 16 + 2 * gh), 0u);
    }
    float4 fsx[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (QG == 4) {
        const uint4 f = lds128(mg + t * mstep + 4 * gh);
        fsx[t] = make_float4(__uint_as_float(f.x), __uint_as_float(f.y), __uint_as_float(f.z), __uint_as_float(f.w));
      } else {
        const uint2 f = lds64(mg + t * mstep + 4 * gh);
        fsx[t] = make_float4(__uint_as_float(f.x), __uint_as_float(f.y), 0.0f, 0.0f);
      }
    }
    uint4 wA4 = make_uint4(0u, 0u, 0u, 0u), wB4 = make_uint4(0u, 0u, 0u, 0u);
    if (TILED) {
      // fragment-ordered chunk: [half][A/B][slot r*4+c][4 words]
      wA4 = lds128(wq + (2 * h) * 512);
      wB4 = lds128(wq + (2 * h + 1) * 512);
    }
#pragma unroll
    for (int j = 0; j < QG; ++j) {
      if (TAIL && g0 + gh + j >= Gc) break;
      uint32_t qa[WB], qb[WB];
#pragma unroll
      for (int wb = 0; wb < WB; ++wb) {
        if (TILED) {
          qa[wb] = word_at(wA4, j * WB + wb);
          qb[wb] = word_at(wB4, j * WB + wb);
        } else {
          const int off = (gh + j) * (G / 2) + wb * 16;
          qa[wb] = lds32(wq + off);
          qb[wb] = lds32(wq + 8 * kRowPitch + off);
        }
      }
      float fs[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) fs[t] = f_at(fsx[t], j);
      group_step<G, NT>(qa, qb, bf16_at(sA2, j), bf16_at(bA2, j), bf16_at(sB2, j), bf16_at(bB2, j),
                        xg + (gh + j) * (4 * G), xstep, fs, accA, accB);
    }
  }
}

// Epilogue of one (pair, row pair): bfloat16 activations -- gate/up rounded
// to bfloat16, the bfloat16 SwiGLU sequence, bfloat16 stores -- or, with
// float32 activations (a.f32), the same in float32 into float32 rows.
// DUAL: yA = gate and yB = up of row oA; else yA, yB = rows oA, oB.
template <bool DUAL>
__device__ __forceinline__ void store_rows(const ExpertCallArgs &a, int pair, int O, int oA, int oB, float yA,
                                           float yB, uint16_t *out, uint16_t *g_out, uint16_t *u_out) {
  const size_t base = static_cast<size_t>(pair) * O;
  if (a.f32) {
    float *o = reinterpret_cast<float *>(out);
    if (DUAL) {
      if (oA < O) {
        o[base + oA] = swiglu_f32(yA, yB);
        if (g_out != nullptr && pair < a.n_pairs) {
          reinterpret_cast<float *>(g_out)[base + oA] = yA;
          reinterpret_cast<float *>(u_out)[base + oA] = yB;
        }
      }
    } else {
      if (oA < O) o[base + oA] = yA;
      if (oB < O) o[base + oB] = yB;
    }
    return;
  }
  if (DUAL) {
    if (oA < O) {
      const float gvv = round_bf16(yA), uvv = round_bf16(yB);
      out[base + oA] = f32_to_bf16(swiglu_bf16(g_exp_bf16, gvv, uvv));
      if (g_out != nullptr && pair < a.n_pairs) {
        g_out[base + oA] = f32_to_bf16(gvv);
        u_out[base + oA] = f32_to_bf16(uvv);
      }
    }
  } else {
    if (oA < O) out[base + oA] = f32_to_bf16(yA);
    if (oB < O) out[base + oB] = f32_to_bf16(yB);
  }
}

// Compute one item's rows for NT token tiles (4 pairs each) and write them.
template <int G, int WARPS, bool DUAL, int R, bool TILED, int NT>
__device__ __forceinline__ void run_item(const ExpertCallArgs &a, const ItemInfo &cur, const uint8_t *xst,
                                         const int *s_pairs, const XStage &xs, int O, int K, int nblk, Ring &rg,
                                         const Src &sc, const Src &sn, int nb_nxt, int sb_mode, uint32_t *err,
                                         uint16_t *__restrict__ out, uint16_t *__restrict__ g_out,
                                         uint16_t *__restrict__ u_out) {
  constexpr int GPB = 2 * kBlkBytes / G;
  constexpr int RPW = DUAL ? 8 : 16;
  constexpr int ROWS = RPW * WARPS;
  const int Gc = xs.Gc;
  const int rowbytes = K / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int o0 = cur.rt * ROWS + warp * RPW + r;
  const int oA = o0;
  const int oB = DUAL ? o0 : o0 + 8;
  const uint32_t xs0 = smem_u32(xst);
  const uint32_t xb = xs0 + (r >> 1) * xs.Xrow + (r & 1) * (G * 2) + c * 16;
  const uint32_t mrow = xs0 + xs.m_off + c * xs.Mp;
  const uint32_t ring0 = smem_u32(rg.base);
  const int xstep = 4 * xs.Xrow, mstep = 4 * xs.Mp;
  const int full = Gc / GPB;  // blocks without a tail
  float accA[NT], accB[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) accA[t] = accB[t] = -0.0f;
#pragma unroll 1
  for (int cb = 0; cb < nblk; ++cb) {
    if (rg.fetched == rg.consumed) {  // nothing in flight (the previous item was skipped): fetch now
      __syncwarp();
      ring_fill<G, R, TILED>(rg, sc, sn, nblk, nb_nxt, lane, rowbytes, Gc, sb_mode);
    }
    ring_wait<TILED>(rg, err);  // block rg.consumed landed; all lanes are done with the previous one
    const uint32_t st = ring0 + rg.c_stage * kStageBytes;
    ring_fill<G, R, TILED>(rg, sc, sn, nblk, nb_nxt, lane, rowbytes, Gc, sb_mode);
    const int g0 = cb * GPB;
    if (cb < full)
      compute_block<G, NT, false, TILED>(st, xb + g0 * (4 * G), mrow + g0 * 4, xstep, mstep, g0, Gc, r, c, accA,
                                         accB);
    else
      compute_block<G, NT, true, TILED>(st, xb + g0 * (4 * G), mrow + g0 * 4, xstep, mstep, g0, Gc, r, c, accA,
                                        accB);
    ++rg.consumed;
    if (++rg.c_stage == R) rg.c_stage = 0;
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int q = 4 * t + c;
    if (q < cur.len) {
      const int pair = s_pairs[q];
      const uint2 abw = lds64(mrow + t * mstep + xs.a_off);
      const float2 ab = make_float2(__uint_as_float(abw.x), __uint_as_float(abw.y));
      const float yA = __fmul_rn(__fmul_rn(accA[t], ab.x), ab.y);
      const float yB = __fmul_rn(__fmul_rn(accB[t], ab.x), ab.y);
      store_rows<DUAL>(a, pair, O, oA, oB, yA, yB, out, g_out, u_out);
    }
  }
}

// Tiles are visited in the order t = (pos * P) mod n_tiles, P a prime not
// dividing n_tiles (a bijection).  Bins come sorted by key with the shared
// expert's tiles -- all of them full -- last, so walking them in plain order
// would hand a few CTAs the heaviest items; the stride spreads them over the
// contiguous item ranges.
__device__ __forceinline__ int tile_stride(int n) {
  const int primes[6] = {97, 89, 83, 79, 73, 71};
#pragma unroll
  for (int i = 0; i < 6; ++i)
    if (n % primes[i] != 0) return primes[i] % max(n, 1);
  return 1;
}

template <int G, int WARPS, bool DUAL, int R, bool TILED>
__global__ void __launch_bounds__(WARPS * 32, 1) k_expert_rows(ExpertCallArgs a, GroupView gv,
                                                               const uint16_t *xl,
                                                               const float *xm,
                                                               uint16_t *__restrict__ out,
                                                               uint16_t *__restrict__ g_out,
                                                               uint16_t *__restrict__ u_out, int sb_mode,
                                                               uint32_t *err) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPW = DUAL ? 8 : 16;
  constexpr int ROWS = RPW * WARPS;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = DUAL ? a.H : a.I;
  const int O = DUAL ? a.I : a.H;
  const XStage xs = xstage_geom(K, G);
  const int row_tiles = (O + ROWS - 1) / ROWS;
  const int n_items = gv.n_tiles[0] * row_tiles;
  if (n_items == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rowbytes = K / 2;
  const int nblk = (rowbytes + kBlkBytes - 1) / kBlkBytes;
  const int wbase = warp * RPW;
  uint8_t *ring_base = smem + xs.bytes + warp * R * kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + xs.bytes + WARPS * R * kStageBytes) + warp * R;
  int *s_pairs = reinterpret_cast<int *>(smem + xs.bytes + WARPS * R * (kStageBytes + 8));
  if (TILED) {
    if (lane == 0) {
      for (int i = 0; i < R; ++i) mbar_init(bars + i, 1);
      mbar_init_fence();
    }
    __syncwarp();
  }
  Ring rg{ring_base, bars, 0, 0, 0, 0, 0, 0, 0u, false};

  // Tiled tables hold whole row groups only: a warp whose rows start past
  // the last row has nothing to do (len -1 marks it: no bad-route error).
  //
  // Tiled tables: every warp asks L2 for its item's whole row-group range at
  // setup (one bulk prefetch), so all of an item's blocks are in flight at
  // once and the ring's copies find them in L2.  Not in the 16-warp gate/up
  // kernel: there the rings alone keep enough bytes in flight, and the
  // prefetch one item ahead added ~38% DRAM re-reads (lines evicted before
  // their ring copy) at the 64-token layer.  Small batches (4-warp CTAs, few
  // experts) also prefetch, from the gate/up kernel, the row tile's share of
  // the same expert's down record, which the down kernel then reads from L2.
  auto setup = [&](const RawDesc &rd, int rt, Src &src) {
    ItemInfo it = item_setup<DUAL, TILED>(a, rd, rt, ROWS, wbase, O, K, xs.Gc, nblk, lane, src);
    if (TILED && it.rt * ROWS + wbase >= O) {
      it.ok = false;
      it.len = -1;
      src = Src{nullptr, nullptr};
    }
    if (TILED && (WARPS <= 4 || !DUAL) && it.ok && lane == 0) {
      bulk_prefetch_l2(src.w, static_cast<unsigned>(nblk) * kTileChunk);
      uint32_t rec = 0;
      if (DUAL && WARPS <= 4 && warp == 0 && a.tiled.down != nullptr &&
          tiled_record(a, static_cast<uint32_t>(rd.d0.x), rec)) {
        const uint64_t slice = (a.tiled.down_record / row_tiles) & ~static_cast<uint64_t>(15);
        const uint64_t lo = slice * it.rt;
        const uint64_t hi = it.rt == row_tiles - 1 ? a.tiled.down_record : lo + slice;
        if (hi > lo) bulk_prefetch_l2(a.tiled.down + rec * a.tiled.down_record + lo, static_cast<unsigned>(hi - lo));
      }
    }
    return it;
  };

  // Each CTA takes a contiguous range of items: consecutive items usually
  // share a tile and its staged activations.  Item cursors (row tile, tile)
  // advance incrementally; tiles follow the stride order of tile_stride.
  const int i0 = static_cast<int>(static_cast<long long>(n_items) * blockIdx.x / gridDim.x);
  const int i1 = static_cast<int>(static_cast<long long>(n_items) * (blockIdx.x + 1) / gridDim.x);
  if (i0 >= i1) return;
  const int n_tiles = gv.n_tiles[0];
  const int stride = tile_stride(n_tiles);
  struct Cursor {
    int rt, tile;
  };
  auto advance = [&](Cursor c) {
    if (++c.rt == row_tiles) {
      c.rt = 0;
      c.tile += stride;
      if (c.tile >= n_tiles) c.tile -= n_tiles;
    }
    return c;
  };
  const int pos0 = i0 / row_tiles;
  Cursor c_cur{i0 - pos0 * row_tiles, static_cast<int>((static_cast<long long>(pos0) * stride) % n_tiles)};
  Cursor c_nxt = advance(c_cur);
  Cursor c_nn = advance(c_nxt);

  Src sc, sn;
  const RawDesc rd0 = load_desc(gv, c_cur.tile);
  ItemInfo cur = setup(rd0, c_cur.rt, sc);
  RawDesc rd_nxt = load_desc(gv, i0 + 1 < i1 ? c_nxt.tile : -1);
  int4 d0_nn = i0 + 2 < i1 ? gv.tiles[3 * c_nn.tile] : make_int4(0, 0, 0, 0);
  ItemInfo nxt{};
  sn = Src{nullptr, nullptr};
  if (i0 + 1 < i1) nxt = setup(rd_nxt, c_nxt.rt, sn);
  int nb_cur = cur.ok ? nblk : 0;
  int nb_nxt = nxt.ok ? nblk : 0;

  // tiled weight blocks (bulk copies on mbarriers) start before the
  // activation stage lands; the generic layout shares the cp.async groups
  if (TILED) ring_fill<G, R, TILED>(rg, sc, sn, nb_cur, nb_nxt, lane, rowbytes, xs.Gc, sb_mode);
  load_xstage(smem, s_pairs, xs, rd0, rd0.d0.z > 0, xl, xm, a.n_pairs, a.slots, DUAL);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  if (!TILED) ring_fill<G, R, TILED>(rg, sc, sn, nb_cur, nb_nxt, lane, rowbytes, xs.Gc, sb_mode);

  for (int item = i0; item < i1; ++item) {
    if (!cur.ok) {
      if (cur.len >= 0 && lane == 0) set_error(err, kErrBadRoute);
    } else if (cur.len > 4) {
      run_item<G, WARPS, DUAL, R, TILED, 2>(a, cur, smem, s_pairs, xs, O, K, nblk, rg, sc, sn, nb_nxt, sb_mode, err,
                                            out, g_out, u_out);
    } else {
      run_item<G, WARPS, DUAL, R, TILED, 1>(a, cur, smem, s_pairs, xs, O, K, nblk, rg, sc, sn, nb_nxt, sb_mode, err,
                                            out, g_out, u_out);
    }
    const int ni = item + 1;
    if (ni >= i1) break;
    if (c_nxt.rt == 0) {  // the next item starts a new tile
      __syncthreads();    // every warp is done with the staged activations and pair ids
      load_xstage(smem, s_pairs, xs, rd_nxt, rd_nxt.d0.z > 0, xl, xm, a.n_pairs, a.slots, DUAL);
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
    }
    // rotate: the next item becomes current; the fetch cursor follows it
    if (rg.f_next == 0) rg.f_blk = 0;
    rg.f_next = 0;
    cur = nxt;
    sc = sn;
    nb_cur = nb_nxt;
    c_cur = c_nxt;
    c_nxt = c_nn;
    c_nn = advance(c_nn);
    const int nn = ni + 1;
    rd_nxt.d0 = d0_nn;  // prefetched one item ahead; the pair ids are needed only at a tile change
    if (nn < i1) {
      rd_nxt.d1 = gv.tiles[3 * c_nxt.tile + 1];
      rd_nxt.d2 = gv.tiles[3 * c_nxt.tile + 2];
    }
    d0_nn = nn + 1 < i1 ? gv.tiles[3 * c_nn.tile] : make_int4(0, 0, 0, 0);
    nxt = ItemInfo{};
    sn = Src{nullptr, nullptr};
    if (nn < i1) nxt = setup(rd_nxt, c_nxt.rt, sn);
    nb_nxt = nxt.ok ? nblk : 0;
  }
  // Every issued block was consumed (items run to completion), so no copy is
  // in flight; drain per-lane copy groups.
  cp_async_wait<0>();
}

// Small decode batches on tiled tables: a K-split GEMV.  Work item = (tile,
// one tiled row group: 8 gate + 8 up rows, or 16 down rows), one CTA of KS
// warps (KS = min(4, blocks)).  Warp ks bulk-copies its contiguous share of
// the row group's blocks (all at once, one mbarrier) and the activation limbs
// and group sums fl(SX) of its groups, then writes the exact per-group MMA
// sums S = C0 * 4096 + C1 of its groups to shared memory.  After a CTA
// barrier warp 0 folds the groups in order with the same two fmas per group
// as k_expert_rows -- scales and biases read from the staged chunks -- and
// runs the same epilogue, so the results are bit-identical to it.  The work
// of a long contraction is spread over KS warps instead of one, and an item
// touches 20 KB (gate/up at K = 2048), so a batch of one token spreads over
// every SM.  Pairs are processed 4 at a time (one MMA token tile); a tile
// with more pairs takes several passes over the staged weights.
constexpr int kGemvMaxBlocks = 16;

template <int G, bool DUAL>
__global__ void __launch_bounds__(128) k_expert_gemv(ExpertCallArgs a, GroupView gv, const uint16_t *xl,
                                                     const float *xm, int P, uint16_t *out, uint16_t *g_out,
                                                     uint16_t *u_out, uint32_t *err) {
  constexpr int GPB = 2 * kBlkBytes / G;  // groups per block
  constexpr int QG = GPB / 2;             // groups per half block
  constexpr int WB = G / 32;
  constexpr int RPW = DUAL ? 8 : 16;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar[4];
  __shared__ int s_pairs[kTokPerItem];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = blockDim.x >> 5;
  const int K = DUAL ? a.H : a.I;
  const int O = DUAL ? a.I : a.H;
  const XStage xs = xstage_geom(K, G);
  const int Gc = xs.Gc;
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  const int n_rg = O / RPW;
  if (lane == 0) {
    mbar_init(bar + warp, 1);
    mbar_init_fence();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();
  // the tile count and the whole descriptor in one round trip (the grid never
  // exceeds max_tiles tiles, so the descriptor slot exists even past n_tiles)
  const int tile = blockIdx.x / n_rg, rg = blockIdx.x - tile * n_rg;
  const int n_tiles = gv.n_tiles[0];
  const int4 d0 = gv.tiles[3 * tile];
  const int4 dp = threadIdx.x < kTokPerItem ? gv.tiles[3 * tile + 1 + (threadIdx.x >> 2)] : make_int4(0, 0, 0, 0);
  if (tile >= n_tiles) return;
  const int len = d0.z;
  if (len <= 0) return;  // nothing to run: issue no copy
  uint32_t rec = 0;
  if (!tiled_record(a, static_cast<uint32_t>(d0.x), rec)) {
    if (threadIdx.x == 0) set_error(err, kErrBadRoute);
    return;
  }
  if (threadIdx.x < kTokPerItem) {
    const int q = threadIdx.x & 3;
    s_pairs[threadIdx.x] = q == 0 ? dp.x : q == 1 ? dp.y : q == 2 ? dp.z : dp.w;
  }
  // smem: staged blocks | limbs [P][Xrow] | metadata [P][Mp] | sums [Gc][32] float2
  uint8_t *stages = smem;
  uint8_t *xst = stages + static_cast<size_t>(nblk) * kTileChunk;
  const int m_off = P * xs.Xrow;
  float2 *sums = reinterpret_cast<float2 *>(xst + ((m_off + P * xs.Mp + 15) & ~15));
  const int b0 = warp * nblk / KS, b1 = (warp + 1) * nblk / KS;
  const int g0 = b0 * GPB, g1 = min(b1 * GPB, Gc);
  if (lane == 0 && b1 > b0) {
    const uint8_t *base = (DUAL ? a.tiled.gate_up + rec * a.tiled.gate_up_record
                                : a.tiled.down + rec * a.tiled.down_record) +
                          static_cast<size_t>(rg) * nblk * kTileChunk;
    fence_proxy_async();
    mbar_expect_tx(bar + warp, static_cast<unsigned>(b1 - b0) * kTileChunk);
    for (int b = b0; b < b1; ++b)
      bulk_g2s(stages + static_cast<size_t>(b) * kTileChunk, base + static_cast<size_t>(b) * kTileChunk, kTileChunk,
               bar + warp);
  }
  __syncthreads();  // s_pairs
  const int r = lane >> 2, c = lane & 3;
  const uint32_t x0 = smem_u32(xst);
  const int passes = (len + P - 1) / P;
  bool waited = false;
  for (int pass = 0; pass < passes; ++pass) {
    const int q0 = pass * P, np = min(P, len - q0);
    // this warp's groups of the pass's pairs (and warp 0: every pair's {A, B})
    for (int q = 0; q < np; ++q) {
      const int pair = s_pairs[q0 + q];
      const int row = DUAL ? token_of_pair(pair, a.n_pairs, a.slots) : pair;
      const uint8_t *src = reinterpret_cast<const uint8_t *>(xl) + static_cast<size_t>(row) * xs.Xrow;
      const uint8_t *msrc = reinterpret_cast<const uint8_t *>(xm) + static_cast<size_t>(row) * xs.Mp;
      const int lb0 = g0 * 4 * G, lb1 = g1 * 4 * G;
      for (int o = lb0 + lane * 16; o < lb1; o += 512) cp_async16(xst + q * xs.Xrow + o, src + o);
      const int mb0 = g0 * 4, mb1 = (g1 * 4 + 15) & ~15;
      for (int o = mb0 + lane * 16; o < mb1; o += 512) cp_async16(xst + m_off + q * xs.Mp + o, msrc + o);
      if (warp == 0 && lane == 0) cp_async16(xst + m_off + q * xs.Mp + xs.a_off, msrc + xs.a_off);
    }
    cp_async_commit();
    cp_async_wait<0>();
    if (!waited && b1 > b0) {
      uint32_t spins = 0;
      while (!mbar_try_wait(bar + warp, 0)) {
        if (++spins >= kSpinLimit) {
          set_error(err, kErrTimeout);
          break;
        }
      }
    }
    waited = true;
    __syncwarp();
    // exact group sums of this warp's blocks; token columns past np reuse pair np - 1
    const uint32_t xb = x0 + min(r >> 1, np - 1) * xs.Xrow + (r & 1) * (G * 2) + c * 16;
    for (int b = b0; b < b1; ++b) {
      const uint32_t wq = smem_u32(stages + static_cast<size_t>(b) * kTileChunk) + (r * 4 + c) * 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 wA4 = lds128(wq + (2 * h) * 512);
        const uint4 wB4 = lds128(wq + (2 * h + 1) * 512);
#pragma unroll
        for (int j = 0; j < QG; ++j) {
          const int g = b * GPB + h * QG + j;
          if (g >= Gc) break;
          uint32_t A0[WB][4], A1[WB][4];
#pragma unroll
          for (int wb = 0; wb < WB; ++wb) nibble_operands(word_at(wA4, j * WB + wb), word_at(wB4, j * WB + wb), A0[wb], A1[wb]);
          float C[4];
#pragma unroll
          for (int wb = 0; wb < WB; ++wb) {
            const uint4 v = lds128(xb + g * (4 * G) + wb * 64);
            if (wb == 0) mma_16816_z(C, A0[wb], v.x, v.y);
            else mma_16816(C, A0[wb], v.x, v.y);
            mma_16816(C, A1[wb], v.z, v.w);
          }
          sums[g * 32 + lane] = make_float2(__fmaf_rn(C[0], 4096.0f, C[1]), __fmaf_rn(C[2], 4096.0f, C[3]));
        }
      }
    }
    // canonical fold over the groups in order (k_expert_rows' group_step):
    // warp 0 folds its own blocks, the first ones, before the barrier and the
    // other warps' blocks after it
    const uint32_t mrow = x0 + m_off + min(c, np - 1) * xs.Mp;
    float accA = -0.0f, accB = -0.0f;
    auto fold = [&](int bs, int be) {
      for (int b = bs; b < be; ++b) {
        // the block's scales and biases of rows r (A) and r + 8 (B): 8 bf16 each
        const uint32_t sbA = smem_u32(stages + static_cast<size_t>(b) * kTileChunk) + kTileW + r * 32;
        const uint4 sA8 = lds128(sbA), bA8 = lds128(sbA + 16);
        const uint4 sB8 = lds128(sbA + 8 * 32), bB8 = lds128(sbA + 8 * 32 + 16);
#pragma unroll
        for (int j = 0; j < GPB; ++j) {
          const int g = b * GPB + j;
          if (g >= Gc) break;
          const int sh = 16 * (j & 1);
          const float sA = bf16_to_f32(static_cast<uint16_t>(word_at(sA8, j >> 1) >> sh));
          const float bA = bf16_to_f32(static_cast<uint16_t>(word_at(bA8, j >> 1) >> sh));
          const float sB = bf16_to_f32(static_cast<uint16_t>(word_at(sB8, j >> 1) >> sh));
          const float bB = bf16_to_f32(static_cast<uint16_t>(word_at(bB8, j >> 1) >> sh));
          const float fs = __uint_as_float(lds32(mrow + 4 * g));
          const float2 S = sums[g * 32 + lane];
          accA = __fmaf_rn(bA, fs, __fmaf_rn(sA, S.x, accA));
          accB = __fmaf_rn(bB, fs, __fmaf_rn(sB, S.y, accB));
        }
      }
    };
    if (warp == 0) fold(0, b1);
    __syncthreads();
    if (warp == 0) {
      fold(b1, nblk);
      if (c < np) {
        const int pair = s_pairs[q0 + c];
        const uint2 abw = lds64(mrow + xs.a_off);
        const float2 ab = make_float2(__uint_as_float(abw.x), __uint_as_float(abw.y));
        const float yA = __fmul_rn(__fmul_rn(accA, ab.x), ab.y);
        const float yB = __fmul_rn(__fmul_rn(accB, ab.x), ab.y);
        const int oA = rg * RPW + r;
        store_rows<DUAL>(a, pair, O, oA, oA + 8, yA, yB, out, g_out, u_out);
      }
    }
    if (pass + 1 < passes) __syncthreads();  // sums and limbs are rewritten by the next pass
  }
}

namespace {

constexpr size_t kSmemLimit = 227 * 1024;

template <int G, int WARPS, bool DUAL, int R, bool TILED>
cudaError_t launch_rows(const ExpertCallArgs &a, const GroupView &gv, const uint16_t *xl, const float *xm,
                        uint16_t *out, uint16_t *g_out, uint16_t *u_out, int sb_mode, size_t smem, cudaStream_t s) {
  auto kernel = k_expert_rows<G, WARPS, DUAL, R, TILED>;
  const int threads = WARPS * 32;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const DeviceInfo di = device_info();
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm <= 0)
    per_sm = 1;
  cudaError_t e = launch_pdl(kernel, di.sms * per_sm, threads, smem, s, a, gv, xl, xm, out, g_out, u_out, sb_mode,
                             device_error_word());
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

size_t ring_smem(int xbytes, int warps, int r) {
  return static_cast<size_t>(xbytes) + static_cast<size_t>(warps) * r * (kStageBytes + 8) + (kTokPerItem + 4) * sizeof(int);
}

// Deepest ring (4, 3 or 2 stages) whose shared memory fits beside the
// activation stage.
template <int G, int WARPS, bool DUAL, bool TILED>
cudaError_t launch_ring(const ExpertCallArgs &a, const GroupView &gv, int K, const uint16_t *xl, const float *xm,
                        uint16_t *out, uint16_t *g_out, uint16_t *u_out, int sb_mode, cudaStream_t s) {
  const int x = xstage_geom(K, G).bytes;
  if (ring_smem(x, WARPS, 4) <= kSmemLimit)
    return launch_rows<G, WARPS, DUAL, 4, TILED>(a, gv, xl, xm, out, g_out, u_out, sb_mode, ring_smem(x, WARPS, 4), s);
  if (ring_smem(x, WARPS, 3) <= kSmemLimit)
    return launch_rows<G, WARPS, DUAL, 3, TILED>(a, gv, xl, xm, out, g_out, u_out, sb_mode, ring_smem(x, WARPS, 3), s);
  if (ring_smem(x, WARPS, 2) <= kSmemLimit)
    return launch_rows<G, WARPS, DUAL, 2, TILED>(a, gv, xl, xm, out, g_out, u_out, sb_mode, ring_smem(x, WARPS, 2), s);
  return cudaErrorInvalidValue;
}

// Shared memory of k_expert_gemv for P pairs per pass.
size_t gemv_smem(int K, int G, int P) {
  const XStage xs = xstage_geom(K, G);
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  const size_t x = (static_cast<size_t>(P) * (xs.Xrow + xs.Mp) + 15) & ~static_cast<size_t>(15);
  return static_cast<size_t>(nblk) * kTileChunk + x + static_cast<size_t>(xs.Gc) * 32 * sizeof(float2);
}

template <int G, bool DUAL>
cudaError_t launch_gemv(const ExpertCallArgs &a, const GroupView &gv, int K, const uint16_t *xl, const float *xm,
                        uint16_t *out, uint16_t *g_out, uint16_t *u_out, cudaStream_t s) {
  const int O = DUAL ? a.I : a.H;
  const int rpw = DUAL ? 8 : 16;
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  if (nblk > kGemvMaxBlocks || O % rpw != 0) return cudaErrorNotSupported;
  const int ks = std::min(4, nblk);
  const int P = std::min(4, std::max(1, a.tokens));
  const size_t smem = gemv_smem(K, G, P);
  if (smem > kSmemLimit) return cudaErrorNotSupported;
  auto kernel = k_expert_gemv<G, DUAL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  // every tile holds at least one pair: pairs + shared tokens bound the tiles
  const long long tiles = std::min<long long>(gv.max_tiles, static_cast<long long>(a.n_pairs) + a.tokens);
  const long long grid = tiles * (O / rpw);
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7FFFFFFF) return cudaErrorNotSupported;
  cudaError_t e = launch_pdl(kernel, static_cast<int>(grid), ks * 32, smem, s, a, gv, xl, xm, P, out, g_out, u_out,
                             device_error_word());
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int G, bool DUAL, bool TILED>
cudaError_t launch_width(const ExpertCallArgs &a, const GroupView &gv, int K, const uint16_t *xl, const float *xm,
                         uint16_t *out, uint16_t *g_out, uint16_t *u_out, int sb_mode, cudaStream_t s) {
  // Many pairs -> 16-warp CTAs (one per SM); few pairs (batch-1 decode) ->
  // 4-warp CTAs so that the handful of experts still spreads over every SM.
  // Tiled tables and few pairs: the K-split GEMV spreads each expert's rows
  // over many more warps.
  if ((a.n_pairs + a.tokens) >= 64)
    return launch_ring<G, 16, DUAL, TILED>(a, gv, K, xl, xm, out, g_out, u_out, sb_mode, s);
  if (TILED && !gemv_disabled()) {
    cudaError_t e = launch_gemv<G, DUAL>(a, gv, K, xl, xm, out, g_out, u_out, s);
    if (e != cudaErrorNotSupported) return e;
  }
  return launch_ring<G, 4, DUAL, TILED>(a, gv, K, xl, xm, out, g_out, u_out, sb_mode, s);
}

template <bool DUAL>
cudaError_t launch_family(const ExpertCallArgs &a, const GroupView &gv, int K, const uint16_t *xl,
                          const float *xm, uint16_t *out, uint16_t *g_out, uint16_t *u_out, cudaStream_t s) {
  const int Gc = K / a.G;
  const bool tiled = DUAL ? a.tiled.gate_up != nullptr : a.tiled.down != nullptr;
  if (tiled) {
    if (a.G == 32) return launch_width<32, DUAL, true>(a, gv, K, xl, xm, out, g_out, u_out, kSB16, s);
    return launch_width<64, DUAL, true>(a, gv, K, xl, xm, out, g_out, u_out, kSB16, s);
  }
  // Scale/bias rows move as one 16-byte piece per block when every row starts
  // on a 16-byte boundary (group size 32, a multiple of 8 groups per row,
  // aligned bases), as 4-byte pieces when rows are 4-byte aligned, else by
  // plain loads.
  const int sb_mode = (a.G == 32 && Gc % 8 == 0 && a.sb_bulk) ? kSB16 : (a.sb_async && Gc % 2 == 0) ? kSB4 : kSBSync;
  if (a.G == 32) return launch_width<32, DUAL, false>(a, gv, K, xl, xm, out, g_out, u_out, sb_mode, s);
  return launch_width<64, DUAL, false>(a, gv, K, xl, xm, out, g_out, u_out, sb_mode, s);
}

}  // namespace

cudaError_t launch_gate_up(const ExpertCallArgs &a, const GroupView &gv,
                           const uint16_t *x_limbs, const float *x_meta,
                           uint16_t *act, uint16_t *g_out, uint16_t *u_out,
                           cudaStream_t s) {
  return launch_family<true>(a, gv, a.H, x_limbs, x_meta, act, g_out, u_out, s);
}

cudaError_t launch_down(const ExpertCallArgs &a, const GroupView &gv,
                        const uint16_t *act_limbs, const float *act_meta,
                        uint16_t *d, cudaStream_t s) {
  return launch_family<false>(a, gv, a.I, act_limbs, act_meta, d, nullptr, nullptr, s);
}

// ---------------------------------------------------------------------------
// tiled expert tables: one 2560-byte chunk per (row group, block)
// ---------------------------------------------------------------------------
// Chunk layout (bytes): [half h 0-1][side 0 = A rows, 1 = B rows][slot
// r*4+c][4 words] (2048 bytes), then [16 MMA rows][scales 8 x bf16][biases
// 8 x bf16] (512 bytes).  Slot (r, c) of half h holds the words thread
// (r, c) feeds to the MMA for the groups of that half: G = 32 -- word c of
// groups 4h..4h+3; G = 64 -- words c and c+4 of groups 2h and 2h+1.  Bytes
// past the end of a row (tail block) are zero.  Gate/up chunks cover 8 gate
// rows (A) and the same 8 up rows (B); down chunks cover 16 consecutive rows
// (A = first 8).

__global__ void k_tile_experts(const uint32_t *__restrict__ wA_base, const uint32_t *__restrict__ wB_base,
                               const uint16_t *__restrict__ sA_base, const uint16_t *__restrict__ bA_base,
                               const uint16_t *__restrict__ sB_base, const uint16_t *__restrict__ bB_base,
                               int experts, int O, int K, int G, int dual, uint8_t *__restrict__ dst,
                               uint64_t record_bytes) {
  const int Gc = K / G;
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  const int rows_per_group = dual ? 8 : 16;
  const int n_rg = O / rows_per_group;
  const long long units = static_cast<long long>(experts) * n_rg * nblk * (kTileChunk / 16);
  const int GPB = 2 * kBlkBytes / G;
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int piece = static_cast<int>(u % (kTileChunk / 16));  // 16-byte piece of the chunk
    long long rest = u / (kTileChunk / 16);
    const int blk = static_cast<int>(rest % nblk);
    rest /= nblk;
    const int rg = static_cast<int>(rest % n_rg);
    const int e = static_cast<int>(rest / n_rg);
    uint32_t out[4] = {0u, 0u, 0u, 0u};
    // MMA row m (0-15) of this chunk -> (matrix, row)
    auto mat_row = [&](int m, bool &side_b) {
      side_b = dual ? (m >= 8) : false;
      return dual ? rg * 8 + (m & 7) : rg * 16 + m;
    };
    if (piece < 128) {
      const int h = piece >> 6, side = (piece >> 5) & 1, slot = piece & 31;
      const int r = slot >> 2, c = slot & 3;
      bool sb;
      const int row = mat_row(side * 8 + r, sb);
      const uint32_t *w = (sb ? wB_base : wA_base) + (static_cast<size_t>(e) * O + row) * (K / 8);
      for (int i = 0; i < 4; ++i) {
        int word;
        if (G == 32) {
          const int g = blk * GPB + 4 * h + i;
          word = 4 * g + c;
        } else {
          const int g = blk * GPB + 2 * h + (i >> 1);
          word = 8 * g + c + 4 * (i & 1);
        }
        out[i] = word < K / 8 ? w[word] : 0u;
      }
    } else {
      const int q = piece - 128;  // 0..31: MMA row q/2, scales (even) or biases (odd)
      const int m = q >> 1, kind = q & 1;
      bool sb;
      const int row = mat_row(m, sb);
      const uint16_t *src = kind ? (sb ? bB_base : bA_base) : (sb ? sB_base : sA_base);
      src += (static_cast<size_t>(e) * O + row) * Gc;
      uint16_t v[8];
      for (int j = 0; j < 8; ++j) {
        const int g = blk * GPB + j;
        v[j] = (j < GPB && g < Gc) ? src[g] : static_cast<uint16_t>(0);
      }
      for (int i = 0; i < 4; ++i) out[i] = static_cast<uint32_t>(v[2 * i]) | (static_cast<uint32_t>(v[2 * i + 1]) << 16);
    }
    uint8_t *chunk = dst + static_cast<size_t>(e) * record_bytes + (static_cast<size_t>(rg) * nblk + blk) * kTileChunk;
    *reinterpret_cast<uint4 *>(chunk + piece * 16) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

cudaError_t launch_tile_experts(const uint32_t *wA, const uint32_t *wB, const uint16_t *sA, const uint16_t *bA,
                                const uint16_t *sB, const uint16_t *bB, int experts, int O, int K, int G, bool dual,
                                uint8_t *dst, uint64_t record_bytes, cudaStream_t s) {
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  const long long units = static_cast<long long>(experts) * (O / (dual ? 8 : 16)) * nblk * (kTileChunk / 16);
  if (units <= 0) return cudaSuccess;
  const int threads = 256;
  const long long want = (units + threads - 1) / threads;
  const int blocks = static_cast<int>(std::min<long long>(want, 148LL * 16));
  k_tile_experts<<<blocks, threads, 0, s>>>(wA, wB, sA, bA, sB, bB, experts, O, K, G, dual ? 1 : 0, dst,
                                            record_bytes);
  return cudaGetLastError();
}

uint64_t tiled_record_bytes(int O, int K, bool dual) {
  const int nblk = (K / 2 + kBlkBytes - 1) / kBlkBytes;
  return static_cast<uint64_t>(O / (dual ? 8 : 16)) * nblk * kTileChunk;
}

// ---------------------------------------------------------------------------
// combine (metal_runtime.py:301-333)
// ---------------------------------------------------------------------------

constexpr int kCombineMaxSlots = 16;

__device__ __forceinline__ float bf16_lane(const uint4 &v, int e) {
  const uint32_t w = e < 2 ? v.x : e < 4 ? v.y : e < 6 ? v.z : v.w;
  return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
}

// Thread = 8 consecutive hidden elements of one token.  Every slot's route,
// score and 16-byte output slice is loaded before the slot-ordered float32
// accumulation (no fused multiply-add), so the loads overlap.
__global__ void __launch_bounds__(256) k_combine(const uint16_t *d, const uint32_t *routes,
                                                 const void *scores, int sf32, int T, int S, int H,
                                                 int mode, const uint16_t *sy,
                                                 const uint16_t *sh, const uint16_t *sg,
                                                 int E_arr, int records, uint16_t *__restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int h8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (8 * h8 >= H || t >= T) return;
  float sc[kCombineMaxSlots];
  uint4 dv[kCombineMaxSlots];
#pragma unroll
  for (int s = 0; s < kCombineMaxSlots; ++s) {
    sc[s] = 0.0f;
    dv[s] = make_uint4(0u, 0u, 0u, 0u);
    if (s < S) {
      const uint32_t r = routes[t * S + s];
      const bool valid = (r & kSlotBit) ? ((r & 0x7FFFFFFFu) < static_cast<uint32_t>(records))
                                        : (r < static_cast<uint32_t>(E_arr));
      if (valid) {
        sc[s] = sf32 ? static_cast<const float *>(scores)[t * S + s]
                     : bf16_to_f32(static_cast<const uint16_t *>(scores)[t * S + s]);
        dv[s] = *reinterpret_cast<const uint4 *>(d + (static_cast<size_t>(t) * S + s) * H + 8 * h8);
      } else {
        sc[s] = __int_as_float(0x7FC00000);  // marks an invalid slot (skipped below)
      }
    }
  }
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
  for (int s = 0; s < kCombineMaxSlots; ++s) {
    if (s < S && !isnan(sc[s])) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(bf16_lane(dv[s], e), sc[s]));
    }
  }
  const size_t base = static_cast<size_t>(t) * H + 8 * h8;
  uint4 extra = make_uint4(0u, 0u, 0u, 0u);
  float gate = 0.0f;
  if (mode == kCombineSharedY) extra = *reinterpret_cast<const uint4 *>(sy + base);
  if (mode == kCombineParts) {
    extra = *reinterpret_cast<const uint4 *>(sh + base);
    gate = bf16_to_f32(sg[t]);
  }
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float r2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 2 * q + h;
      const float routed = round_bf16(acc[e]);
      float res = routed;
      if (mode == kCombineSharedY) res = __fadd_rn(routed, bf16_lane(extra, e));
      else if (mode == kCombineParts) res = __fadd_rn(routed, bmul(bf16_lane(extra, e), gate));
      r2[h] = res;
    }
    o[q] = static_cast<uint32_t>(f32_to_bf16(r2[0])) | (static_cast<uint32_t>(f32_to_bf16(r2[1])) << 16);
  }
  *reinterpret_cast<uint4 *>(out + base) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Any slot count: one element per thread, loads in the slot loop.
__global__ void k_combine_any(const uint16_t *d, const uint32_t *routes,
                              const void *scores, int sf32, int T, int S, int H, int mode,
                              const uint16_t *sy, const uint16_t *sh,
                              const uint16_t *sg, int E_arr, int records, uint16_t *__restrict__ out) {
  pdl_wait();
  pdl_trigger();
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
  float res = routed;
  if (mode == kCombineSharedY) res = __fadd_rn(routed, bf16_to_f32(sy[static_cast<size_t>(t) * H + h]));
  else if (mode == kCombineParts) res = __fadd_rn(routed, bmul(bf16_to_f32(sh[static_cast<size_t>(t) * H + h]), bf16_to_f32(sg[t])));
  out[static_cast<size_t>(t) * H + h] = f32_to_bf16(res);
}

cudaError_t launch_combine(const uint16_t *d, const uint32_t *routes, const void *scores,
                           int scores_f32, int tokens, int slots, int H, int mode,
                           const uint16_t *shared_y, const uint16_t *shared,
                           const uint16_t *shared_gate, int array_experts, int table_records,
                           uint16_t *out, cudaStream_t s) {
  if (slots > kCombineMaxSlots || H % 8) {
    dim3 grid((H + 255) / 256, tokens);
    cudaError_t e = launch_pdl(k_combine_any, grid, 256, 0, s, d, routes, scores, scores_f32, tokens, slots, H, mode,
                               shared_y, shared, shared_gate, array_experts, table_records, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  const int chunks = H / 8;
  const int threads = chunks >= 256 ? 256 : ((chunks + 31) / 32) * 32;
  dim3 grid((chunks + threads - 1) / threads, tokens);
  cudaError_t e = launch_pdl(k_combine, grid, threads, 0, s, d, routes, scores, scores_f32, tokens, slots, H, mode, shared_y,
                             shared, shared_gate, array_experts, table_records, out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// The combine with float32 activations: float32 per-slot rows, shared_y /
// shared / shared_gate float32, float32 output; the same operations without
// the bfloat16 roundings (the reference's kernel with T = float).
__global__ void k_combine_f32(const float *d, const uint32_t *routes, const void *scores, int sf32, int T, int S,
                              int H, int mode, const float *sy, const float *sh, const float *sg, int E_arr,
                              int records, float *__restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H || t >= T) return;
  float acc = 0.0f;
  for (int s = 0; s < S; ++s) {
    const uint32_t r = routes[t * S + s];
    const bool valid = (r & kSlotBit) ? ((r & 0x7FFFFFFFu) < static_cast<uint32_t>(records))
                                      : (r < static_cast<uint32_t>(E_arr));
    if (!valid) continue;
    const float sc = sf32 ? static_cast<const float *>(scores)[t * S + s]
                          : bf16_to_f32(static_cast<const uint16_t *>(scores)[t * S + s]);
    acc = __fadd_rn(acc, __fmul_rn(d[(static_cast<size_t>(t) * S + s) * H + h], sc));
  }
  const size_t o = static_cast<size_t>(t) * H + h;
  float res = acc;
  if (mode == kCombineSharedY) res = __fadd_rn(acc, sy[o]);
  else if (mode == kCombineParts) res = __fadd_rn(acc, __fmul_rn(sh[o], sg[t]));
  out[o] = res;
}

cudaError_t launch_combine_f32(const float *d, const uint32_t *routes, const void *scores, int scores_f32,
                               int tokens, int slots, int H, int mode, const float *shared_y, const float *shared,
                               const float *shared_gate, int array_experts, int table_records, float *out,
                               cudaStream_t s) {
  dim3 grid((H + 255) / 256, tokens);
  cudaError_t e = launch_pdl(k_combine_f32, grid, 256, 0, s, d, routes, scores, scores_f32, tokens, slots, H, mode,
                             shared_y, shared, shared_gate, array_experts, table_records, out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// router logits: exact integer dot products of the row fixed points
// ---------------------------------------------------------------------------

// Router logits as exact integer dot products (GEMV form).  Grid (row
// groups, token blocks).  Each warp keeps kRouterRW router rows in registers
// as their 14-bit fixed points (row exponent from a warp reduction; lane j
// owns 8-element chunks j, j+32, ...); the CTA stages its token block as
// 22-bit fixed points in shared memory (token exponents from shared-memory
// maxima).  Every (row, token) sum is an exact int64 over the lane's
// elements plus an xor butterfly -- exact in any order -- scaled and rounded
// once to bfloat16 (router_logit_bits): the same bits as the tensor-core path.
// With prep_limbs set, CTAs from router_ctas on (one per token row, blockDim
// threads per row) compute the projection's row fixed point of x instead
// (prep_rows_body), which saves small batches a launch.
template <int CH, int kRouterRW, int kRouterTok, int kRouterWarps>
__global__ void __launch_bounds__(kRouterWarps * 32) k_router_logits(
    const uint16_t *x, const uint16_t *__restrict__ W, int T, int H, int E,
    const uint16_t *__restrict__ wsg, uint16_t *__restrict__ logits,
    uint16_t *__restrict__ shared_logit, uint16_t *prep_limbs, float *prep_meta, int prep_G, int router_ctas,
    uint32_t *err) {
  if (prep_limbs != nullptr && static_cast<int>(blockIdx.x) >= router_ctas) {
    constexpr int SPT = CH <= 4 ? 1 : CH <= 8 ? 2 : 4;
    pdl_wait();
    pdl_trigger();
    const int block = blockIdx.x - router_ctas;
    if (prep_G == 32) prep_rows_body<32, SPT>(x, T, H, blockDim.x, prep_limbs, prep_meta, err, block);
    else prep_rows_body<64, SPT>(x, T, H, blockDim.x, prep_limbs, prep_meta, err, block);
    return;
  }
  extern __shared__ __align__(16) int xq[];  // [kRouterTok][H] token fixed points
  __shared__ uint32_t s_mx[kRouterTok];
  __shared__ int s_ex[kRouterTok];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * kRouterWarps + warp) * kRouterRW;
  const int rows = E + (wsg != nullptr ? 1 : 0);
  const int nchunks = H / 8;
  const int t0 = blockIdx.y * kRouterTok;
  const int tb = min(kRouterTok, T - t0);
  int w[kRouterRW][CH * 8];
  int ew[kRouterRW];
  bool live[kRouterRW];
  bool bad = false;
#pragma unroll
  for (int q = 0; q < kRouterRW; ++q) {
    const int row = row0 + q;
    const uint16_t *wrow = row < E ? W + static_cast<size_t>(row) * H : (row < rows ? wsg : nullptr);
    live[q] = wrow != nullptr;
    uint4 wv[CH];
    uint32_t mx = 0;
#pragma unroll
    for (int m = 0; m < CH; ++m) {
      const int cidx = lane + 32 * m;
      wv[m] = (wrow != nullptr && cidx < nchunks) ? ldg_u128(reinterpret_cast<const uint4 *>(wrow + cidx * 8))
                                                  : make_uint4(0u, 0u, 0u, 0u);
      mx = max(mx, max_mag8(wv[m], bad));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
    ew[q] = row_exponent(mx);
    const FixScale sw = fix_scale(ew[q], kRouterWBits);
#pragma unroll
    for (int m = 0; m < CH; ++m) {
      const uint32_t u[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) w[q][m * 8 + i] = fixed_qf((u[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, sw);
    }
  }
  // the router rows are constant: their loads above overlap the previous kernel
  pdl_wait();
  pdl_trigger();
  // token block: exponents from the rows' largest magnitudes, then fixed points
  if (threadIdx.x < kRouterTok) s_mx[threadIdx.x] = 0u;
  __syncthreads();
  const uint4 *xsrc = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t0) * H);
  for (int idx = threadIdx.x; idx < tb * nchunks; idx += blockDim.x)
    atomicMax(&s_mx[idx / nchunks], max_mag8(xsrc[idx], bad));
  __syncthreads();
  if (threadIdx.x < tb) s_ex[threadIdx.x] = row_exponent(s_mx[threadIdx.x]);
  __syncthreads();
  for (int idx = threadIdx.x; idx < tb * nchunks; idx += blockDim.x) {
    const uint4 v = xsrc[idx];
    const FixScale sx = fix_scale(s_ex[idx / nchunks], kRouterXBits);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    int q8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q8[i] = fixed_qf((u[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, sx);
    reinterpret_cast<int4 *>(xq)[2 * idx] = make_int4(q8[0], q8[1], q8[2], q8[3]);
    reinterpret_cast<int4 *>(xq)[2 * idx + 1] = make_int4(q8[4], q8[5], q8[6], q8[7]);
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) set_error(err, kErrNonFinite);
  __syncthreads();
  if (!live[0]) return;
  long long acc[kRouterRW][kRouterTok];
#pragma unroll
  for (int q = 0; q < kRouterRW; ++q)
#pragma unroll
    for (int tt = 0; tt < kRouterTok; ++tt) acc[q][tt] = 0;
#pragma unroll
  for (int m = 0; m < CH; ++m) {
    const int cidx = lane + 32 * m;
    if (cidx < nchunks) {
#pragma unroll
      for (int tt = 0; tt < kRouterTok; ++tt) {
        // rows past tb hold stale data; their results are never stored
        const int4 *xp = reinterpret_cast<const int4 *>(xq + tt * H + cidx * 8);
        const int4 p0 = xp[0], p1 = xp[1];
        const int xv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int q = 0; q < kRouterRW; ++q) {
          long long a = acc[q][tt];
#pragma unroll
          for (int i = 0; i < 8; ++i) a += static_cast<long long>(w[q][m * 8 + i]) * xv[i];
          acc[q][tt] = a;
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kRouterRW; ++q)
#pragma unroll
    for (int tt = 0; tt < kRouterTok; ++tt)
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) acc[q][tt] += __shfl_xor_sync(0xFFFFFFFFu, acc[q][tt], off);
#pragma unroll
  for (int q = 0; q < kRouterRW; ++q) {
    const int row = row0 + q;
    if (!live[q] || lane >= tb) continue;
    long long v = acc[q][0];
#pragma unroll
    for (int tt = 1; tt < kRouterTok; ++tt)
      if (lane == tt) v = acc[q][tt];
    const uint16_t bits = router_logit_bits(v, s_ex[lane], ew[q]);
    if (row < E) logits[static_cast<size_t>(t0 + lane) * E + row] = bits;
    else shared_logit[t0 + lane] = bits;
  }
}

// Router logits for many tokens on integer tensor cores.
//
// k_router_prep: one warp per row -- every token row (22 fraction bits) and
// every router row (14 bits; row E is the shared gate) -- finds the row
// exponent and writes the fixed point as byte planes: token X = X0 + 2^8 X1 +
// 2^16 X2 (X0, X1 unsigned, X2 signed: |X| < 2^23), router W = W0 + 2^8 W1
// (W0 unsigned, W1 signed: |W| < 2^15).
//
// k_router_mma: CTA tile 64 tokens x 32 router rows, 4 warps of 16 tokens x
// 32 rows; K in 128-byte chunks through a 3-stage TMA ring: per chunk one 2D
// box (128 bytes x 64 rows) per token plane and one (128 x 32) per router
// plane, 128-byte swizzle (16-byte chunk j of box row r at j ^ (r & 7), so
// the eight rows of an ldmatrix phase fall in distinct bank groups); thread 0
// refills a stage once all four warps have released it.  Per 32-byte k-step a warp loads its A fragments
// (three token planes) and B fragments (two router planes) with ldmatrix and
// issues mma.sync.m16n8k32 with s32 accumulation for the six limb pairs,
// summed per power of two (2^0, 2^8, 2^16, 2^24: every partial sum stays
// below 2^31 for H <= 8192).  The epilogue forms the exact int64 dot
// product, scales it by 2^(Ex - 22 + Ew - 14) and rounds once to bfloat16:
// the GEMV kernels' bits.
constexpr int kRmTok = 64, kRmRows = 32, kRmK = 128, kRmThreads = 128, kRmStages = 3;
constexpr int kRmTokBox = kRmTok * kRmK, kRmRowBox = kRmRows * kRmK;  // box bytes
constexpr int kRmStage = 3 * kRmTokBox + 2 * kRmRowBox;               // bytes per ring stage
constexpr int kRmBarOff = kRmStages * kRmStage;
constexpr int kRmSmem = kRmBarOff + 16 * kRmStages + 1024;            // + barriers + 1 KiB alignment
constexpr uint32_t kRmSpin = 1u << 22;                                // mbarrier polls before giving up

//
// With prep_limbs set, CTAs from prep_base on compute the projection's row
// fixed point of x (prep_rows_body, prep_tpr threads per row), which saves
// decode batches the separate launch.
__global__ void __launch_bounds__(256) k_router_prep(const uint16_t *x, int T, const uint16_t *__restrict__ W,
                                                     const uint16_t *__restrict__ wsg, int E, int H,
                                                     RouterScratch rs, uint16_t *prep_limbs, float *prep_meta,
                                                     int prep_G, int prep_tpr, int prep_base, uint32_t *err) {
  pdl_wait();
  pdl_trigger();
  if (prep_limbs != nullptr && static_cast<int>(blockIdx.x) >= prep_base) {
    const int block = blockIdx.x - prep_base;
    const int spt = (H / 8 + prep_tpr - 1) / prep_tpr;
    if (prep_G == 32) {
      if (spt == 1) prep_rows_body<32, 1>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
      else if (spt == 2) prep_rows_body<32, 2>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
      else prep_rows_body<32, 4>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
    } else {
      if (spt == 1) prep_rows_body<64, 1>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
      else if (spt == 2) prep_rows_body<64, 2>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
      else prep_rows_body<64, 4>(x, T, H, prep_tpr, prep_limbs, prep_meta, err, block);
    }
    return;
  }
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int R = E + (wsg != nullptr ? 1 : 0);
  if (rs.ksplit > 1) {  // split-K: zero the partial sums and the tile tickets
    const size_t n = static_cast<size_t>(T) * R;
    const size_t tiles = static_cast<size_t>((T + kRmTok - 1) / kRmTok) * ((R + kRmRows - 1) / kRmRows);
    // the router CTAs only (the row fixed point CTAs after them have returned)
    const int ctas = prep_limbs != nullptr ? prep_base : static_cast<int>(gridDim.x);
    const size_t stride = static_cast<size_t>(ctas) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) rs.acc[i] = 0ull;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < tiles; i += stride)
      rs.tickets[i] = 0;
  }
  if (warp >= T + R) return;
  const bool tok = warp < T;
  const int row = tok ? warp : warp - T;
  const uint16_t *src = tok ? x + static_cast<size_t>(row) * H : (row < E ? W + static_cast<size_t>(row) * H : wsg);
  const int nchunks = H / 8;
  bool bad = false;
  uint32_t mx = 0;
  for (int c = lane; c < nchunks; c += 32) mx = max(mx, max_mag8(reinterpret_cast<const uint4 *>(src)[c], bad));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) set_error(err, kErrNonFinite);
  const int ex = row_exponent(mx);
  const FixScale sc = fix_scale(ex, tok ? kRouterXBits : kRouterWBits);
  const size_t plane = tok ? static_cast<size_t>(T) * H : static_cast<size_t>(R) * H;
  uint8_t *dst = (tok ? rs.xq : rs.wq) + static_cast<size_t>(row) * H;
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = reinterpret_cast<const uint4 *>(src)[c];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    uint32_t b0[2] = {0u, 0u}, b1[2] = {0u, 0u}, b2[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = fixed_qf((u[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, sc);
      const int sh = 8 * (i & 3);
      b0[i >> 2] |= (static_cast<uint32_t>(q) & 0xFFu) << sh;
      b1[i >> 2] |= (static_cast<uint32_t>(q >> 8) & 0xFFu) << sh;
      b2[i >> 2] |= (static_cast<uint32_t>(q >> 16) & 0xFFu) << sh;
    }
    reinterpret_cast<uint2 *>(dst)[c] = make_uint2(b0[0], b0[1]);
    reinterpret_cast<uint2 *>(dst + plane)[c] = make_uint2(b1[0], b1[1]);
    if (tok) reinterpret_cast<uint2 *>(dst + 2 * plane)[c] = make_uint2(b2[0], b2[1]);
  }
  if (lane == 0) (tok ? rs.ex : rs.ew)[row] = ex;
}

template <bool AS, bool BS>  // signedness of A (token plane) and B (router plane)
__device__ __forceinline__ void imma(int c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  if (!AS && !BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if (!AS && BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if (AS && !BS)
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// 2D TMA load of one box (no multicast) completing on mbarrier `bar`.
__device__ __forceinline__ void rm_tma(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool rm_wait(uint64_t *bar, unsigned parity, uint32_t *err) {
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins >= kRmSpin) {
      set_error(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t rm_swz(int r, int j) { return r * 128 + (((j ^ r) & 7) << 4); }

__global__ void __launch_bounds__(kRmThreads) k_router_mma(const __grid_constant__ CUtensorMap xmap,
                                                           const __grid_constant__ CUtensorMap wmap,
                                                           RouterScratch rs, int T, int E, int R, int H,
                                                           uint16_t *logits, uint16_t *shared_logit, uint32_t *err) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t rsm_raw[];
  uint8_t *rsm = rsm_raw + ((1024u - (smem_u32(rsm_raw) & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(rsm + kRmBarOff);
  uint64_t *empty = full + kRmStages;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int t0 = blockIdx.x * kRmTok, r0 = blockIdx.y * kRmRows;
  const int wt = 16 * warp, wr = 0;
  // this CTA's k-chunks: slice blockIdx.z of rs.ksplit
  const int nk_all = H / kRmK;
  const int per = (nk_all + rs.ksplit - 1) / rs.ksplit;
  const int kc0 = min(nk_all, static_cast<int>(blockIdx.z) * per);
  const int nk = min(nk_all, kc0 + per) - kc0;
  if (tid == 0) {
    for (int i = 0; i < kRmStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kRmThreads / 32);
    }
    mbar_init_fence();
  }
  __syncthreads();
  // stage: 3 token-plane boxes (plane p rows p*T + t0 ..), 2 router-plane boxes
  auto issue = [&](int kc, int slot) {
    uint8_t *base = rsm + slot * kRmStage;
    mbar_expect_tx(full + slot, kRmStage);
    const int x = (kc0 + kc) * kRmK;
#pragma unroll
    for (int p = 0; p < 3; ++p) rm_tma(smem_u32(base + p * kRmTokBox), &xmap, x, p * T + t0, full + slot);
#pragma unroll
    for (int p = 0; p < 2; ++p)
      rm_tma(smem_u32(base + 3 * kRmTokBox + p * kRmRowBox), &wmap, x, p * R + r0, full + slot);
  };
  bool dead = false;
  if (tid == 0)
    for (int i = 0; i < kRmStages - 1 && i < nk; ++i) issue(i, i);
  int acc[4][4][4];  // [2^(8s)][n-tile][fragment]
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][n][e] = 0;
  // ldmatrix addressing: lane i serves row (i & 7) of matrix (i >> 3)
  const int mi = lane >> 3, ri = lane & 7;
  const int a_row = wt + (mi & 1) * 8 + ri, b_row = wr + (mi & 1) * 8 + ri;
  for (int kc = 0; kc < nk; ++kc) {
    const int slot = kc % kRmStages;
    if (tid == 0 && kc + kRmStages - 1 < nk) {
      // refill the slot chunk kc - 1 used, once every warp has released it
      const int nxt = kc + kRmStages - 1, ns = nxt % kRmStages;
      if (nxt >= kRmStages && !dead) dead = !rm_wait(empty + ns, ((nxt / kRmStages) - 1) & 1, err);
      if (!dead) issue(nxt, ns);
    }
    __syncwarp();
    if (!rm_wait(full + slot, (kc / kRmStages) & 1, err)) break;
    const uint32_t sb = smem_u32(rsm + slot * kRmStage);
#pragma unroll
    for (int ks = 0; ks < kRmK / 32; ++ks) {
      const int jc = 2 * ks + (mi >> 1);  // 16-byte chunk of this lane's matrix row
      uint32_t A[3][4];
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) ldsm4(sb + pl * kRmTokBox + rm_swz(a_row, jc), A[pl]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        // n-tiles 2np and 2np + 1 of both router planes: b0 of each, then b1 of each
        uint32_t B0[4], B1[4];
        ldsm4(sb + 3 * kRmTokBox + rm_swz(b_row + 16 * np, jc), B0);
        ldsm4(sb + 3 * kRmTokBox + kRmRowBox + rm_swz(b_row + 16 * np, jc), B1);
#pragma unroll
        for (int nn = 0; nn < 2; ++nn) {
          const int n = 2 * np + nn;
          imma<false, false>(acc[0][n], A[0], B0[nn], B0[2 + nn]);
          imma<false, false>(acc[1][n], A[1], B0[nn], B0[2 + nn]);
          imma<false, true>(acc[1][n], A[0], B1[nn], B1[2 + nn]);
          imma<true, false>(acc[2][n], A[2], B0[nn], B0[2 + nn]);
          imma<false, true>(acc[2][n], A[1], B1[nn], B1[2 + nn]);
          imma<true, true>(acc[3][n], A[2], B1[nn], B1[2 + nn]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(empty + slot)) : "memory");
  }
  // every box issued lands before the CTA exits
  if (tid == 0)
    for (int kc = max(0, nk - kRmStages); kc < nk; ++kc) rm_wait(full + kc % kRmStages, (kc / kRmStages) & 1, err);
  // fragment e: token g (e < 2) or g + 8, router row 2t + (e & 1) of the n-tile
  const bool split = rs.ksplit > 1;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int tok = t0 + wt + g + (e >> 1) * 8;
    if (tok >= T) continue;
    const int ex = split ? 0 : rs.ex[tok];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int row = r0 + wr + 8 * n + 2 * t + (e & 1);
      if (row >= R) continue;
      const long long S = static_cast<long long>(acc[0][n][e]) + (static_cast<long long>(acc[1][n][e]) << 8) +
                          (static_cast<long long>(acc[2][n][e]) << 16) + (static_cast<long long>(acc[3][n][e]) << 24);
      if (split) {
        // integer sums are exact in any order: slices add into the tile's partial sums
        atomicAdd(rs.acc + static_cast<size_t>(tok) * R + row, static_cast<unsigned long long>(S));
        continue;
      }
      const uint16_t bits = router_logit_bits(S, ex, rs.ew[row]);
      if (row < E) logits[static_cast<size_t>(tok) * E + row] = bits;
      else shared_logit[tok] = bits;
    }
  }
  if (!split) return;
  // the tile's last slice to finish converts its sums (and clears them)
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) s_last = atomicAdd(rs.tickets + tile, 1) == rs.ksplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < kRmTok * kRmRows; i += kRmThreads) {
    const int tok = t0 + i / kRmRows, row = r0 + i % kRmRows;
    if (tok >= T || row >= R) continue;
    unsigned long long *p = rs.acc + static_cast<size_t>(tok) * R + row;
    const long long S = static_cast<long long>(__ldcg(p));
    *p = 0ull;
    const uint16_t bits = router_logit_bits(S, rs.ex[tok], rs.ew[row]);
    if (row < E) logits[static_cast<size_t>(tok) * E + row] = bits;
    else shared_logit[tok] = bits;
  }
  if (tid == 0) rs.tickets[tile] = 0;
}

// Router logits for prefill-sized batches on tcgen05, from the byte planes of
// k_router_prep.  A tile is 128 tokens (MMA M: TMEM lanes) x 64 router rows
// (MMA N).  Per 32-byte k-step six tcgen05.mma.kind::i8 (M128 N64 K32, s32 in
// TMEM) add the limb products into four 64-column accumulators, one per
// power of two: 2^0 X0 W0; 2^8 X1 W0 + X0 W1; 2^16 X2 W0 + X1 W1; 2^24 X2 W1
// (X2 and W1 signed; every partial sum stays below 2^31 for H <= 8192).
// Persistent CTAs, one per SM, walk the tiles; two 256-column accumulator
// sets let the epilogue of one tile overlap the MMAs of the next.
//   warp 0     TMA producer: per 128-byte k-chunk three 128-row token boxes
//              and two 64-row router boxes (128-byte swizzle, the K-major
//              SW128 operand layout), 3-stage ring;
//   warp 1     TMEM allocation and the MMA issuer (one thread);
//   warps 2-5  epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its 32
//              tokens), forms the exact int64 sums, scales them by
//              2^(Ex - 22 + Ew - 14) and rounds once to bfloat16 -- the GEMV
//              kernels' bits.
// Every wait is bounded; a timeout sets kErrTimeout, marks the CTA dead
// (later waits return at once) and every role runs to the teardown.
constexpr int kRuTok = 128, kRuRows = 64, kRuStages = 3, kRuThreads = 192;
constexpr int kRuTokBox = kRuTok * kRmK, kRuRowBox = kRuRows * kRmK;  // box bytes
constexpr int kRuStage = 3 * kRuTokBox + 2 * kRuRowBox;               // 64 KB per ring stage
constexpr int kRuBarOff = kRuStages * kRuStage;
constexpr int kRuFull = 0, kRuEmpty = kRuStages, kRuAccFull = 2 * kRuStages, kRuAccEmpty = kRuAccFull + 2,
              kRuBars = kRuAccEmpty + 2;
constexpr int kRuSmem = kRuBarOff + 8 * kRuBars + 16 + 1024;  // + tmem slot, dead flag, 1 KiB alignment
constexpr uint32_t kRuTmemCols = 512;                         // two sets of four 64-column accumulators
static_assert(kRuSmem <= 227 * 1024, "router tcgen05 shared memory");

// Instruction descriptor of kind::i8: s32 D, A/B signedness, K-major A and B, N 64, M 128.
__host__ __device__ constexpr uint32_t ru_idesc(bool a_signed, bool b_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(kRuRows >> 3) << 17) | (static_cast<uint32_t>(kRuTok >> 4) << 24);
}

template <bool AS, bool BS>
__device__ __forceinline__ void umma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(ru_idesc(AS, BS)), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool ru_wait(uint32_t bar, uint32_t parity, volatile uint32_t *dead, uint32_t *err) {
  uint32_t spins = 0;
  while (!mbar_try_wait_u32(bar, parity)) {
    if (*dead) return false;
    if (++spins >= kRmSpin) {
      *dead = 1u;
      set_error(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kRuThreads, 1) k_router_umma(const __grid_constant__ CUtensorMap xmap,
                                                               const __grid_constant__ CUtensorMap wmap,
                                                               RouterScratch rs, int T, int E, int R, int H,
                                                               uint16_t *logits, uint16_t *shared_logit,
                                                               uint32_t *err) {
  extern __shared__ __align__(128) uint8_t rsm_raw[];
  uint8_t *rsm = rsm_raw + ((1024u - (smem_u32(rsm_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(rsm);
  const uint32_t bars = sbase + kRuBarOff;
  auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rsm + kRuBarOff + 8 * kRuBars);
  volatile uint32_t *dead = tmem_slot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rt = (R + kRuRows - 1) / kRuRows;
  const int n_items = ((T + kRuTok - 1) / kRuTok) * n_rt;
  const int nk = H / kRmK;
  if (tid == 0) {
    for (int i = 0; i < kRuBars; ++i) {
      const uint32_t count = (i >= kRuAccEmpty) ? 4u : 1u;  // acc_empty: the four epilogue warps
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar(i)), "r"(count));
    }
    *dead = 0u;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kRuTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  pdl_wait();  // the byte planes and exponents come from k_router_prep
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t st = 0, ph = 0;
      bool live = true;
      for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
        const int t0 = (item / n_rt) * kRuTok, r0 = (item % n_rt) * kRuRows;
        for (int kc = 0; kc < nk; ++kc) {
          live = ru_wait(bar(kRuEmpty + st), ph ^ 1u, dead, err);
          if (!live) break;
          mbar_expect_tx_u32(bar(kRuFull + st), kRuStage);
          const uint32_t base = sbase + st * kRuStage;
#pragma unroll
          for (int p = 0; p < 3; ++p) tma_box2d(base + p * kRuTokBox, &xmap, kc * kRmK, p * T + t0, bar(kRuFull + st));
#pragma unroll
          for (int p = 0; p < 2; ++p)
            tma_box2d(base + 3 * kRuTokBox + p * kRuRowBox, &wmap, kc * kRmK, p * R + r0, bar(kRuFull + st));
          if (++st == kRuStages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t st = 0, ph = 0;
      int n = 0;
      bool live = true;
      for (int item = blockIdx.x; item < n_items && live; item += gridDim.x) {
        const uint32_t b = n & 1, bph = (n >> 1) & 1;
        ++n;
        live = ru_wait(bar(kRuAccEmpty + b), bph ^ 1u, dead, err);
        if (!live) break;
        tc_fence_after();
        const uint32_t d = tmem + b * 256;
        for (int kc = 0; kc < nk; ++kc) {
          live = ru_wait(bar(kRuFull + st), ph, dead, err);
          if (!live) break;
          tc_fence_after();
          const uint32_t base = sbase + st * kRuStage;
          const uint64_t a0 = sw128_desc(base), a1 = sw128_desc(base + kRuTokBox),
                         a2 = sw128_desc(base + 2 * kRuTokBox);
          const uint64_t b0 = sw128_desc(base + 3 * kRuTokBox), b1 = sw128_desc(base + 3 * kRuTokBox + kRuRowBox);
#pragma unroll
          for (int kk = 0; kk < kRmK / 32; ++kk) {
            const uint32_t acc = (kc | kk) != 0 ? 1u : 0u;
            const uint64_t o = 2ull * kk;  // 32 bytes along the swizzled row
            umma_i8<false, false>(d, a0 + o, b0 + o, acc);
            umma_i8<false, false>(d + 64, a1 + o, b0 + o, acc);
            umma_i8<false, true>(d + 64, a0 + o, b1 + o, 1u);
            umma_i8<true, false>(d + 128, a2 + o, b0 + o, acc);
            umma_i8<false, true>(d + 128, a1 + o, b1 + o, 1u);
            umma_i8<true, true>(d + 192, a2 + o, b1 + o, acc);
          }
          umma_commit(bar(kRuEmpty + st));
          if (++st == kRuStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (live) umma_commit(bar(kRuAccFull + b));
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. + 31
    const bool vec = (E % 8) == 0;
    int n = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const uint32_t b = n & 1, bph = (n >> 1) & 1;
      ++n;
      if (!ru_wait(bar(kRuAccFull + b), bph, dead, err)) break;
      tc_fence_after();
      const int t0 = (item / n_rt) * kRuTok, r0 = (item % n_rt) * kRuRows;
      const int tok = t0 + 32 * quarter + lane;
      const bool valid = tok < T;
      const int ex = valid ? rs.ex[tok] : 0;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + b * 256;
#pragma unroll 1
      for (int c = 0; c < kRuRows / 16; ++c) {
        uint32_t v0[16], v1[16], v2[16], v3[16];
        tmem_ld16_nowait(taddr + 16 * c, v0);
        tmem_ld16_nowait(taddr + 64 + 16 * c, v1);
        tmem_ld16_nowait(taddr + 128 + 16 * c, v2);
        tmem_ld16_nowait(taddr + 192 + 16 * c, v3);
        tmem_wait_ld();
        if (!valid) continue;
        const int row0 = r0 + 16 * c;
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int row = row0 + j;
          const long long S = static_cast<long long>(static_cast<int>(v0[j])) +
                              static_cast<long long>(static_cast<int>(v1[j])) * 256LL +
                              static_cast<long long>(static_cast<int>(v2[j])) * 65536LL +
                              static_cast<long long>(static_cast<int>(v3[j])) * 16777216LL;
          const uint32_t bits = row < R ? router_logit_bits(S, ex, __ldg(rs.ew + row)) : 0u;
          if (j & 1) o[j >> 1] |= bits << 16;
          else o[j >> 1] = bits;
        }
        if (vec && row0 + 16 <= E) {
          uint4 *dst = reinterpret_cast<uint4 *>(logits + static_cast<size_t>(tok) * E + row0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = row0 + j;
            const uint16_t bits = static_cast<uint16_t>(o[j >> 1] >> (16 * (j & 1)));
            if (row < E) logits[static_cast<size_t>(tok) * E + row] = bits;
            else if (row < R) shared_logit[tok] = bits;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kRuAccEmpty + b));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kRuTmemCols));
  }
}

template <int CH, int RW, int TOK, int NW = 8>
cudaError_t launch_router_cfg(const uint16_t *x, const uint16_t *W, int T, int H, int E,
                              const uint16_t *w_shared_gate, uint16_t *logits, uint16_t *shared_logit,
                              cudaStream_t s, uint16_t *prep_limbs = nullptr, float *prep_meta = nullptr,
                              int prep_G = 32, bool *prep_done = nullptr) {
  const int rows = E + (w_shared_gate ? 1 : 0);
  const int rows_per_cta = NW * RW;
  const int router_ctas = (rows + rows_per_cta - 1) / rows_per_cta;
  // the fused prep needs one token block and NW*32 threads covering a row in <= 4 passes
  const bool prep = prep_limbs != nullptr && T <= TOK && H / 8 <= 4 * NW * 32;
  const dim3 grid(router_ctas + (prep ? T : 0), (T + TOK - 1) / TOK);
  const size_t smem = static_cast<size_t>(TOK) * H * sizeof(float);
  auto kernel = k_router_logits<CH, RW, TOK, NW>;
  if (smem + 1024 > 48 * 1024) {  // the static shared memory (prep rows) counts toward the default limit
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = launch_pdl(kernel, grid, NW * 32, smem, s, x, W, T, H, E, w_shared_gate, logits, shared_logit,
                             prep ? prep_limbs : nullptr, prep_meta, prep_G, router_ctas, device_error_word());
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (prep_done != nullptr) *prep_done = prep && e == cudaSuccess;
  return e;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

namespace {
EncodeTiledFn router_encode_fn() {
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
}  // namespace

// A byte matrix [rows][cols] (row pitch cols, a multiple of 128) as a tensor
// map with 128-byte x box_rows boxes, 128-byte swizzle; rows past the end
// read as zero.
bool make_u8_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, int box_rows) {
  EncodeTiledFn fn = router_encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRmK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int router_tiles(int T, int R) { return ((T + kRmTok - 1) / kRmTok) * ((R + kRmRows - 1) / kRmRows); }

int router_ksplit(int T, int R, int H) {
  const long long tiles = router_tiles(T, R);
  const int nk = H / kRmK;
  const long long want = (3LL * device_info().sms + tiles - 1) / tiles;  // three CTAs per SM
  return static_cast<int>(std::max(1LL, std::min<long long>(nk, want)));
}

uint64_t router_scratch_bytes(int T, int R, int H) {
  if (T < 64 || H % kRmK != 0 || H > 8192) return 0;
  auto up = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
  uint64_t b = up(3ull * T * H) + up(2ull * R * H) + up(4ull * T) + up(4ull * R);
  if (router_ksplit(T, R, H) > 1) {
    b += up(8ull * T * R) + up(4ull * router_tiles(T, R));
  }
  return b;
}

cudaError_t launch_router_logits(const uint16_t *x, const uint16_t *W, int T, int H, int E,
                                 const uint16_t *w_shared_gate, uint16_t *logits,
                                 uint16_t *shared_logit, cudaStream_t s, uint16_t *prep_limbs, float *prep_meta,
                                 int prep_G, bool *prep_done, const RouterScratch *rs) {
  const int ch = (H / 8 + 31) / 32;
  if (prep_done != nullptr) *prep_done = false;
  const int rows = E + (w_shared_gate ? 1 : 0);
  if (rs != nullptr && router_scratch_bytes(T, rows, H) > 0) {
    // many tokens: byte planes, then the integer tensor-core GEMM
    const int warps = T + rows;
    const int base = (warps + 7) / 8;
    // decode batches: the row fixed point of x in extra CTAs of the same
    // launch when its threads per row divide the 256-thread CTA
    const int slices = H / 8;
    const int tpr = std::min(256, ((slices + 31) / 32) * 32);
    const bool prep = prep_limbs != nullptr && 256 % tpr == 0 && slices <= 4 * tpr && (prep_G == 32 || prep_G == 64);
    const int prep_ctas = prep ? (T + 256 / tpr - 1) / (256 / tpr) : 0;
    cudaError_t e = launch_pdl(k_router_prep, base + prep_ctas, 256, 0, s, x, T, W, w_shared_gate, E, H, *rs,
                               prep ? prep_limbs : nullptr, prep_meta, prep_G, tpr, base, device_error_word());
    if (e == cudaSuccess && prep_done != nullptr) *prep_done = prep;
    if (e != cudaSuccess) return e;
    CUtensorMap xmap{}, wmap{};
    const int sms = device_info().sms;
    const int u_items = ((T + kRuTok - 1) / kRuTok) * ((rows + kRuRows - 1) / kRuRows);
    if (u_items >= sms) {
      // enough 128-token x 64-row tiles to fill the SMs: tcgen05
      static const cudaError_t uattr =
          cudaFuncSetAttribute(k_router_umma, cudaFuncAttributeMaxDynamicSharedMemorySize, kRuSmem);
      if (uattr != cudaSuccess) return uattr;
      if (!make_u8_map(&xmap, rs->xq, 3ull * T, H, kRuTok) || !make_u8_map(&wmap, rs->wq, 2ull * rows, H, kRuRows))
        return cudaErrorInvalidValue;
      e = launch_pdl(k_router_umma, std::min(u_items, sms), kRuThreads, kRuSmem, s, xmap, wmap, *rs, T, E, rows, H,
                     logits, shared_logit, device_error_word());
      if (e != cudaSuccess) return e;
      return cudaGetLastError();
    }
    static const cudaError_t attr =
        cudaFuncSetAttribute(k_router_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, kRmSmem);
    if (attr != cudaSuccess) return attr;
    if (!make_u8_map(&xmap, rs->xq, 3ull * T, H, kRmTok) || !make_u8_map(&wmap, rs->wq, 2ull * rows, H, kRmRows))
      return cudaErrorInvalidValue;
    e = launch_pdl(k_router_mma, dim3((T + kRmTok - 1) / kRmTok, (rows + kRmRows - 1) / kRmRows, rs->ksplit),
                   kRmThreads, kRmSmem, s, xmap, wmap, *rs, T, E, rows, H, logits, shared_logit,
                   device_error_word());
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  // Small batches: one router row per warp and 4-warp CTAs, so ~E/4 CTAs
  // share the weight read instead of E/16.
  if (T <= 4) {
#define FNMOE_ROUTER_SMALL(C)                                                                                 \
  if (ch <= C)                                                                                                  \
    return launch_router_cfg<C, 1, 4, 4>(x, W, T, H, E, w_shared_gate, logits, shared_logit, s, prep_limbs,    \
                                         prep_meta, prep_G, prep_done);
    FNMOE_ROUTER_SMALL(4)
    FNMOE_ROUTER_SMALL(8)
    FNMOE_ROUTER_SMALL(12)
    FNMOE_ROUTER_SMALL(16)
#undef FNMOE_ROUTER_SMALL
    return cudaErrorInvalidValue;
  }
  if (ch <= 4) return launch_router_cfg<4, 1, 16>(x, W, T, H, E, w_shared_gate, logits, shared_logit, s);
  if (ch <= 8) return launch_router_cfg<8, 1, 16>(x, W, T, H, E, w_shared_gate, logits, shared_logit, s);
  if (ch <= 12) return launch_router_cfg<12, 1, 8>(x, W, T, H, E, w_shared_gate, logits, shared_logit, s);
  if (ch <= 16) return launch_router_cfg<16, 1, 8>(x, W, T, H, E, w_shared_gate, logits, shared_logit, s);
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// softmax (precise) + top-k + renorm, one warp per token
// ---------------------------------------------------------------------------

// Logits per lane (experts <= 32 * PER) is a template parameter: 16 at 512 experts.

// Adaptive keep (adaptive_topk.py:43-50): with 0 < threshold < 1, the first
// position whose cumulative share of the top-k mass reaches the threshold
// (IEEE double, sequential, as the reference's Python floats), at least
// max(1, min(k, min_keep)); otherwise k.  `sel(s)` is slot s's probability.
template <typename Sel>
__device__ __forceinline__ int keep_count(Sel sel, int k, double threshold, int min_keep) {
  if (!(threshold > 0.0 && threshold < 1.0)) return k;
  double total = 0.0;
  for (int s = 0; s < k; ++s) total += static_cast<double>(sel(s));
  double acc = 0.0;
  int keep = k;
  for (int s = 0; s < k; ++s) {
    acc += static_cast<double>(sel(s)) / total;
    if (acc >= threshold) {
      keep = s + 1;
      break;
    }
  }
  return max(keep, max(1, min(k, min_keep)));
}

template <int kMaxPerLane>
__global__ void __launch_bounds__(128) k_softmax_topk(
    const uint16_t *logits, int T, int E, int k, float blend,
    const uint32_t *__restrict__ route_map, int table_routes, uint32_t *__restrict__ inds,
    uint32_t *__restrict__ routes, uint16_t *__restrict__ raw_scores,
    uint16_t *__restrict__ scores, uint16_t *__restrict__ mass,
    const uint16_t *shl, uint16_t *__restrict__ shg, double keep_threshold, int min_keep) {
  pdl_wait();
  pdl_trigger();
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
    best = __reduce_max_sync(0xFFFFFFFFu, best);  // one redux.sync: keys are unique, order-free
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
    const int keep = keep_count([&](int s) { return sel[s]; }, k, keep_threshold, min_keep);
    float kept = 0.0f;  // kept mass in slot order (all of it when nothing is dropped)
    for (int s = 0; s < keep; ++s) kept = __fadd_rn(kept, sel[s]);
    const float selected = round_bf16(kept);
    const float bl = round_bf16(blend);
    const float normalizer = badd(topm, bmul(bl, bsub(selected, topm)));
    for (int s = 0; s < k; ++s) {
      const bool live = s < keep;  // dropped slots: slot 0's expert, score 0, no expert run
      const uint32_t e = live ? idx[s] : idx[0];
      inds[static_cast<size_t>(t) * k + s] = e;
      routes[static_cast<size_t>(t) * k + s] =
          !live ? kRouteNone : route_map ? route_map[e] : (table_routes ? (kSlotBit | e) : e);
      if (raw_scores) raw_scores[static_cast<size_t>(t) * k + s] = live ? f32_to_bf16(sel[s]) : 0;
      if (scores) scores[static_cast<size_t>(t) * k + s] = live ? f32_to_bf16(__fdiv_rn(sel[s], normalizer)) : 0;
    }
    if (mass) mass[t] = f32_to_bf16(topm);
    if (shl && shg) shg[t] = f32_to_bf16(sigmoid_bf16(g_exp_bf16, bf16_to_f32(shl[t])));
  }
}

// Softmax, top-k and renorm for up to kRouteSmallTokens tokens, then the
// grouping, in one 1024-thread CTA (small decode batches: one launch instead
// of two, and the exps of a token spread over 32/Tp warps, Tp = T rounded up
// to a power of two).  Max, exps, the canonical 32-lane sum, the key order
// and the renorm are those of k_softmax_topk, so results are identical.
constexpr int kRouteSmallTokens = 8;
constexpr int kRouteSmallPairs = kRouteSmallTokens * 33;  // <= 8 tokens x (32 slots + shared)

// Decode tiles of a few pairs straight from the routes in shared memory (one
// CTA of 1024 threads): each pair's place in the stable bin order is counted
// directly (bins, then pair index, as the grouping), and the runs of each bin
// are cut into 8-pair tiles.  Writes order, tiles and n_tiles only: the
// decode expert kernels read nothing else.  `sm` holds >= 5 * 264 ints.
__device__ __forceinline__ void route_tiles(const uint32_t *s_route, int n_pairs, int shared_tokens, int E_arr,
                                            int records, const GroupView &gv, uint32_t *err, int *sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_total = n_pairs + shared_tokens;
  const int n_bins = gv.n_bins;
  int *s_bin = sm;                          // [n_total]
  int *s_ord = sm + kRouteSmallPairs;       // sorted position -> pair
  int *s_less = sm + 2 * kRouteSmallPairs;  // sorted position -> first position of its bin
  int *s_cnt = sm + 3 * kRouteSmallPairs;   // sorted position -> pairs in its bin
  int *s_wsum = sm + 4 * kRouteSmallPairs;  // tile starts per warp
  __shared__ int s_valid;
  if (tid == 0) s_valid = 0;
  if (tid < n_total) {
    const int b = tid < n_pairs ? bin_of_route(s_route[tid], E_arr, records) : n_bins - 1;
    s_bin[tid] = b;
    if (b == -1) set_error(err, kErrBadRoute);
  }
  __syncthreads();
  if (tid < n_total && s_bin[tid] >= 0) {
    const int b = s_bin[tid];
    int less = 0, before = 0, cnt = 0;
    for (int j = 0; j < n_total; ++j) {
      const int bj = s_bin[j];
      less += (bj >= 0 && bj < b);
      cnt += (bj == b);
      before += (bj == b && j < tid);
    }
    const int r = less + before;
    s_ord[r] = tid;
    s_less[r] = less;
    s_cnt[r] = cnt;
    gv.order[r] = tid;
    atomicAdd(&s_valid, 1);
  }
  __syncthreads();
  const int n_valid = s_valid;
  const bool start = tid < n_valid && ((tid - s_less[tid]) % kTokPerItem) == 0;
  const unsigned bal = __ballot_sync(0xFFFFFFFFu, start);
  if (lane == 0) s_wsum[warp] = __popc(bal);
  __syncthreads();
  int t = __popc(bal & ((1u << lane) - 1u));
  for (int w = 0; w < warp; ++w) t += s_wsum[w];
  if (start && t < gv.max_tiles) {
    const int b = s_bin[s_ord[tid]];
    const int off = tid - s_less[tid];
    const int len = min(kTokPerItem, s_cnt[tid] - off);
    int p[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) p[q] = q < len ? s_ord[tid + q] : -1;
    const uint32_t key = (b < E_arr) ? static_cast<uint32_t>(b)
                         : (b < E_arr + records) ? (kSlotBit | static_cast<uint32_t>(b - E_arr))
                                                 : kSharedKey;
    gv.tiles[3 * t] = make_int4(static_cast<int>(key), tid, len, b);
    gv.tiles[3 * t + 1] = make_int4(p[0], p[1], p[2], p[3]);
    gv.tiles[3 * t + 2] = make_int4(p[4], p[5], p[6], p[7]);
  }
  if (tid == 0) {
    int total = 0;
    for (int w = 0; w < 32; ++w) total += s_wsum[w];
    gv.n_tiles[0] = min(total, gv.max_tiles);
  }
}


template <int PER>
__global__ void __launch_bounds__(1024) k_route_small(
    const uint16_t *logits, int T, int E, int k, float blend,
    const uint32_t *__restrict__ route_map, int table_routes, uint32_t *inds, uint32_t *routes,
    uint16_t *raw_scores, uint16_t *scores, uint16_t *mass, const uint16_t *shl,
    uint16_t *shg, int shared_tokens, int E_arr, int records, GroupView gv, int seg_warps, double keep_threshold,
    int min_keep, int tiles_only, uint32_t *err) {
  extern __shared__ int sm[];
  pdl_wait();
  pdl_trigger();
  float *ev = reinterpret_cast<float *>(sm);  // [T][E]: exps, then keys
  uint32_t *kv = reinterpret_cast<uint32_t *>(sm);
  __shared__ float s_max[kRouteSmallTokens][32];
  __shared__ float s_sum[kRouteSmallTokens];
  __shared__ uint32_t s_route[kRouteSmallTokens * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tp = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;
  const int wpt = 32 / tp;
  const int t = warp / wpt, wl = warp - t * wpt;
  const int per = (E + 31) / 32;
  const bool tok = t < T;
  const uint16_t *lrow = logits + static_cast<size_t>(tok ? t : 0) * E;
  float mx = -INFINITY;
  if (tok)
    for (int m = wl; m < per; m += wpt)
      if (lane + 32 * m < E) mx = fmaxf(mx, bf16_to_f32(lrow[lane + 32 * m]));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  if (tok && lane == 0) s_max[t][wl] = mx;
  __syncthreads();
  if (tok) {
    float M = -INFINITY;
    for (int w = 0; w < wpt; ++w) M = fmaxf(M, s_max[t][w]);
    for (int m = wl; m < per; m += wpt) {
      const int i = lane + 32 * m;
      if (i < E) ev[t * E + i] = __double2float_rn(exp(static_cast<double>(__fsub_rn(bf16_to_f32(lrow[i]), M))));
    }
  }
  __syncthreads();
  if (tok && wl == 0) {
    float sum = -0.0f;
#pragma unroll
    for (int m = 0; m < PER; ++m)
      if (m < per && lane + 32 * m < E) sum = __fadd_rn(sum, ev[t * E + lane + 32 * m]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, off));
    if (lane == 0) s_sum[t] = sum;
  }
  __syncthreads();
  if (tok) {
    const float sum = s_sum[t];
    for (int m = wl; m < per; m += wpt) {
      const int i = lane + 32 * m;
      if (i < E) {
        const uint32_t pb = f32_to_bf16(__fdiv_rn(ev[t * E + i], sum));
        kv[t * E + i] = (pb << 16) | (0xFFFFu - static_cast<uint32_t>(i));
      }
    }
  }
  __syncthreads();
  if (tok && wl == 0) {
    uint32_t key[PER];
#pragma unroll
    for (int m = 0; m < PER; ++m) key[m] = (m < per && lane + 32 * m < E) ? kv[t * E + lane + 32 * m] : 0u;
    float acc = 0.0f;
    float sel = 0.0f;
    uint32_t idx = 0;
    for (int q = 0; q < k; ++q) {
      uint32_t best = 0u;
#pragma unroll
      for (int m = 0; m < PER; ++m) best = max(best, key[m]);
      best = __reduce_max_sync(0xFFFFFFFFu, best);  // one redux.sync: keys are unique, order-free
#pragma unroll
      for (int m = 0; m < PER; ++m)
        if (key[m] == best) key[m] = 0u;
      const float p = bf16_to_f32(static_cast<uint16_t>(best >> 16));
      if (lane == q) {
        sel = p;
        idx = 0xFFFFu - (best & 0xFFFFu);
      }
      acc = __fadd_rn(acc, p);
    }
    const float topm = round_bf16(acc);
    // every lane runs the same keep test on the slot probabilities (lane s holds slot s)
    const int keep = keep_count([&](int s) { return __shfl_sync(0xFFFFFFFFu, sel, s); }, k, keep_threshold, min_keep);
    float kept = 0.0f;
    for (int s = 0; s < keep; ++s) kept = __fadd_rn(kept, __shfl_sync(0xFFFFFFFFu, sel, s));
    const float selected = round_bf16(kept);
    const uint32_t idx0 = __shfl_sync(0xFFFFFFFFu, idx, 0);
    const float bl = round_bf16(blend);
    const float normalizer = badd(topm, bmul(bl, bsub(selected, topm)));
    if (lane < k) {
      const bool live = lane < keep;  // dropped slots: slot 0's expert, score 0, no expert run
      const uint32_t e = live ? idx : idx0;
      const size_t o = static_cast<size_t>(t) * k + lane;
      inds[o] = e;
      const uint32_t route = !live ? kRouteNone : route_map ? route_map[e] : (table_routes ? (kSlotBit | e) : e);
      routes[o] = route;
      s_route[o] = route;
      if (raw_scores) raw_scores[o] = live ? f32_to_bf16(sel) : 0;
      if (scores) scores[o] = live ? f32_to_bf16(__fdiv_rn(sel, normalizer)) : 0;
    }
    if (lane == 0) {
      if (mass) mass[t] = f32_to_bf16(topm);
      if (shl && shg) shg[t] = f32_to_bf16(sigmoid_bf16(g_exp_bf16, bf16_to_f32(shl[t])));
    }
  }
  __syncthreads();
  if (tiles_only) {
    route_tiles(s_route, T * k, shared_tokens, E_arr, records, gv, err, sm);
    return;
  }
  group_body(routes, T * k, shared_tokens, E_arr, records, gv, seg_warps, err, sm);
}

cudaError_t launch_route_small(const uint16_t *logits, int T, int E, int k, float blend,
                               const uint32_t *route_map, int table_routes, uint32_t *inds,
                               uint32_t *routes, uint16_t *raw_scores, uint16_t *scores,
                               uint16_t *mass, const uint16_t *shared_logit, uint16_t *shared_gate,
                               int shared_tokens, int array_experts, int table_records, GroupView gv,
                               cudaStream_t s, double keep_threshold, int min_keep, bool tiles_only) {
  const int per = (E + 31) / 32;
  if (T > kRouteSmallTokens || per > 32 || k > 32) return cudaErrorNotSupported;
  int seg_warps = 1;
  const size_t gsm = tiles_only ? 5 * kRouteSmallPairs * sizeof(int)
                                : group_smem_bytes(T * k + shared_tokens, gv.n_bins, &seg_warps);
  const size_t smem = std::max(gsm, static_cast<size_t>(T) * E * sizeof(float));
#define FNMOE_ROUTE_CASE(P)                                                                            \
  if (per <= P) {                                                                                      \
    if (smem > 48 * 1024) {                                                                            \
      cudaError_t e = cudaFuncSetAttribute(k_route_small<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                           static_cast<int>(smem));                                    \
      if (e != cudaSuccess) return e;                                                                  \
    }                                                                                                  \
    cudaError_t e = launch_pdl(k_route_small<P>, 1, 1024, smem, s, logits, T, E, k, blend, route_map,     \
                               table_routes, inds, routes, raw_scores, scores, mass, shared_logit,      \
                               shared_gate, shared_tokens, array_experts, table_records, gv, seg_warps, \
                               keep_threshold, min_keep, tiles_only ? 1 : 0, device_error_word());      \
    if (e != cudaSuccess) return e;                                                                    \
    return cudaGetLastError();                                                                         \
  }
  FNMOE_ROUTE_CASE(4)
  FNMOE_ROUTE_CASE(8)
  FNMOE_ROUTE_CASE(16)
  FNMOE_ROUTE_CASE(32)
#undef FNMOE_ROUTE_CASE
  return cudaErrorNotSupported;
}

cudaError_t launch_softmax_topk(const uint16_t *logits, int T, int E, int k, float blend,
                                const uint32_t *route_map, int table_routes, uint32_t *inds,
                                uint32_t *routes, uint16_t *raw_scores, uint16_t *scores,
                                uint16_t *mass, const uint16_t *shared_logit,
                                uint16_t *shared_gate, cudaStream_t s, double keep_threshold, int min_keep) {
  const int per = (E + 31) / 32;
#define FNMOE_TOPK_CASE(P)                                                                           \
  if (per <= P) {                                                                                   \
    cudaError_t e = launch_pdl(k_softmax_topk<P>, (T + 3) / 4, 128, 0, s, logits, T, E, k, blend,       \
                               route_map, table_routes, inds, routes, raw_scores, scores, mass,        \
                               shared_logit, shared_gate, keep_threshold, min_keep);                    \
    if (e != cudaSuccess) return e;                                                                    \
    return cudaGetLastError();                                                                    \
  }
  FNMOE_TOPK_CASE(4)
  FNMOE_TOPK_CASE(8)
  FNMOE_TOPK_CASE(16)
  FNMOE_TOPK_CASE(32)
#undef FNMOE_TOPK_CASE
  return cudaErrorInvalidValue;
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

// the batch-1 layer as one persistent kernel (uses the kernels above)
#include "decode_layer.cuh"

}  // namespace fnmoe
