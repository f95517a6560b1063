// common.cuh -- shared device helpers for the fnmoe sm_100a kernels.
//
// Rounding conventions (identical to the CPU oracle):
//   * bfloat16 results are float32 results rounded to nearest even;
//   * float32 arithmetic uses the explicit _rn intrinsics wherever the oracle
//     fixes the operation order, so the compiler cannot contract to FMA;
//   * exp() feeding bfloat16 is correctly rounded through a 64 Ki-entry table
//     built once per device from double-precision exp().
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fnmoe {

constexpr uint32_t kSlotBit = 0x80000000u;
constexpr uint32_t kRouteNone = 0xFFFFFFFFu;  // FNMOE_ROUTE_NONE: an empty slot, skipped
constexpr int kWarp = 32;

// Device error word bits (fnmoe_read_device_errors).
constexpr uint32_t kErrBadRoute = 1u;
constexpr uint32_t kErrNonFinite = 2u;
constexpr uint32_t kErrTimeout = 4u;
constexpr uint32_t kErrBadTile = 8u;  // a prefill tile descriptor out of range (skipped)

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float round_bf16(float f) {
  return bf16_to_f32(f32_to_bf16(f));
}

// double -> bfloat16 bits with a single rounding (nearest even).
__device__ __forceinline__ uint16_t f64_to_bf16_once(double d) {
  if (isnan(d)) return 0x7FC0u;
  const uint64_t u = static_cast<uint64_t>(__double_as_longlong(d));
  const uint16_t sign = static_cast<uint16_t>((u >> 48) & 0x8000u);
  const double a = fabs(d);
  // (2 - 2^-8) * 2^127: at or above it bfloat16 rounds to infinity.
  if (a >= 0x1.FEp+127) return sign | 0x7F80u;
  if (a >= 0x1p-126) {  // bfloat16 normal range
    uint64_t bits = u & 0x7FFFFFFFFFFFFFFFull;
    const uint64_t lsb = (bits >> 45) & 1ull;
    bits += (1ull << 44) - 1ull + lsb;
    bits &= ~((1ull << 45) - 1ull);
    const float f = static_cast<float>(__longlong_as_double(static_cast<long long>(bits)));
    return sign | static_cast<uint16_t>(__float_as_uint(f) >> 16);
  }
  // subnormal bfloat16: multiples of 2^-133.
  const long long n = __double2ll_rn(a * 0x1p133);  // a * 2^133 (exact scaling)
  return sign | static_cast<uint16_t>(n);
}

// exp() of a bfloat16 value rounded once to bfloat16, read from a 64 Ki-entry
// table (built once per device by the translation unit that owns it).
__device__ __forceinline__ float exp_bf16(const uint16_t *tab, float v) {
  return bf16_to_f32(tab[f32_to_bf16(v)]);
}

// One bfloat16 operation: float32 op then round (Metal bfloat semantics).
__device__ __forceinline__ float badd(float a, float b) { return round_bf16(__fadd_rn(a, b)); }
__device__ __forceinline__ float bsub(float a, float b) { return round_bf16(__fsub_rn(a, b)); }
__device__ __forceinline__ float bmul(float a, float b) { return round_bf16(__fmul_rn(a, b)); }
__device__ __forceinline__ float bdiv(float a, float b) { return round_bf16(__fdiv_rn(a, b)); }

// Stable bfloat16 sigmoid: |g| -> exp -> 1+e -> 1/d -> select
// (metal_runtime.py:272-281).
__device__ __forceinline__ float sigmoid_bf16(const uint16_t *tab, float g) {
  const float mag = fabsf(g);
  const float ex = exp_bf16(tab, mag);
  const float den = badd(1.0f, ex);
  const float small = bdiv(1.0f, den);
  return (g < 0.0f) ? small : bsub(1.0f, small);
}

// (g * sigmoid(g)) * u, each op rounded to bfloat16 (metal_runtime.py:282).
__device__ __forceinline__ float swiglu_bf16(const uint16_t *tab, float g, float u) {
  return bmul(bmul(g, sigmoid_bf16(tab, g)), u);
}

// The same two sequences with exp computed in registers instead of read from
// the table: the table holds exactly f64_to_bf16_once(exp(double(v))) for
// every bfloat16 v, so the bits are identical; used where a table lookup (an
// L2 round trip) would sit on a latency-critical path.
__device__ __forceinline__ float exp_bf16_direct(float v) {
  return bf16_to_f32(f64_to_bf16_once(exp(static_cast<double>(round_bf16(v)))));
}
__device__ __forceinline__ float sigmoid_bf16_direct(float g) {
  const float mag = fabsf(g);
  const float ex = exp_bf16_direct(mag);
  const float den = badd(1.0f, ex);
  const float small = bdiv(1.0f, den);
  return (g < 0.0f) ? small : bsub(1.0f, small);
}
__device__ __forceinline__ float swiglu_bf16_direct(float g, float u) {
  return bmul(bmul(g, sigmoid_bf16_direct(g)), u);
}

// The same sequence with float32 activations (the reference's kernel with
// T = float): every op rounded to float32, exp correctly rounded (float64
// exp, one rounding).
__device__ __forceinline__ float swiglu_f32(float g, float u) {
  const float ex = __double2float_rn(exp(static_cast<double>(fabsf(g))));
  const float small = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
  const float sig = (g < 0.0f) ? small : __fsub_rn(1.0f, small);
  return __fmul_rn(__fmul_rn(g, sig), u);
}

// m16n8k16 fp16 MMA, fp32 accumulate (exact here: all operands are small
// integers and every partial sum stays below 2^24).
__device__ __forceinline__ void mma_16816(float c[4], const uint32_t a[4],
                                          uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// The same with a zero accumulator input.
__device__ __forceinline__ void mma_16816_z(float c[4], const uint32_t a[4],
                                            uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// Nibbles j and j+4 of a packed word as an fp16x2 pair (low half = nibble j).
// (w >> 4j) & 0x000F000F | 0x6400 6400 encodes 1024+q; subtracting 1024 is
// exact in fp16.
__device__ __forceinline__ uint32_t nibble_pair(uint32_t w, int j) {
  const uint32_t v = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
  __half2 h = *reinterpret_cast<const __half2 *>(&v);
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  h = __hsub2(h, k1024);
  return *reinterpret_cast<uint32_t *>(&h);
}

// MMA A operands of one 32-value group for two rows: A0 = {a j0, b j0, a j1,
// b j1} and A1 = {a j2, b j2, a j3, b j3}, where "x jN" is the fp16x2 pair of
// nibbles (N, N+4) of word x (rows r and r+8 of the m16n8k16 fragment).
// Even pairs use the 1024 + q encoding, odd pairs the unshifted 1024 + 16q.
__device__ __forceinline__ void nibble_operands(uint32_t wa, uint32_t wb, uint32_t A0[4], uint32_t A1[4]) {
  // (w & mask) | 0x6400 per half is 1024 + q (mask 0x000F) or 1024 + 16q
  // (mask 0x00F0); subtracting 1024, or scaling by 1/16 and adding -64,
  // leaves q exactly.  lop3 LUT 0xEA = (a & b) | c.
  asm("{\n"
      ".reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, a8, b8;\n"
      "shr.b32 a8, %8, 8;\n"
      "shr.b32 b8, %9, 8;\n"
      "lop3.b32 t0, %8, 0x000F000F, 0x64006400, 0xEA;\n"
      "lop3.b32 t1, %9, 0x000F000F, 0x64006400, 0xEA;\n"
      "lop3.b32 t2, %8, 0x00F000F0, 0x64006400, 0xEA;\n"
      "lop3.b32 t3, %9, 0x00F000F0, 0x64006400, 0xEA;\n"
      "lop3.b32 t4, a8, 0x000F000F, 0x64006400, 0xEA;\n"
      "lop3.b32 t5, b8, 0x000F000F, 0x64006400, 0xEA;\n"
      "lop3.b32 t6, a8, 0x00F000F0, 0x64006400, 0xEA;\n"
      "lop3.b32 t7, b8, 0x00F000F0, 0x64006400, 0xEA;\n"
      "sub.f16x2 %0, t0, %10;\n"
      "sub.f16x2 %1, t1, %10;\n"
      "fma.rn.f16x2 %2, t2, %11, %12;\n"
      "fma.rn.f16x2 %3, t3, %11, %12;\n"
      "sub.f16x2 %4, t4, %10;\n"
      "sub.f16x2 %5, t5, %10;\n"
      "fma.rn.f16x2 %6, t6, %11, %12;\n"
      "fma.rn.f16x2 %7, t7, %11, %12;\n"
      "}\n"
      : "=r"(A0[0]), "=r"(A0[1]), "=r"(A0[2]), "=r"(A0[3]), "=r"(A1[0]), "=r"(A1[1]), "=r"(A1[2]), "=r"(A1[3])
      : "r"(wa), "r"(wb), "r"(0x64006400u), "r"(0x2C002C00u), "r"(0xD400D400u));
}

// All four nibble pairs (j, j+4), j = 0..3, of a packed word as fp16x2.
// Odd pairs are taken unshifted from bits 4-7 / 20-23: the encoded value is
// 1024 + 16q, and 1024 + 16q scaled by 1/16 minus 64 is q exactly.
__device__ __forceinline__ void nibble_pairs4(uint32_t w, uint32_t out[4]) {
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  const __half2 k16th = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
  const __half2 km64 = __halves2half2(__ushort_as_half(0xD400), __ushort_as_half(0xD400));   // -64
  const uint32_t w8 = w >> 8;
  uint32_t v0 = (w & 0x000F000Fu) | 0x64006400u;
  uint32_t v1 = (w & 0x00F000F0u) | 0x64006400u;
  uint32_t v2 = (w8 & 0x000F000Fu) | 0x64006400u;
  uint32_t v3 = (w8 & 0x00F000F0u) | 0x64006400u;
  __half2 h0 = __hsub2(*reinterpret_cast<const __half2 *>(&v0), k1024);
  __half2 h1 = __hfma2(*reinterpret_cast<const __half2 *>(&v1), k16th, km64);
  __half2 h2 = __hsub2(*reinterpret_cast<const __half2 *>(&v2), k1024);
  __half2 h3 = __hfma2(*reinterpret_cast<const __half2 *>(&v3), k16th, km64);
  out[0] = *reinterpret_cast<uint32_t *>(&h0);
  out[1] = *reinterpret_cast<uint32_t *>(&h1);
  out[2] = *reinterpret_cast<uint32_t *>(&h2);
  out[3] = *reinterpret_cast<uint32_t *>(&h3);
}

// Load helpers with read-only caching.
__device__ __forceinline__ uint32_t ldg_u32(const uint32_t *p) { return __ldg(p); }
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t *p) { return __ldg(p); }
__device__ __forceinline__ uint4 ldg_u128(const uint4 *p) { return __ldg(p); }

__device__ __forceinline__ void set_error(uint32_t *err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

// Metadata row of a fixed-point input row (floats): fl(SX) of each of the
// Gc groups, zero padding to a multiple of 4, then {A, B, 0, 0} with
// A * B = 2^(E-22), A = 2^max(E-22, -126).
__host__ __device__ __forceinline__ int meta_a_index(int groups) { return ((groups + 3) / 4) * 4; }
__host__ __device__ __forceinline__ int meta_pitch(int groups) { return meta_a_index(groups) + 4; }

// Programmatic dependent launch.  A kernel started by launch_pdl may begin
// while the previous kernel of its stream is still running: pdl_wait()
// blocks until that kernel has completed and its writes are visible.  Every
// kernel launched this way calls pdl_wait() before it reads data written by
// an earlier kernel and before its own global writes, so each kernel still
// completes after all earlier ones.  pdl_trigger() lets the next kernel of
// the stream start launching.  Since such a kernel is alive while its
// predecessor writes, data produced by earlier kernels is never read through
// the non-coherent path (no __ldg, no const __restrict__ pointers): that
// path assumes data read-only for the kernel's whole lifetime.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// false when FNMOE_NO_PDL is set in the environment (plain stream order).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace fnmoe
