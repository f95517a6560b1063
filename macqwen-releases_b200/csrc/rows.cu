// rows.cu -- quantized embedding / n-gram row lookup for sm_100a.
//
// Replaces the decode-time row reads of StreamingQuantizedEmbedding
// (models/flashnext/ngram.py:28-69) and StreamingShardedEmbedding
// (ngram.py:82-188): there a lookup reads a few packed rows from the
// checkpoint and runs mx.dequantize on them.  Here the whole table -- the
// shards of a sharded table concatenated in shard order -- is resident in
// HBM, and one launch gathers and dequantises every requested row:
//
//   out[i, k] = bf16(s * q + b),  q = value k of packed row r(i), s and b the
//   bfloat16 scale and bias of k's group, rounded once from the exact value.
//
// r(i) follows the sharded lookup's clamping (ngram.py:106-119): an index in
// [0, table_rows) addresses that row of the concatenated table; any other
// index reads shard 0's row clamp(index, 0, first_shard_rows - 1).
//
// Layout: weight [table_rows][dims * bits / 32] uint32, value j of a word in
// bits [j * bits, (j + 1) * bits) (low bits first, MLX's affine packing for
// bits 2, 4 and 8); scales, biases [table_rows][dims / group_size] bf16;
// out [count][dims] bf16.
//
// Decomposition: one warp per output row.  A unit is 8 consecutive values
// (16 output bytes, `bits` packed bytes, one group); lane l takes units l,
// l + 32, ... so every load and store instruction of the warp covers a
// contiguous span.  The table is read-only for the launch (__ldg).
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/fnmoe.h"
#include "common.cuh"
#include "rows.cuh"

namespace fnmoe {

namespace {

constexpr int kRowsWarps = 8;

struct RowsView {
  const uint8_t *weight;
  const uint16_t *scales, *biases;
  const int64_t *indices;
  uint16_t *out;
  uint64_t count, table_rows, first_shard_rows;
  int dims, group_shift, groups;
};

// bf16(s * q + b) rounded once from the exact value.  fma rounds the exact
// value once to float32; rounding that to bfloat16 is the single rounding
// unless the float32 result sits exactly on a bfloat16 midpoint (low half
// 0x8000), where the float32 rounding may have moved the value onto the tie:
// that case (and NaN) takes the exact float64 route.
__device__ __forceinline__ uint16_t dequant_once(float s, float b, uint32_t q) {
  const float r = __fmaf_rn(s, static_cast<float>(q), b);
  const uint32_t bits = __float_as_uint(r);
  if ((bits & 0xFFFFu) == 0x8000u || r != r)
    return f64_to_bf16_once(static_cast<double>(s) * static_cast<double>(q) + static_cast<double>(b));
  return f32_to_bf16(r);
}

template <int BITS>
__global__ void __launch_bounds__(kRowsWarps * 32) k_rows_dequant(RowsView v) {
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * kRowsWarps + warp;
  if (i >= v.count) return;
  const int64_t idx = v.indices[i];
  uint64_t r;
  if (idx >= 0 && static_cast<uint64_t>(idx) < v.table_rows) {
    r = static_cast<uint64_t>(idx);
  } else {
    r = idx < 0 ? 0 : v.first_shard_rows - 1;
  }
  const uint8_t *wrow = v.weight + r * static_cast<uint64_t>(v.dims) * BITS / 8;
  const uint16_t *srow = v.scales + r * v.groups;
  const uint16_t *brow = v.biases + r * v.groups;
  uint4 *orow = reinterpret_cast<uint4 *>(v.out + i * v.dims);
  const int units = v.dims / 8;
  for (int u = lane; u < units; u += 32) {
    // 8 values = BITS packed bytes
    uint32_t w0, w1 = 0;
    if (BITS == 4) {
      w0 = __ldg(reinterpret_cast<const uint32_t *>(wrow) + u);
    } else if (BITS == 8) {
      const uint2 t = __ldg(reinterpret_cast<const uint2 *>(wrow) + u);
      w0 = t.x;
      w1 = t.y;
    } else {
      w0 = __ldg(reinterpret_cast<const uint16_t *>(wrow) + u);
    }
    const int g = (u * 8) >> v.group_shift;
    const float s = bf16_to_f32(__ldg(srow + g));
    const float b = bf16_to_f32(__ldg(brow + g));
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      uint32_t q0, q1;
      if (BITS == 8) {
        const uint32_t w = e < 4 ? w0 : w1;
        q0 = (w >> (8 * (e & 3))) & kMask;
        q1 = (w >> (8 * ((e + 1) & 3))) & kMask;
      } else {
        q0 = (w0 >> (BITS * e)) & kMask;
        q1 = (w0 >> (BITS * (e + 1))) & kMask;
      }
      o[e >> 1] = static_cast<uint32_t>(dequant_once(s, b, q0)) |
                  (static_cast<uint32_t>(dequant_once(s, b, q1)) << 16);
    }
    orow[u] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

int rows_dequant(const FnRowsArgs *a, cudaStream_t s, std::string &err) {
  if (a == nullptr) { err = "args is NULL"; return FNMOE_ERR_NULL; }
  if (a->abi_version != FNMOE_ABI_VERSION) { err = "abi_version mismatch"; return FNMOE_ERR_ABI; }
  if (a->count == 0) return FNMOE_OK;
  if (!a->weight || !a->scales || !a->biases || !a->indices || !a->out) {
    err = "weight, scales, biases, indices and out are required";
    return FNMOE_ERR_NULL;
  }
  if (a->bits != 2 && a->bits != 4 && a->bits != 8) { err = "bits must be 2, 4 or 8"; return FNMOE_ERR_UNSUPPORTED; }
  if (a->group_size != 32 && a->group_size != 64 && a->group_size != 128) {
    err = "group_size must be 32, 64 or 128";
    return FNMOE_ERR_UNSUPPORTED;
  }
  if (a->dims == 0 || a->dims % a->group_size) { err = "dims must be a positive multiple of group_size"; return FNMOE_ERR_SHAPE; }
  if (a->table_rows == 0 || a->first_shard_rows == 0 || a->first_shard_rows > a->table_rows) {
    err = "table_rows and first_shard_rows must satisfy 0 < first_shard_rows <= table_rows";
    return FNMOE_ERR_SHAPE;
  }
  // packed rows are read in bits-byte units, outputs stored 16 bytes at a time
  if ((reinterpret_cast<uintptr_t>(a->weight) & 7u) || (reinterpret_cast<uintptr_t>(a->out) & 15u) ||
      (reinterpret_cast<uintptr_t>(a->scales) & 1u) || (reinterpret_cast<uintptr_t>(a->biases) & 1u) ||
      (reinterpret_cast<uintptr_t>(a->indices) & 7u)) {
    err = "weight must be 8-byte, out 16-byte, indices 8-byte and scales/biases 2-byte aligned";
    return FNMOE_ERR_VALUE;
  }
  RowsView v{};
  v.weight = reinterpret_cast<const uint8_t *>(a->weight);
  v.scales = static_cast<const uint16_t *>(a->scales);
  v.biases = static_cast<const uint16_t *>(a->biases);
  v.indices = a->indices;
  v.out = static_cast<uint16_t *>(a->out);
  v.count = a->count;
  v.table_rows = a->table_rows;
  v.first_shard_rows = a->first_shard_rows;
  v.dims = static_cast<int>(a->dims);
  v.group_shift = a->group_size == 32 ? 5 : a->group_size == 64 ? 6 : 7;
  v.groups = static_cast<int>(a->dims / a->group_size);
  const uint64_t blocks = (a->count + kRowsWarps - 1) / kRowsWarps;
  if (blocks > 0x7FFFFFFFull) { err = "too many rows"; return FNMOE_ERR_SHAPE; }
  switch (a->bits) {
    case 2: k_rows_dequant<2><<<static_cast<unsigned>(blocks), kRowsWarps * 32, 0, s>>>(v); break;
    case 4: k_rows_dequant<4><<<static_cast<unsigned>(blocks), kRowsWarps * 32, 0, s>>>(v); break;
    default: k_rows_dequant<8><<<static_cast<unsigned>(blocks), kRowsWarps * 32, 0, s>>>(v); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("rows dequant: ") + cudaGetErrorString(e);
    return FNMOE_ERR_LAUNCH;
  }
  return FNMOE_OK;
}

}  // namespace fnmoe
