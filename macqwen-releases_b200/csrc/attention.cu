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
// Decomposition: one warp per (sequence, kv head, split of `split_tokens`
// tokens); the warp walks its split 16 tokens at a time with tensor-core MMAs
//   S^T = K Q^T   (M = 16 tokens, N = 8 query heads of the GQA group, K = D)
//   O^T += V^T P^T (M = 16 head dims, N = 8 query heads, K = 16 tokens)
// and writes float32 partials (m, l, o); a second kernel merges the splits
// of a sequence in split order.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "attention.cuh"
#include "common.cuh"

namespace fnmoe {

namespace {

constexpr int kAttnWarps = 4;
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

// Address of K/V row (token t of sequence b, kv head h); nullptr if invalid.
template <int D>
__device__ __forceinline__ const uint16_t *kv_row(const PagedView &p, const uint16_t *cache, int b,
                                                  int t, int h) {
  const int pi = t / p.page_size;
  if (pi >= p.max_pages) return nullptr;
  const int page = p.table[static_cast<size_t>(b) * p.max_pages + pi];
  if (page < 0 || page >= p.num_pages) return nullptr;
  const int slot = t - pi * p.page_size;
  return cache + ((static_cast<size_t>(page) * p.page_size + slot) * p.Hkv + h) * D;
}

template <int D>
__global__ void __launch_bounds__(kAttnWarps * 32) k_paged_split(PagedView p, uint32_t *err) {
  constexpr int KS2 = D / 32;   // k-step pairs along D
  constexpr int NT = D / 16;    // output MMA tiles along D
  __shared__ __align__(16) uint16_t ps[kAttnWarps][kHeadsPerMma][16];  // P^T per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int wid = blockIdx.x * kAttnWarps + warp;
  const int per_seq = p.Hkv * p.splits_max;
  const int b = wid / per_seq;
  if (b >= p.B) return;
  const int rem = wid - b * per_seq;
  const int h = rem / p.splits_max;
  const int sp = rem - h * p.splits_max;
  const int ctx = p.ctx[b];
  const int t0 = sp * p.split;
  if (t0 >= ctx) return;
  const int t1 = min(ctx, t0 + p.split);

  // Q^T fragments: head n = r of this kv group (zero beyond gq).
  uint32_t qf[KS2][4];
  {
    const int head = h * p.gq + r;
    const bool hv = r < p.gq;
    const uint16_t *qrow = p.q + (static_cast<size_t>(b) * p.Hq + (hv ? head : 0)) * D;
#pragma unroll
    for (int m = 0; m < KS2; ++m) {
      uint4 v = hv ? __ldg(reinterpret_cast<const uint4 *>(qrow + 32 * m + 8 * c)) : make_uint4(0, 0, 0, 0);
      qf[m][0] = v.x;
      qf[m][1] = v.y;
      qf[m][2] = v.z;
      qf[m][3] = v.w;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float mrun[2] = {-INFINITY, -INFINITY};
  float lrun[2] = {0.0f, 0.0f};
  const float sl2 = p.scale * 1.4426950408889634f;

  for (int tc = t0; tc < t1; tc += 16) {
    // ---- S^T = K Q^T ----
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int ta = tc + r, tb = tc + r + 8;
    const uint16_t *ka = (ta < t1) ? kv_row<D>(p, p.k, b, ta, h) : nullptr;
    const uint16_t *kb = (tb < t1) ? kv_row<D>(p, p.k, b, tb, h) : nullptr;
#pragma unroll
    for (int m = 0; m < KS2; ++m) {
      const uint4 u = ka ? __ldg(reinterpret_cast<const uint4 *>(ka + 32 * m + 8 * c)) : make_uint4(0, 0, 0, 0);
      const uint4 w = kb ? __ldg(reinterpret_cast<const uint4 *>(kb + 32 * m + 8 * c)) : make_uint4(0, 0, 0, 0);
      mma_bf16_16816(s, u.x, w.x, u.y, w.y, qf[m][0], qf[m][1]);
      mma_bf16_16816(s, u.z, w.z, u.w, w.w, qf[m][2], qf[m][3]);
    }
    // s[0]: (tok r, head 2c) s[1]: (tok r, head 2c+1) s[2]: (tok r+8, 2c) s[3]: (tok r+8, 2c+1)
    const bool va = ka != nullptr, vb = kb != nullptr;
    float x0 = va ? s[0] * sl2 : -INFINITY;
    float x1 = va ? s[1] * sl2 : -INFINITY;
    float x2 = vb ? s[2] * sl2 : -INFINITY;
    float x3 = vb ? s[3] * sl2 : -INFINITY;
    float cm0 = fmaxf(x0, x2), cm1 = fmaxf(x1, x3);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      cm0 = fmaxf(cm0, __shfl_xor_sync(0xFFFFFFFFu, cm0, off));
      cm1 = fmaxf(cm1, __shfl_xor_sync(0xFFFFFFFFu, cm1, off));
    }
    const float mn0 = fmaxf(mrun[0], cm0), mn1 = fmaxf(mrun[1], cm1);
    // A chunk whose rows were all skipped (invalid pages) keeps -inf; use a
    // finite reference so exp2 never sees -inf - -inf.
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
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al1;
      o[j][2] *= al0;
      o[j][3] *= al1;
    }
    // P^T to shared memory: ps[head][token]
    ps[warp][2 * c][r] = f32_to_bf16(p0);
    ps[warp][2 * c + 1][r] = f32_to_bf16(p1);
    ps[warp][2 * c][r + 8] = f32_to_bf16(p2);
    ps[warp][2 * c + 1][r + 8] = f32_to_bf16(p3);
    __syncwarp();
    const uint32_t pb0 = *reinterpret_cast<const uint32_t *>(&ps[warp][r][2 * c]);
    const uint32_t pb1 = *reinterpret_cast<const uint32_t *>(&ps[warp][r][2 * c + 8]);
    __syncwarp();
    // ---- O^T += V^T P^T ----
    const int tv0 = tc + 2 * c, tv1 = tv0 + 1, tv2 = tv0 + 8, tv3 = tv0 + 9;
    const uint16_t *v0 = (tv0 < t1) ? kv_row<D>(p, p.v, b, tv0, h) : nullptr;
    const uint16_t *v1 = (tv1 < t1) ? kv_row<D>(p, p.v, b, tv1, h) : nullptr;
    const uint16_t *v2 = (tv2 < t1) ? kv_row<D>(p, p.v, b, tv2, h) : nullptr;
    const uint16_t *v3 = (tv3 < t1) ? kv_row<D>(p, p.v, b, tv3, h) : nullptr;
#pragma unroll
    for (int J = 0; J < D / 64; ++J) {
      const int off = 64 * J + 8 * r;
      const uint4 u0 = v0 ? __ldg(reinterpret_cast<const uint4 *>(v0 + off)) : make_uint4(0, 0, 0, 0);
      const uint4 u1 = v1 ? __ldg(reinterpret_cast<const uint4 *>(v1 + off)) : make_uint4(0, 0, 0, 0);
      const uint4 u2 = v2 ? __ldg(reinterpret_cast<const uint4 *>(v2 + off)) : make_uint4(0, 0, 0, 0);
      const uint4 u3 = v3 ? __ldg(reinterpret_cast<const uint4 *>(v3 + off)) : make_uint4(0, 0, 0, 0);
      const uint32_t a0s[4] = {u0.x, u0.y, u0.z, u0.w};
      const uint32_t a1s[4] = {u1.x, u1.y, u1.z, u1.w};
      const uint32_t a2s[4] = {u2.x, u2.y, u2.z, u2.w};
      const uint32_t a3s[4] = {u3.x, u3.y, u3.z, u3.w};
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const uint32_t A0 = __byte_perm(a0s[jj], a1s[jj], 0x5410);
        const uint32_t A1 = __byte_perm(a0s[jj], a1s[jj], 0x7632);
        const uint32_t A2 = __byte_perm(a2s[jj], a3s[jj], 0x5410);
        const uint32_t A3 = __byte_perm(a2s[jj], a3s[jj], 0x7632);
        mma_bf16_16816(o[4 * J + jj], A0, A1, A2, A3, pb0, pb1);
      }
    }
  }
  // o[j]: c0 (dim x, head 2c) c1 (dim x, head 2c+1) c2 (dim x+1, head 2c) c3 (dim x+1, head 2c+1)
  // with x = 64*(j/4) + 8r + 2*(j%4).
  const size_t seq_base = ((static_cast<size_t>(b) * p.Hkv + h) * p.splits_max + sp) * p.gq;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int head = 2 * c + hh;
    if (head >= p.gq) continue;
    float *dst = p.part + (seq_base + head) * (D + 2);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int x = 64 * (j >> 2) + 8 * r + 2 * (j & 3);
      dst[x] = o[j][hh];
      dst[x + 1] = o[j][2 + hh];
    }
    if (r == 0) {
      dst[D] = mrun[hh];
      dst[D + 1] = lrun[hh];
    }
  }
}

template <int D>
__global__ void k_paged_merge(PagedView p, uint16_t *__restrict__ out) {
  const int bh = blockIdx.x;  // b * Hq + head
  const int b = bh / p.Hq, head = bh - b * p.Hq;
  const int h = head / p.gq, hq = head - h * p.gq;
  const int d = threadIdx.x;
  if (d >= D) return;
  const int ctx = p.ctx[b];
  const int ns = (ctx + p.split - 1) / p.split;
  float m = -INFINITY;
  for (int s = 0; s < ns; ++s) {
    const float *src = p.part + ((((static_cast<size_t>(b) * p.Hkv + h) * p.splits_max + s) * p.gq) + hq) * (D + 2);
    m = fmaxf(m, src[D]);
  }
  float L = 0.0f, O = 0.0f;
  for (int s = 0; s < ns; ++s) {
    const float *src = p.part + ((((static_cast<size_t>(b) * p.Hkv + h) * p.splits_max + s) * p.gq) + hq) * (D + 2);
    const float w = (src[D] == -INFINITY) ? 0.0f : exp2f(src[D] - m);
    L += src[D + 1] * w;
    O += src[d] * w;
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
  return FNMOE_OK;
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
  const uint64_t warps = static_cast<uint64_t>(p.B) * p.Hkv * p.splits_max;
  const unsigned blocks = static_cast<unsigned>((warps + kAttnWarps - 1) / kAttnWarps);
  cudaError_t e;
  switch (a->head_dim) {
    case 64:
      k_paged_split<64><<<blocks, kAttnWarps * 32, 0, s>>>(p, nullptr);
      k_paged_merge<64><<<p.B * p.Hq, 64, 0, s>>>(p, static_cast<uint16_t *>(a->out));
      break;
    case 128:
      k_paged_split<128><<<blocks, kAttnWarps * 32, 0, s>>>(p, nullptr);
      k_paged_merge<128><<<p.B * p.Hq, 128, 0, s>>>(p, static_cast<uint16_t *>(a->out));
      break;
    default:
      k_paged_split<256><<<blocks, kAttnWarps * 32, 0, s>>>(p, nullptr);
      k_paged_merge<256><<<p.B * p.Hq, 256, 0, s>>>(p, static_cast<uint16_t *>(a->out));
      break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("paged decode: ") + cudaGetErrorString(e);
    return FNMOE_ERR_LAUNCH;
  }
  return FNMOE_OK;
}

}  // namespace fnmoe
