// ep.cu -- expert-parallel token exchange over NVLink peer memory.
//
// One process per GPU; rank r owns routed experts [r*per, (r+1)*per).  Each
// rank holds one exchange window (cudaMalloc'd at set-up, shared with the
// other ranks of the node through CUDA IPC handles) that its peers write
// into with plain stores over NVLink -- no collective library, no padding to
// a fixed capacity, no host synchronisation, so a step can be captured in a
// CUDA graph.  Per step (epoch e = step + 1, `step` a counter in the window):
//
//   dispatch  for every (token t, destination d): the k + 1 owner-local
//             expert ids of t's slots on d (FNMOE_ROUTE_NONE elsewhere; slot
//             k is the shared expert, run by the token's own rank) go to
//             d's window at [src = this rank][t]; t's x row goes there too
//             when any id is live.  Each destination's last CTA publishes
//             flag dflag[src] = e in d's window (release, system scope).
//   wait      this rank waits (bounded) until every source's dflag >= e.
//   experts   the caller runs its experts on the window's [world * cap]
//             rows with k + 1 slots each (fnmoe_moe_execute, per-slot
//             outputs into the window's local output area).
//   return    every live routed (row, slot) output goes back to the row's
//             source rank, into its return area at [t][slot]; then rflag.
//   combine   the source waits for every rflag >= e and combines its tokens
//             in slot order with the gated shared expert (k_combine's
//             arithmetic), bit-identical to the one-GPU layer.
//   advance   step += 1.
//
// One buffer per area is enough: a rank writes a peer's dispatch area for
// step n + 1 only after its own step-n combine, which waited for every
// peer's step-n return, which each peer issues after its step-n experts
// have read that area; the return area is covered the same way.  Waits give
// up after ~1 s, set kErrTimeout and skip their work.  No TMA or bulk copy
// touches peer memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/fnmoe.h"
#include "common.cuh"
#include "moe_kernels.cuh"

namespace fnmoe {

namespace {

constexpr int kEpMaxWorld = 8;
constexpr int kEpThreads = 256;
constexpr int kEpMaxSlots = 16;  // top_k limit
constexpr uint32_t kEpSpinLimit = 1u << 24;  // polls with a 64 ns back-off: ~1-2 s

struct EpLayout {
  uint64_t rows, ids, ret, dflag, rflag, ddone, rdone, step, dlocal, total;
};

EpLayout ep_layout(int world, int cap, int H, int k) {
  auto up = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
  EpLayout L{};
  uint64_t o = 0;
  L.rows = o;
  o = up(o + static_cast<uint64_t>(world) * cap * H * 2);
  L.ids = o;
  o = up(o + static_cast<uint64_t>(world) * cap * (k + 1) * 4);
  L.ret = o;
  o = up(o + static_cast<uint64_t>(cap) * k * H * 2);
  L.dflag = o;
  o = up(o + kEpMaxWorld * 64);  // one 64-byte line per source
  L.rflag = o;
  o = up(o + kEpMaxWorld * 64);
  L.ddone = o;
  o = up(o + kEpMaxWorld * 64);
  L.rdone = o;
  o = up(o + kEpMaxWorld * 64);
  L.step = o;
  o = up(o + 64);
  L.dlocal = o;
  o = up(o + static_cast<uint64_t>(world) * cap * (k + 1) * H * 2);
  L.total = o;
  return L;
}

struct EpView {
  uint8_t *peer[kEpMaxWorld];  // every rank's window (this rank's own included)
  int world, rank, cap, H, k, per;
  EpLayout L;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t *flag_at(uint8_t *base, uint64_t off, int src) {
  return reinterpret_cast<uint32_t *>(base + off + static_cast<uint64_t>(src) * 64);
}

// Bounded wait until *f >= e; false (and kErrTimeout) if it gave up.
__device__ __forceinline__ bool wait_flag(const uint32_t *f, uint32_t e, uint32_t *err) {
  uint32_t spins = 0;
  while (ld_acquire_sys(f) < e) {
    if (++spins >= kEpSpinLimit) {
      set_error(err, kErrTimeout);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// After this CTA's stores to destination `d`: fence them, count the CTA in
// this rank's `done` counter for d, and let the last CTA of the step publish
// flag = e in d's window.  `done` counts monotonically: e * ctas after step e.
__device__ __forceinline__ void publish(const EpView &v, uint64_t done_off, uint64_t flag_off, int d, uint32_t e) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t *done = flag_at(v.peer[v.rank], done_off, d);
    const uint32_t prev = atomicAdd(done, 1u);
    if (prev + 1u == e * gridDim.y) {
      __threadfence_system();
      st_release_sys(flag_at(v.peer[d], flag_off, v.rank), e);
    }
  }
}

// grid (world, ctas per destination): CTA (d, c) sends tokens c, c + ctas, ...
__global__ void __launch_bounds__(kEpThreads) k_ep_dispatch(EpView v, const uint16_t *x, const uint32_t *inds,
                                                            int T, uint32_t *err) {
  __shared__ uint32_t s_ids[kEpMaxSlots + 1];
  __shared__ int s_any;
  const int d = blockIdx.x, c = blockIdx.y;
  const int tid = threadIdx.x;
  const int k = v.k;
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(v.peer[v.rank] + v.L.step) + 1u;
  uint8_t *dst = v.peer[d];
  for (int t = c; t < v.cap; t += gridDim.y) {
    if (tid == 0) s_any = 0;
    __syncthreads();
    if (tid <= k) {
      uint32_t id = kRouteNone;
      if (t < T) {
        if (tid < k) {
          const uint32_t r = inds[static_cast<size_t>(t) * k + tid];
          if (r / static_cast<uint32_t>(v.per) == static_cast<uint32_t>(d)) id = r - static_cast<uint32_t>(d * v.per);
        } else if (d == v.rank) {
          id = static_cast<uint32_t>(v.per);  // the shared expert: the last local record
        }
      }
      s_ids[tid] = id;
      if (id != kRouteNone) s_any = 1;
    }
    __syncthreads();
    uint32_t *ids = reinterpret_cast<uint32_t *>(dst + v.L.ids) + (static_cast<size_t>(v.rank) * v.cap + t) * (k + 1);
    if (tid <= k) ids[tid] = s_ids[tid];
    if (s_any) {
      const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * v.H);
      uint4 *row = reinterpret_cast<uint4 *>(dst + v.L.rows) + (static_cast<size_t>(v.rank) * v.cap + t) * (v.H / 8);
      for (int i = tid; i < v.H / 8; i += kEpThreads) row[i] = src[i];
    }
    __syncthreads();  // s_any / s_ids are rewritten for the next token
  }
  publish(v, v.L.ddone, v.L.dflag, d, e);
}

// one warp: wait until every source has published flag >= e in this window
__global__ void k_ep_wait(EpView v, uint64_t flag_off, uint32_t *err) {
  const int src = threadIdx.x;
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(v.peer[v.rank] + v.L.step) + 1u;
  if (src < v.world) wait_flag(flag_at(v.peer[v.rank], flag_off, src), e, err);
}

// grid (world, ctas per source): CTA (s, c) returns rows c, c + ctas, ... of
// source s: every live routed slot's output row to s's return area
__global__ void __launch_bounds__(kEpThreads) k_ep_return(EpView v, uint32_t *err) {
  const int src = blockIdx.x, c = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k = v.k;
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(v.peer[v.rank] + v.L.step) + 1u;
  uint8_t *self = v.peer[v.rank];
  uint8_t *dst = v.peer[src];
  const int chunks = v.H / 8;
  for (int t = c; t < v.cap; t += gridDim.y) {
    const uint32_t *ids = reinterpret_cast<const uint32_t *>(self + v.L.ids) + (static_cast<size_t>(src) * v.cap + t) * (k + 1);
    // warp w copies slots w, w + 8, ...
    for (int s = warp; s < k; s += kEpThreads / 32) {
      if (ids[s] == kRouteNone) continue;
      const uint4 *from = reinterpret_cast<const uint4 *>(self + v.L.dlocal) +
                          ((static_cast<size_t>(src) * v.cap + t) * (k + 1) + s) * chunks;
      uint4 *to = reinterpret_cast<uint4 *>(dst + v.L.ret) + (static_cast<size_t>(t) * k + s) * chunks;
      for (int i = lane; i < chunks; i += 32) to[i] = from[i];
    }
  }
  publish(v, v.L.rdone, v.L.rflag, src, e);
}

// One CTA per token (8 hidden elements per thread): wait for every owner's
// return, then the slot-ordered float32 combine (no fused multiply-add) and
// the gated shared expert -- k_combine's kCombineParts arithmetic.
__global__ void __launch_bounds__(512) k_ep_combine(EpView v, const uint16_t *scores, const uint16_t *shared_gate,
                                                    int T, uint16_t *__restrict__ out, uint32_t *err) {
  __shared__ int s_ok;
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  const int k = v.k;
  uint8_t *self = v.peer[v.rank];
  const uint32_t e = *reinterpret_cast<volatile uint32_t *>(self + v.L.step) + 1u;
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < v.world && !wait_flag(flag_at(self, v.L.rflag, tid), e, err)) s_ok = 0;
  __syncthreads();
  if (!s_ok || t >= T || 8 * tid >= v.H) return;
  const int chunks = v.H / 8;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  for (int s = 0; s < k; ++s) {
    const uint4 dv = __ldcg(reinterpret_cast<const uint4 *>(self + v.L.ret) + (static_cast<size_t>(t) * k + s) * chunks + tid);
    const float sc = bf16_to_f32(scores[static_cast<size_t>(t) * k + s]);
    const uint32_t w[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float dj = __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
      acc[j] = __fadd_rn(acc[j], __fmul_rn(dj, sc));
    }
  }
  const uint4 sv = __ldcg(reinterpret_cast<const uint4 *>(self + v.L.dlocal) +
                          ((static_cast<size_t>(v.rank) * v.cap + t) * (k + 1) + k) * chunks + tid);
  const float gate = bf16_to_f32(shared_gate[t]);
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float r2[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = 2 * q + hh;
      const float sh = __uint_as_float(hh ? (sw[q] & 0xFFFF0000u) : (sw[q] << 16));
      r2[hh] = __fadd_rn(round_bf16(acc[j]), bmul(sh, gate));
    }
    o[q] = static_cast<uint32_t>(f32_to_bf16(r2[0])) | (static_cast<uint32_t>(f32_to_bf16(r2[1])) << 16);
  }
  reinterpret_cast<uint4 *>(out + static_cast<size_t>(t) * v.H)[tid] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void k_ep_advance(EpView v) {
  uint32_t *step = reinterpret_cast<uint32_t *>(v.peer[v.rank] + v.L.step);
  *step = *step + 1u;
}

struct EpHandle {
  int device;
  int world, rank, cap, H, k, per;
  EpLayout L;
  uint8_t *window;
  uint8_t *peers[kEpMaxWorld];
  bool opened;
  cudaIpcMemHandle_t ipc;
};

EpView view_of(const EpHandle *h) {
  EpView v{};
  for (int i = 0; i < kEpMaxWorld; ++i) v.peer[i] = i < h->world ? h->peers[i] : nullptr;
  v.world = h->world;
  v.rank = h->rank;
  v.cap = h->cap;
  v.H = h->H;
  v.k = h->k;
  v.per = h->per;
  v.L = h->L;
  return v;
}

}  // namespace

int ep_create(const FnEpConfig *cfg, void **out, std::string &err) {
  if (cfg == nullptr || out == nullptr) { err = "config and handle pointers are required"; return FNMOE_ERR_NULL; }
  if (cfg->abi_version != FNMOE_ABI_VERSION) { err = "abi_version mismatch"; return FNMOE_ERR_ABI; }
  if (cfg->world < 1 || cfg->world > kEpMaxWorld || cfg->rank >= cfg->world) {
    err = "world must be in 1..8 and rank below it";
    return FNMOE_ERR_VALUE;
  }
  if (cfg->capacity_tokens == 0 || cfg->hidden_size == 0 || cfg->hidden_size % 8 || cfg->hidden_size > 4096) {
    err = "capacity_tokens must be positive and hidden_size a multiple of 8 up to 4096";
    return FNMOE_ERR_SHAPE;
  }
  if (cfg->top_k == 0 || cfg->top_k > kEpMaxSlots || cfg->experts_per_rank == 0) {
    err = "top_k must be in 1..16 and experts_per_rank positive";
    return FNMOE_ERR_VALUE;
  }
  EpHandle *h = new EpHandle{};
  cudaGetDevice(&h->device);
  h->world = static_cast<int>(cfg->world);
  h->rank = static_cast<int>(cfg->rank);
  h->cap = static_cast<int>(cfg->capacity_tokens);
  h->H = static_cast<int>(cfg->hidden_size);
  h->k = static_cast<int>(cfg->top_k);
  h->per = static_cast<int>(cfg->experts_per_rank);
  h->L = ep_layout(h->world, h->cap, h->H, h->k);
  cudaError_t e = cudaMalloc(&h->window, h->L.total);
  if (e == cudaSuccess) e = cudaMemset(h->window, 0, h->L.total);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h->ipc, h->window);
  if (e != cudaSuccess) {
    err = std::string("exchange window: ") + cudaGetErrorString(e);
    if (h->window) cudaFree(h->window);
    delete h;
    return FNMOE_ERR_LAUNCH;
  }
  for (int i = 0; i < kEpMaxWorld; ++i) h->peers[i] = nullptr;
  h->peers[h->rank] = h->window;
  *out = h;
  return FNMOE_OK;
}

int ep_ipc_handle(void *handle, void *out64, std::string &err) {
  if (handle == nullptr || out64 == nullptr) { err = "handle and output are required"; return FNMOE_ERR_NULL; }
  static_assert(sizeof(cudaIpcMemHandle_t) == FNMOE_EP_IPC_BYTES, "IPC handle size");
  std::memcpy(out64, &static_cast<EpHandle *>(handle)->ipc, sizeof(cudaIpcMemHandle_t));
  return FNMOE_OK;
}

int ep_open_peers(void *handle, const void *handles, std::string &err) {
  if (handle == nullptr || handles == nullptr) { err = "handle and peer handles are required"; return FNMOE_ERR_NULL; }
  EpHandle *h = static_cast<EpHandle *>(handle);
  if (h->opened) { err = "peers already opened"; return FNMOE_ERR_VALUE; }
  const uint8_t *hs = static_cast<const uint8_t *>(handles);
  for (int r = 0; r < h->world; ++r) {
    if (r == h->rank) continue;
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, hs + static_cast<size_t>(r) * FNMOE_EP_IPC_BYTES, sizeof(ipc));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      err = "open peer " + std::to_string(r) + " window: " + cudaGetErrorString(e);
      for (int q = 0; q < r; ++q)
        if (q != h->rank && h->peers[q]) { cudaIpcCloseMemHandle(h->peers[q]); h->peers[q] = nullptr; }
      return FNMOE_ERR_LAUNCH;
    }
    h->peers[r] = static_cast<uint8_t *>(p);
  }
  h->opened = true;
  return FNMOE_OK;
}

int ep_destroy(void *handle, std::string &err) {
  if (handle == nullptr) { err = "handle is NULL"; return FNMOE_ERR_NULL; }
  EpHandle *h = static_cast<EpHandle *>(handle);
  cudaDeviceSynchronize();
  for (int r = 0; r < h->world; ++r)
    if (r != h->rank && h->peers[r]) cudaIpcCloseMemHandle(h->peers[r]);
  cudaFree(h->window);
  delete h;
  return FNMOE_OK;
}

int ep_window(void *handle, FnEpWindow *w, std::string &err) {
  if (handle == nullptr || w == nullptr) { err = "handle and window are required"; return FNMOE_ERR_NULL; }
  const EpHandle *h = static_cast<const EpHandle *>(handle);
  w->rows = h->window + h->L.rows;
  w->ids = reinterpret_cast<const uint32_t *>(h->window + h->L.ids);
  w->slot_outputs = h->window + h->L.dlocal;
  w->row_count = static_cast<uint32_t>(h->world * h->cap);
  w->slots = static_cast<uint32_t>(h->k + 1);
  w->bytes = h->L.total;
  return FNMOE_OK;
}

static int ep_ready(const EpHandle *h, std::string &err) {
  if (!h->opened && h->world > 1) { err = "peer windows are not open (fnmoe_ep_open_peers)"; return FNMOE_ERR_VALUE; }
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != h->device) { err = "the exchange belongs to another device"; return FNMOE_ERR_DEVICE; }
  return FNMOE_OK;
}

int ep_dispatch(void *handle, const void *x, const uint32_t *inds, uint32_t tokens, cudaStream_t s, std::string &err) {
  if (handle == nullptr || x == nullptr || inds == nullptr) { err = "handle, x and inds are required"; return FNMOE_ERR_NULL; }
  const EpHandle *h = static_cast<const EpHandle *>(handle);
  if (int rc = ep_ready(h, err)) return rc;
  if (tokens > static_cast<uint32_t>(h->cap)) {
    err = std::to_string(tokens) + " tokens exceed the exchange capacity of " + std::to_string(h->cap);
    return FNMOE_ERR_SHAPE;
  }
  const EpView v = view_of(h);
  const int ctas = std::min(h->cap, 16);
  k_ep_dispatch<<<dim3(h->world, ctas), kEpThreads, 0, s>>>(v, static_cast<const uint16_t *>(x), inds,
                                                             static_cast<int>(tokens), device_error_word());
  k_ep_wait<<<1, 32, 0, s>>>(v, h->L.dflag, device_error_word());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { err = std::string("ep dispatch: ") + cudaGetErrorString(e); return FNMOE_ERR_LAUNCH; }
  return FNMOE_OK;
}

int ep_return_combine(void *handle, const void *scores, const void *shared_gate, uint32_t tokens, void *out,
                      cudaStream_t s, std::string &err) {
  if (handle == nullptr || scores == nullptr || shared_gate == nullptr || out == nullptr) {
    err = "handle, scores, shared_gate and out are required";
    return FNMOE_ERR_NULL;
  }
  const EpHandle *h = static_cast<const EpHandle *>(handle);
  if (int rc = ep_ready(h, err)) return rc;
  if (tokens > static_cast<uint32_t>(h->cap)) { err = "tokens exceed the exchange capacity"; return FNMOE_ERR_SHAPE; }
  const EpView v = view_of(h);
  const int ctas = std::min(h->cap, 16);
  k_ep_return<<<dim3(h->world, ctas), kEpThreads, 0, s>>>(v, device_error_word());
  const int threads = ((h->H / 8 + 31) / 32) * 32;
  if (tokens > 0)
    k_ep_combine<<<tokens, threads, 0, s>>>(v, static_cast<const uint16_t *>(scores),
                                           static_cast<const uint16_t *>(shared_gate), static_cast<int>(tokens),
                                           static_cast<uint16_t *>(out), device_error_word());
  else
    k_ep_wait<<<1, 32, 0, s>>>(v, h->L.rflag, device_error_word());
  k_ep_advance<<<1, 1, 0, s>>>(v);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { err = std::string("ep return: ") + cudaGetErrorString(e); return FNMOE_ERR_LAUNCH; }
  return FNMOE_OK;
}

}  // namespace fnmoe
