// api.cu -- extern "C" entry points of libfnmoe (declared in include/fnmoe.h).
//
// Host-side responsibilities: argument validation (mirroring the checks of
// MetalMoEExecutor.execute, metal_runtime.py:803-859), workspace carving and
// kernel sequencing on the caller's stream.  No entry point allocates device
// memory; none synchronises except fnmoe_available (first use per device) and
// fnmoe_read_device_errors.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/fnmoe.h"
#include "attention.cuh"
#include "rows.cuh"
#include "common.cuh"
#include "moe_kernels.cuh"

using namespace fnmoe;

namespace {

thread_local std::string g_last_error;

// ---- optional per-kernel event timing (fnmoe_profile_*) ----
struct ProfRecord {
  const char *name;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mutex;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof;

struct Prof {
  ProfRecord rec{};
  cudaStream_t s;
  bool on;
  Prof(const char *name, cudaStream_t stream) : s(stream) {
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    on = g_prof_on;
    if (!on) return;
    rec.name = name;
    cudaEventCreate(&rec.start);
    cudaEventCreate(&rec.stop);
    cudaEventRecord(rec.start, s);
  }
  ~Prof() {
    if (!on) return;
    cudaEventRecord(rec.stop, s);
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    g_prof.push_back(rec);
  }
};

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char *where) {
  return fail(FNMOE_ERR_LAUNCH, std::string(where) + ": " + cudaGetErrorString(e));
}

// Bump allocator over the caller's workspace (or a size probe when base is
// null).  The base is first rounded up to a 256-byte boundary (`shift`
// bytes of the workspace are skipped), so every carve is 256-byte aligned
// whatever pointer the caller passes; the *_workspace_size calls add 256
// bytes of slack for that shift.
constexpr uint64_t kWorkspaceSlack = 256;

struct Carver {
  uint8_t *base;
  uint64_t shift = 0;
  uint64_t off = 0;
  explicit Carver(void *b) : base(static_cast<uint8_t *>(b)) {
    if (base != nullptr) {
      const uintptr_t p = reinterpret_cast<uintptr_t>(base);
      shift = ((p + 255) & ~uintptr_t(255)) - p;
      base += shift;
    }
  }
  template <typename T>
  T *take(uint64_t count) {
    off = (off + 255) & ~uint64_t(255);
    T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
  // workspace bytes the carves so far use, the alignment shift included
  uint64_t used() const { return shift + off; }
};

// The many-token router's scratch (byte planes of the fixed points, row
// exponents, split-K partial sums and tile tickets) carved from `cv`; false
// when T tokens x R rows take the GEMV path, which needs none.
bool carve_router(Carver &cv, int T, int R, int H, RouterScratch &rs) {
  if (router_scratch_bytes(T, R, H) == 0) return false;
  const uint64_t TH = static_cast<uint64_t>(T) * H;
  rs.xq = cv.take<uint8_t>(3 * TH);
  rs.wq = cv.take<uint8_t>(2ull * R * H);
  rs.ex = cv.take<int32_t>(T);
  rs.ew = cv.take<int32_t>(R);
  rs.ksplit = router_ksplit(T, R, H);
  rs.acc = nullptr;
  rs.tickets = nullptr;
  if (rs.ksplit > 1) {
    rs.acc = cv.take<unsigned long long>(static_cast<uint64_t>(T) * R);
    rs.tickets = cv.take<int32_t>(static_cast<uint64_t>(router_tiles(T, R)));
  }
  return true;
}

bool device_ok(std::string &why) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    why = "no CUDA device";
    return false;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) {
    why = "device is not sm_100 (compute capability " + std::to_string(major) + ".x)";
    return false;
  }
  return true;
}

struct Layout {
  // activations
  uint16_t *xl;
  float *xm;
  // grouping
  GroupView gv;
  // intermediates
  uint16_t *act;
  uint16_t *al;
  float *am;
  uint16_t *d;
};

// Carve the shared part of the executor / layer workspace.
// elem: bytes per activation element (2: bfloat16, 4: float32 activations).
void carve_core(Carver &cv, Layout &L, int T, int H, int I, int G, int n_total, int n_bins,
                bool need_d, int elem = 2) {
  const int Gh = H / G, Gi = I / G;
  L.xl = cv.take<uint16_t>(static_cast<uint64_t>(T) * Gh * 2 * G);
  L.xm = cv.take<float>(static_cast<uint64_t>(T) * meta_pitch(Gh));
  L.gv.n_bins = n_bins;
  L.gv.max_tiles = n_total / kTokPerItem + (n_bins < n_total ? n_bins : n_total) + 1;
  L.gv.counts = cv.take<int32_t>(n_bins);
  L.gv.offsets = cv.take<int32_t>(static_cast<uint64_t>(n_bins) + 1);
  L.gv.order = cv.take<int32_t>(n_total);
  L.gv.tiles = cv.take<int4>(3 * static_cast<uint64_t>(L.gv.max_tiles));
  L.gv.n_tiles = cv.take<int32_t>(4);
  L.gv.bin_key = cv.take<uint32_t>(n_bins);
  L.act = cv.take<uint16_t>(static_cast<uint64_t>(n_total) * I * (elem / 2));
  L.al = cv.take<uint16_t>(static_cast<uint64_t>(n_total) * Gi * 2 * G);
  L.am = cv.take<float>(static_cast<uint64_t>(n_total) * meta_pitch(Gi));
  L.d = need_d ? cv.take<uint16_t>(static_cast<uint64_t>(n_total) * H * (elem / 2)) : nullptr;
}

constexpr int kMaxBins = 16384;

// Range of route values without bit 31: stream-pack records or array experts.
uint32_t non_slot_keys(const FnMoEArgs *a) {
  if (a->stream_table.base != nullptr) return a->stream_table.records;
  return (a->gate_weight != nullptr || a->tiled.gate_up != nullptr) ? a->expert_count : 0u;
}
constexpr uint32_t kMaxTopK = 16;

int validate_moe(const FnMoEArgs *a) {
  if (a == nullptr) return fail(FNMOE_ERR_NULL, "args is NULL");
  if (a->abi_version != FNMOE_ABI_VERSION)
    return fail(FNMOE_ERR_ABI, "abi_version mismatch: library " + std::to_string(FNMOE_ABI_VERSION) +
                                   ", caller " + std::to_string(a->abi_version));
  if (a->tokens == 0 || a->slots == 0 || a->hidden_size == 0 || a->inter_size == 0)
    return fail(FNMOE_ERR_SHAPE, "tokens, slots, hidden_size and inter_size must be positive");
  if (a->group_size != 32 && a->group_size != 64)
    return fail(FNMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (a->hidden_size % a->group_size || a->inter_size % a->group_size)
    return fail(FNMOE_ERR_SHAPE, "Q4 projection inputs must be group aligned");
  if (a->x_dtype != FNMOE_DTYPE_BF16 && a->x_dtype != FNMOE_DTYPE_F32)
    return fail(FNMOE_ERR_UNSUPPORTED, "x must be bfloat16 or float32");
  if (a->x_dtype == FNMOE_DTYPE_F32 && a->hidden_size > 4096)
    return fail(FNMOE_ERR_SHAPE, "float32 activations need hidden_size <= 4096");
  if (a->x == nullptr || a->routes == nullptr) return fail(FNMOE_ERR_NULL, "x and routes are required");
  const bool has_table = a->table.base != nullptr;
  const bool has_stream = a->stream_table.base != nullptr;
  if (has_stream && !has_table) return fail(FNMOE_ERR_VALUE, "stream pack requires a resident slab pack");
  const bool has_tiled = a->tiled.gate_up != nullptr;
  if (has_tiled) {
    if (has_table) return fail(FNMOE_ERR_VALUE, "provide a slab pack or tiled tables, not both");
    if (a->tiled.down == nullptr) return fail(FNMOE_ERR_NULL, "tiled tables need both gate_up and down");
    if (a->inter_size % 8 || a->hidden_size % 16)
      return fail(FNMOE_ERR_SHAPE, "tiled tables need inter_size % 8 == 0 and hidden_size % 16 == 0");
    if (a->tiled.gate_up_record_bytes != tiled_record_bytes(a->inter_size, a->hidden_size, true) ||
        a->tiled.down_record_bytes != tiled_record_bytes(a->hidden_size, a->inter_size, false))
      return fail(FNMOE_ERR_SHAPE, "tiled record sizes do not match hidden/inter sizes");
    if (a->tiled.has_shared) return fail(FNMOE_ERR_VALUE, "executor tiled tables hold routed experts only");
    if (a->tiled.records != a->expert_count) return fail(FNMOE_ERR_SHAPE, "tiled records must equal expert_count");
  } else if (!has_table && (a->gate_weight == nullptr || a->up_weight == nullptr || a->down_weight == nullptr)) {
    return fail(FNMOE_ERR_NULL, "packed execution needs gate, up, and down projections");
  }
  if (!has_tiled && a->gate_weight && (!a->gate_scales || !a->gate_biases || !a->up_scales || !a->up_biases ||
                         !a->down_scales || !a->down_biases))
    return fail(FNMOE_ERR_NULL, "Q4 projections need scales and biases");
  if ((a->shared == nullptr) != (a->shared_gate == nullptr))
    return fail(FNMOE_ERR_VALUE, "shared and shared_gate must be provided together");
  if (a->shared_y != nullptr && a->shared != nullptr)
    return fail(FNMOE_ERR_VALUE, "provide shared_y or shared parts, not both");
  const bool ret_all = a->flags & FNMOE_FLAG_RETURN_ALL;
  const bool per_slot = ret_all || (a->flags & FNMOE_FLAG_NO_COMBINE) || a->scores == nullptr;
  if (ret_all && (!a->gate_out || !a->up_out || !a->down_out))
    return fail(FNMOE_ERR_NULL, "return_all needs gate_out, up_out and down_out");
  if (per_slot && !a->down_out) return fail(FNMOE_ERR_NULL, "per-slot execution needs down_out");
  if (!per_slot && !a->output) return fail(FNMOE_ERR_NULL, "output is NULL");
  if (!per_slot && a->scores_dtype != FNMOE_DTYPE_F32 && a->scores_dtype != FNMOE_DTYPE_BF16)
    return fail(FNMOE_ERR_UNSUPPORTED, "scores must be float32 or bfloat16");
  const uint64_t bins = static_cast<uint64_t>(non_slot_keys(a)) + (has_table ? a->table.records : 0);
  if (bins == 0 || bins > kMaxBins)
    return fail(FNMOE_ERR_SHAPE, "expert_count + table records must be in 1.." + std::to_string(kMaxBins));
  if (static_cast<uint64_t>(a->tokens) * a->slots > (1u << 24))
    return fail(FNMOE_ERR_SHAPE, "too many (token, slot) pairs");
  return FNMOE_OK;
}

// Bytes of the executor's carves from a 256-byte aligned base (no slack).
uint64_t moe_workspace_aligned(const FnMoEArgs *a) {
  Carver cv(nullptr);
  Layout L{};
  const bool has_table = a->table.base != nullptr;
  const int n_bins = static_cast<int>(non_slot_keys(a) + (has_table ? a->table.records : 0));
  const int n_total = static_cast<int>(a->tokens * a->slots);
  const bool per_slot = (a->flags & (FNMOE_FLAG_RETURN_ALL | FNMOE_FLAG_NO_COMBINE)) || a->scores == nullptr;
  carve_core(cv, L, a->tokens, a->hidden_size, a->inter_size, a->group_size, n_total, n_bins, !per_slot,
             a->x_dtype == FNMOE_DTYPE_F32 ? 4 : 2);
  return cv.off;
}

// Workspace bytes for any base pointer (aligned carves plus the slack).
uint64_t moe_workspace(const FnMoEArgs *a) { return moe_workspace_aligned(a) + kWorkspaceSlack; }

bool aligned(const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; }

// The expert kernels copy packed rows in 16-byte pieces and scale/bias rows
// in 4-byte pieces.  Rows of K/8 words are 16-byte multiples (K is a multiple
// of 32), so only the bases (and table offsets/strides) need checking; scale
// and bias rows additionally need an even group count for 4-byte copies,
// which the kernels check per projection.
int check_expert_alignment(ExpertCallArgs &c) {
  bool w_ok = true, sb_ok = true, sb16 = true;
  auto arr = [&](const ProjArrays &pa) {
    if (pa.w == nullptr) return;
    w_ok = w_ok && aligned(pa.w, 16);
    sb_ok = sb_ok && aligned(pa.s, 4) && aligned(pa.b, 4);
    sb16 = sb16 && aligned(pa.s, 16) && aligned(pa.b, 16);
  };
  arr(c.gate);
  arr(c.up);
  arr(c.down);
  arr(c.sh_gate);
  arr(c.sh_up);
  arr(c.sh_down);
  for (const TableView *t : {&c.table, &c.stream}) {
    if (t->base == nullptr) continue;
    const uintptr_t b = reinterpret_cast<uintptr_t>(t->base) + t->header;
    w_ok = w_ok && (t->stride % 16) == 0;
    sb_ok = sb_ok && (t->stride % 4) == 0;
    sb16 = sb16 && (t->stride % 16) == 0;
    for (int part = 0; part < 3; ++part) {
      w_ok = w_ok && ((b + t->off[3 * part]) % 16) == 0;
      sb_ok = sb_ok && ((b + t->off[3 * part + 1]) % 4) == 0 && ((b + t->off[3 * part + 2]) % 4) == 0;
      sb16 = sb16 && ((b + t->off[3 * part + 1]) % 16) == 0 && ((b + t->off[3 * part + 2]) % 16) == 0;
    }
  }
  if (c.tiled.gate_up != nullptr) w_ok = w_ok && aligned(c.tiled.gate_up, 16) && aligned(c.tiled.down, 16);
  if (!w_ok) return fail(FNMOE_ERR_VALUE, "packed expert weights must start on 16-byte boundaries");
  c.sb_async = sb_ok ? 1 : 0;
  c.sb_bulk = (sb_ok && sb16) ? 1 : 0;
  return FNMOE_OK;
}

ExpertCallArgs make_call(const FnMoEArgs *a) {
  ExpertCallArgs c{};
  c.gate = {a->gate_weight, static_cast<const uint16_t *>(a->gate_scales), static_cast<const uint16_t *>(a->gate_biases)};
  c.up = {a->up_weight, static_cast<const uint16_t *>(a->up_scales), static_cast<const uint16_t *>(a->up_biases)};
  c.down = {a->down_weight, static_cast<const uint16_t *>(a->down_scales), static_cast<const uint16_t *>(a->down_biases)};
  c.sh_gate = c.sh_up = c.sh_down = {nullptr, nullptr, nullptr};
  c.table.base = static_cast<const uint8_t *>(a->table.base);
  c.table.header = a->table.header_bytes;
  c.table.stride = a->table.record_stride;
  for (int i = 0; i < 9; ++i) c.table.off[i] = a->table.part_offset[i];
  c.table.records = a->table.base ? a->table.records : 0;
  c.stream.base = static_cast<const uint8_t *>(a->stream_table.base);
  c.stream.header = a->stream_table.header_bytes;
  c.stream.stride = a->stream_table.record_stride;
  for (int i = 0; i < 9; ++i) c.stream.off[i] = a->stream_table.part_offset[i];
  c.stream.records = a->stream_table.base ? a->stream_table.records : 0;
  c.array_experts = a->stream_table.base ? static_cast<int>(a->stream_table.records)
                    : ((a->gate_weight || a->tiled.gate_up) ? static_cast<int>(a->expert_count) : 0);
  if (a->tiled.gate_up != nullptr) {
    c.gate = c.up = c.down = {nullptr, nullptr, nullptr};
    c.tiled.gate_up = static_cast<const uint8_t *>(a->tiled.gate_up);
    c.tiled.down = static_cast<const uint8_t *>(a->tiled.down);
    c.tiled.gate_up_record = a->tiled.gate_up_record_bytes;
    c.tiled.down_record = a->tiled.down_record_bytes;
    c.tiled.records = a->tiled.records;
    c.tiled.has_shared = 0;
  }
  c.tokens = static_cast<int>(a->tokens);
  c.slots = static_cast<int>(a->slots);
  c.n_pairs = c.tokens * c.slots;
  c.H = static_cast<int>(a->hidden_size);
  c.I = static_cast<int>(a->inter_size);
  c.I_shared = c.I;
  c.G = static_cast<int>(a->group_size);
  c.f32 = a->x_dtype == FNMOE_DTYPE_F32 ? 1 : 0;
  return c;
}

}  // namespace

// Library-owned scratch of fnmoe_moe_execute_static: file-scope device
// storage, no runtime allocation.
static __device__ __align__(256) uint8_t g_static_scratch[FNMOE_STATIC_SCRATCH_BYTES];

namespace {

// Device address of g_static_scratch on the current device.  In host code
// the symbol's name is only a host-side stand-in, so the address is looked
// up with the device current, on every call: the lookup allocates nothing
// and does not synchronise, and a per-device cache would outlive a
// cudaDeviceReset (or primary-context teardown) and hand out a stale
// address afterwards.  The first lookup on a device may load the library's
// device code, which is why the first call belongs before any stream capture.
int static_scratch(void **ptr) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "static scratch: cudaGetSymbolAddress");
  *ptr = p;
  return FNMOE_OK;
}

}  // namespace

extern "C" {

int fnmoe_available(void) {
  std::string why;
  if (!device_ok(why)) {
    g_last_error = why;
    return 0;
  }
  cudaError_t e = ensure_exp_table(0);
  if (e != cudaSuccess) {
    g_last_error = std::string("initialisation failed: ") + cudaGetErrorString(e);
    return 0;
  }
  return 1;
}

int fnmoe_get_last_error(char *buf, uint32_t max_len) {
  if (buf == nullptr || max_len == 0) return FNMOE_ERR_NULL;
  std::strncpy(buf, g_last_error.c_str(), max_len - 1);
  buf[max_len - 1] = '\0';
  return FNMOE_OK;
}

uint32_t fnmoe_abi_version(void) { return FNMOE_ABI_VERSION; }

int fnmoe_moe_workspace_size(const FnMoEArgs *args, uint64_t *bytes) {
  if (bytes == nullptr) return fail(FNMOE_ERR_NULL, "bytes is NULL");
  const int v = validate_moe(args);
  if (v != FNMOE_OK) return v;
  *bytes = moe_workspace(args);
  return FNMOE_OK;
}

int fnmoe_moe_execute(const FnMoEArgs *a, void *stream) {
  const int v = validate_moe(a);
  if (v != FNMOE_OK) return v;
  std::string why;
  if (!device_ok(why)) return fail(FNMOE_ERR_DEVICE, why);
  if (a->workspace == nullptr)
    return fail(FNMOE_ERR_WORKSPACE, "workspace needs " + std::to_string(moe_workspace(a)) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");

  const bool has_table = a->table.base != nullptr;
  const bool ret_all = a->flags & FNMOE_FLAG_RETURN_ALL;
  const bool per_slot = ret_all || (a->flags & FNMOE_FLAG_NO_COMBINE) || a->scores == nullptr;
  const int T = static_cast<int>(a->tokens), S = static_cast<int>(a->slots);
  const int H = static_cast<int>(a->hidden_size), I = static_cast<int>(a->inter_size);
  const int G = static_cast<int>(a->group_size);
  const int n_pairs = T * S;
  const int n_bins = static_cast<int>(non_slot_keys(a) + (has_table ? a->table.records : 0));
  const bool f32 = a->x_dtype == FNMOE_DTYPE_F32;
  Carver cv(a->workspace);
  Layout L{};
  carve_core(cv, L, T, H, I, G, n_pairs, n_bins, !per_slot, f32 ? 4 : 2);
  if (cv.used() > a->workspace_bytes)
    return fail(FNMOE_ERR_WORKSPACE, "workspace needs " + std::to_string(moe_workspace(a)) + " bytes");
  uint16_t *d = per_slot ? static_cast<uint16_t *>(a->down_out) : L.d;
  ExpertCallArgs call = make_call(a);
  if (int rc = check_expert_alignment(call)) return rc;

  {
    Prof p("prep_x", s);
    e = f32 ? launch_prep_rows_f32(static_cast<const float *>(a->x), T, H, G, L.xl, L.xm, s)
            : launch_prep_rows(static_cast<const uint16_t *>(a->x), T, H, G, L.xl, L.xm, s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "prep x");
  {
    Prof p("group", s);
    e = launch_group(a->routes, n_pairs, 0, call.array_experts, static_cast<int>(call.table.records), L.gv, s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "group");
  {
    Prof p("gate_up", s);
    e = launch_gate_up(call, L.gv, L.xl, L.xm, L.act,
                       ret_all ? static_cast<uint16_t *>(a->gate_out) : nullptr,
                       ret_all ? static_cast<uint16_t *>(a->up_out) : nullptr, s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gate_up");
  {
    Prof p("prep_act", s);
    // empty slots (FNMOE_ROUTE_NONE) have no activation row: skipped
    e = f32 ? launch_prep_rows_f32(reinterpret_cast<const float *>(L.act), n_pairs, I, G, L.al, L.am, s, a->routes,
                                   n_pairs)
            : launch_prep_rows(L.act, n_pairs, I, G, L.al, L.am, s, a->routes, n_pairs);
  }
  if (e != cudaSuccess) return cuda_fail(e, "prep act");
  {
    Prof p("down", s);
    e = launch_down(call, L.gv, L.al, L.am, d, s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "down");
  if (per_slot) return FNMOE_OK;
  int mode = kCombineNone;
  if (a->shared_y) mode = kCombineSharedY;
  else if (a->shared) mode = kCombineParts;
  {
    Prof p("combine", s);
    if (f32)
      e = launch_combine_f32(reinterpret_cast<const float *>(d), a->routes, a->scores,
                             a->scores_dtype == FNMOE_DTYPE_F32, T, S, H, mode,
                             static_cast<const float *>(a->shared_y), static_cast<const float *>(a->shared),
                             static_cast<const float *>(a->shared_gate), call.array_experts,
                             static_cast<int>(call.table.records), static_cast<float *>(a->output), s);
    else
      e = launch_combine(d, a->routes, a->scores, a->scores_dtype == FNMOE_DTYPE_F32, T, S, H, mode,
                         static_cast<const uint16_t *>(a->shared_y), static_cast<const uint16_t *>(a->shared),
                         static_cast<const uint16_t *>(a->shared_gate), call.array_experts,
                         static_cast<int>(call.table.records), static_cast<uint16_t *>(a->output), s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "combine");
  return FNMOE_OK;
}

int fnmoe_moe_execute_static(const FnMoEArgs *a, void *stream) {
  const int v = validate_moe(a);
  if (v != FNMOE_OK) return v;
  // the array is 256-byte aligned: the carves need no slack
  const uint64_t need = moe_workspace_aligned(a);
  if (need > FNMOE_STATIC_SCRATCH_BYTES)
    return fail(FNMOE_ERR_WORKSPACE, "this call needs " + std::to_string(need) +
                                         " bytes of scratch; the static scratch holds " +
                                         std::to_string(FNMOE_STATIC_SCRATCH_BYTES) +
                                         " (use fnmoe_moe_execute with a workspace)");
  std::string why;
  if (!device_ok(why)) return fail(FNMOE_ERR_DEVICE, why);
  void *scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  FnMoEArgs local = *a;
  local.workspace = scratch;
  local.workspace_bytes = FNMOE_STATIC_SCRATCH_BYTES;
  return fnmoe_moe_execute(&local, stream);
}

int fnmoe_weighted_combine(const float *outputs, const int32_t *routes, const float *scores,
                           float *out, uint32_t tokens, uint32_t slots, uint32_t experts,
                           uint32_t hidden, void *stream) {
  if (!outputs || !scores || !out || (experts > 0 && !routes))
    return fail(FNMOE_ERR_NULL, "outputs, scores, out (and routes when experts > 0) are required");
  if (tokens == 0 || slots == 0 || hidden == 0) return fail(FNMOE_ERR_SHAPE, "empty combine");
  cudaError_t e = launch_weighted_combine(outputs, routes, scores, out, tokens, slots, experts,
                                          hidden, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "weighted_combine");
}

int fnmoe_router_topk(const void *x, const void *router_weight, uint32_t tokens, uint32_t hidden,
                      uint32_t experts, uint32_t top_k, float renorm_blend, uint32_t *inds,
                      void *scores, void *mass, void *logits, void *stream) {
  if (!x || !router_weight || !inds || !scores || !logits)
    return fail(FNMOE_ERR_NULL, "x, router_weight, inds, scores and logits are required");
  if (tokens == 0 || hidden == 0 || hidden % 8) return fail(FNMOE_ERR_SHAPE, "hidden must be a positive multiple of 8");
  if (hidden > 4096) return fail(FNMOE_ERR_SHAPE, "hidden must be <= 4096");
  if (experts == 0 || experts > 1024) return fail(FNMOE_ERR_SHAPE, "experts must be in 1..1024");
  if (top_k == 0 || top_k > kMaxTopK || top_k > experts) return fail(FNMOE_ERR_VALUE, "top_k out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");
  e = launch_router_logits(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(router_weight),
                           tokens, hidden, experts, nullptr, static_cast<uint16_t *>(logits), nullptr, s);
  if (e != cudaSuccess) return cuda_fail(e, "router logits");
  // `inds` doubles as the route output (identity mapping).
  e = launch_softmax_topk(static_cast<const uint16_t *>(logits), tokens, experts, top_k, renorm_blend,
                          nullptr, 0, inds, inds, nullptr, static_cast<uint16_t *>(scores),
                          static_cast<uint16_t *>(mass), nullptr, nullptr, s);
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "softmax_topk");
}

int fnmoe_router_topk_shared(const void *x, const void *router_weight, const void *shared_gate_weight,
                             uint32_t tokens, uint32_t hidden, uint32_t experts, uint32_t top_k,
                             float renorm_blend, uint32_t *inds, void *scores, void *mass, void *logits,
                             void *shared_logit, void *shared_gate, void *stream) {
  if (!x || !router_weight || !shared_gate_weight || !inds || !scores || !logits || !shared_logit || !shared_gate)
    return fail(FNMOE_ERR_NULL,
                "x, router_weight, shared_gate_weight, inds, scores, logits, shared_logit and shared_gate are required");
  if (tokens == 0 || hidden == 0 || hidden % 8) return fail(FNMOE_ERR_SHAPE, "hidden must be a positive multiple of 8");
  if (hidden > 4096) return fail(FNMOE_ERR_SHAPE, "hidden must be <= 4096");
  if (experts == 0 || experts > 1024) return fail(FNMOE_ERR_SHAPE, "experts must be in 1..1024");
  if (top_k == 0 || top_k > kMaxTopK || top_k > experts) return fail(FNMOE_ERR_VALUE, "top_k out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");
  e = launch_router_logits(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(router_weight), tokens,
                           hidden, experts, static_cast<const uint16_t *>(shared_gate_weight),
                           static_cast<uint16_t *>(logits), static_cast<uint16_t *>(shared_logit), s);
  if (e != cudaSuccess) return cuda_fail(e, "router logits");
  e = launch_softmax_topk(static_cast<const uint16_t *>(logits), tokens, experts, top_k, renorm_blend, nullptr, 0,
                          inds, inds, nullptr, static_cast<uint16_t *>(scores), static_cast<uint16_t *>(mass),
                          static_cast<const uint16_t *>(shared_logit), static_cast<uint16_t *>(shared_gate), s);
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "softmax_topk");
}

int fnmoe_router_workspace_size(uint32_t tokens, uint32_t hidden, uint32_t experts, uint32_t with_shared_gate,
                                uint64_t *bytes) {
  if (!bytes) return fail(FNMOE_ERR_NULL, "bytes is required");
  if (tokens == 0 || hidden == 0 || hidden % 8 || hidden > 4096)
    return fail(FNMOE_ERR_SHAPE, "tokens must be positive, hidden a multiple of 8 up to 4096");
  if (experts == 0 || experts > 1024) return fail(FNMOE_ERR_SHAPE, "experts must be in 1..1024");
  Carver cv(nullptr);
  RouterScratch rs{};
  const bool need = carve_router(cv, static_cast<int>(tokens), static_cast<int>(experts + (with_shared_gate ? 1 : 0)),
                                 static_cast<int>(hidden), rs);
  *bytes = need ? cv.off + kWorkspaceSlack : 0;
  return FNMOE_OK;
}

int fnmoe_router_topk_shared_ws(const void *x, const void *router_weight, const void *shared_gate_weight,
                                uint32_t tokens, uint32_t hidden, uint32_t experts, uint32_t top_k,
                                float renorm_blend, uint32_t *inds, void *scores, void *mass, void *logits,
                                void *shared_logit, void *shared_gate, void *workspace, uint64_t workspace_bytes,
                                void *stream) {
  if (!x || !router_weight || !shared_gate_weight || !inds || !scores || !logits || !shared_logit || !shared_gate)
    return fail(FNMOE_ERR_NULL,
                "x, router_weight, shared_gate_weight, inds, scores, logits, shared_logit and shared_gate are required");
  if (tokens == 0 || hidden == 0 || hidden % 8) return fail(FNMOE_ERR_SHAPE, "hidden must be a positive multiple of 8");
  if (hidden > 4096) return fail(FNMOE_ERR_SHAPE, "hidden must be <= 4096");
  if (experts == 0 || experts > 1024) return fail(FNMOE_ERR_SHAPE, "experts must be in 1..1024");
  if (top_k == 0 || top_k > kMaxTopK || top_k > experts) return fail(FNMOE_ERR_VALUE, "top_k out of range");
  uint64_t need = 0;
  int rc = fnmoe_router_workspace_size(tokens, hidden, experts, 1, &need);
  if (rc != FNMOE_OK) return rc;
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(FNMOE_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
  RouterScratch rs{};
  bool has_rs = false;
  if (need > 0) {
    Carver cv(workspace);
    has_rs = carve_router(cv, static_cast<int>(tokens), static_cast<int>(experts) + 1, static_cast<int>(hidden), rs);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");
  e = launch_router_logits(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(router_weight), tokens,
                           hidden, experts, static_cast<const uint16_t *>(shared_gate_weight),
                           static_cast<uint16_t *>(logits), static_cast<uint16_t *>(shared_logit), s, nullptr,
                           nullptr, 32, nullptr, has_rs ? &rs : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "router logits");
  e = launch_softmax_topk(static_cast<const uint16_t *>(logits), tokens, experts, top_k, renorm_blend, nullptr, 0,
                          inds, inds, nullptr, static_cast<uint16_t *>(scores), static_cast<uint16_t *>(mass),
                          static_cast<const uint16_t *>(shared_logit), static_cast<uint16_t *>(shared_gate), s);
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "softmax_topk");
}

int fnmoe_combine(const void *slot_outputs, const uint32_t *routes, const void *scores, uint32_t scores_dtype,
                  uint32_t tokens, uint32_t slots, uint32_t hidden, uint32_t expert_count, const void *shared_y,
                  const void *shared, const void *shared_gate, void *out, void *stream) {
  if (!slot_outputs || !routes || !scores || !out)
    return fail(FNMOE_ERR_NULL, "slot_outputs, routes, scores and out are required");
  if (tokens == 0 || slots == 0 || hidden == 0) return fail(FNMOE_ERR_SHAPE, "tokens, slots and hidden must be positive");
  if (scores_dtype != FNMOE_DTYPE_F32 && scores_dtype != FNMOE_DTYPE_BF16)
    return fail(FNMOE_ERR_UNSUPPORTED, "scores must be float32 or bfloat16");
  if ((shared == nullptr) != (shared_gate == nullptr))
    return fail(FNMOE_ERR_VALUE, "shared and shared_gate must be provided together");
  if (shared_y != nullptr && shared != nullptr) return fail(FNMOE_ERR_VALUE, "provide shared_y or shared parts, not both");
  const int mode = shared_y ? kCombineSharedY : (shared ? kCombineParts : kCombineNone);
  cudaError_t e = launch_combine(static_cast<const uint16_t *>(slot_outputs), routes, scores,
                                 scores_dtype == FNMOE_DTYPE_F32, static_cast<int>(tokens), static_cast<int>(slots),
                                 static_cast<int>(hidden), mode, static_cast<const uint16_t *>(shared_y),
                                 static_cast<const uint16_t *>(shared), static_cast<const uint16_t *>(shared_gate),
                                 static_cast<int>(expert_count), 0, static_cast<uint16_t *>(out),
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "combine");
}

int fnmoe_softmax_topk(const void *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                       float renorm_blend, uint32_t *inds, void *raw_scores, void *scores, void *mass,
                       void *stream) {
  if (!logits || !inds || (!scores && !raw_scores))
    return fail(FNMOE_ERR_NULL, "logits, inds and raw_scores or scores are required");
  if (tokens == 0) return fail(FNMOE_ERR_SHAPE, "tokens must be positive");
  if (experts == 0 || experts > 1024) return fail(FNMOE_ERR_SHAPE, "experts must be in 1..1024");
  if (top_k == 0 || top_k > kMaxTopK || top_k > experts) return fail(FNMOE_ERR_VALUE, "top_k out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");
  e = launch_softmax_topk(static_cast<const uint16_t *>(logits), tokens, experts, top_k, renorm_blend,
                          nullptr, 0, inds, inds, static_cast<uint16_t *>(raw_scores),
                          static_cast<uint16_t *>(scores), static_cast<uint16_t *>(mass), nullptr,
                          nullptr, s);
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "softmax_topk");
}

int fnmoe_group_tokens(const uint32_t *routes, uint32_t pairs, uint32_t array_experts,
                       uint32_t table_records, int32_t *counts, int32_t *offsets, int32_t *order,
                       void *workspace, uint64_t workspace_bytes, void *stream) {
  if (!routes || !counts || !offsets || !order) return fail(FNMOE_ERR_NULL, "routes, counts, offsets, order required");
  const uint64_t bins = static_cast<uint64_t>(array_experts) + table_records;
  if (pairs == 0 || bins == 0 || bins > kMaxBins) return fail(FNMOE_ERR_SHAPE, "invalid pairs or key count");
  const int n_bins = static_cast<int>(bins);
  GroupView gv{};
  gv.n_bins = n_bins;
  gv.max_tiles = static_cast<int>(pairs) / kTokPerItem + (n_bins < static_cast<int>(pairs) ? n_bins : static_cast<int>(pairs)) + 1;
  Carver cv(workspace);
  gv.tiles = cv.take<int4>(3 * static_cast<uint64_t>(gv.max_tiles));
  gv.n_tiles = cv.take<int32_t>(4);
  gv.bin_key = cv.take<uint32_t>(n_bins);
  if (workspace == nullptr || workspace_bytes < cv.used())
    return fail(FNMOE_ERR_WORKSPACE, "workspace needs " + std::to_string(cv.off + kWorkspaceSlack) + " bytes");
  gv.counts = counts;
  gv.offsets = offsets;
  gv.order = order;
  cudaError_t e = launch_group(routes, static_cast<int>(pairs), 0, static_cast<int>(array_experts),
                               static_cast<int>(table_records), gv, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "group");
}

namespace {

int validate_layer(const FnMoELayerArgs *a) {
  if (a == nullptr) return fail(FNMOE_ERR_NULL, "args is NULL");
  if (a->abi_version != FNMOE_ABI_VERSION) return fail(FNMOE_ERR_ABI, "abi_version mismatch");
  if (!a->x || !a->router_weight || !a->output) return fail(FNMOE_ERR_NULL, "x, router_weight and output are required");
  if (a->tokens == 0 || a->hidden_size == 0 || a->inter_size == 0) return fail(FNMOE_ERR_SHAPE, "empty layer");
  if (a->group_size != 32 && a->group_size != 64) return fail(FNMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (a->hidden_size % a->group_size || a->inter_size % a->group_size)
    return fail(FNMOE_ERR_SHAPE, "Q4 projection inputs must be group aligned");
  if (a->hidden_size > 4096) return fail(FNMOE_ERR_SHAPE, "hidden must be <= 4096");
  if (a->expert_count == 0 || a->expert_count > 1024) return fail(FNMOE_ERR_SHAPE, "expert_count must be in 1..1024");
  if (a->top_k == 0 || a->top_k > kMaxTopK || a->top_k > a->expert_count) return fail(FNMOE_ERR_VALUE, "top_k out of range");
  const bool has_table = a->table.base != nullptr;
  const bool has_tiled = a->tiled.gate_up != nullptr;
  if (has_tiled) {
    if (has_table) return fail(FNMOE_ERR_VALUE, "provide a slab table or tiled tables, not both");
    if (a->tiled.down == nullptr) return fail(FNMOE_ERR_NULL, "tiled tables need both gate_up and down");
    if (a->inter_size % 8 || a->hidden_size % 16)
      return fail(FNMOE_ERR_SHAPE, "tiled tables need inter_size % 8 == 0 and hidden_size % 16 == 0");
    const uint64_t gu = tiled_record_bytes(a->inter_size, a->hidden_size, true);
    const uint64_t dn = tiled_record_bytes(a->hidden_size, a->inter_size, false);
    if (a->tiled.gate_up_record_bytes != gu || a->tiled.down_record_bytes != dn)
      return fail(FNMOE_ERR_SHAPE, "tiled record sizes do not match hidden/inter sizes");
    const bool sh = a->shared_inter_size != 0;
    if ((a->tiled.has_shared != 0) != sh)
      return fail(FNMOE_ERR_VALUE, "tiled tables must hold the shared expert exactly when the layer has one");
    if (a->tiled.records != a->expert_count + (sh ? 1u : 0u))
      return fail(FNMOE_ERR_SHAPE, "tiled records must be expert_count (+1 for the shared expert)");
  } else if (!has_table && (!a->gate_weight || !a->up_weight || !a->down_weight)) {
    return fail(FNMOE_ERR_NULL, "routed experts need gate, up and down projections or a table");
  }
  if (a->shared_inter_size) {
    if (a->shared_inter_size != a->inter_size)
      return fail(FNMOE_ERR_UNSUPPORTED, "shared expert intermediate must equal the routed intermediate");
    if (!a->shared_expert_gate) return fail(FNMOE_ERR_NULL, "shared expert needs its sigmoid gate weight");
    if (!has_tiled && (!a->shared_gate_weight || !a->shared_up_weight || !a->shared_down_weight))
      return fail(FNMOE_ERR_NULL, "shared expert needs gate, up and down projections");
  }
  const uint64_t bins = (has_table ? a->table.records : a->expert_count) + 1ull;
  if (bins > kMaxBins) return fail(FNMOE_ERR_SHAPE, "too many experts/records");
  return FNMOE_OK;
}

// Whether fnmoe_moe_layer runs the tcgen05 prefill GEMMs for these arguments
// (the same test as prefill_supported on the resolved call, plus the flags
// and the pair-count threshold).
bool layer_prefill(const FnMoELayerArgs *a) {
  const bool supported = a->tiled.gate_up != nullptr && a->tiled.down != nullptr && a->group_size == 32 &&
                         a->hidden_size % 256 == 0 && a->inter_size % 256 == 0;
  const uint64_t n_total = static_cast<uint64_t>(a->tokens) * a->top_k + (a->shared_inter_size ? a->tokens : 0);
  return supported && (a->flags & FNMOE_LAYER_FORCE_DECODE) == 0 &&
         ((a->flags & FNMOE_LAYER_FORCE_PREFILL) != 0 || n_total >= FNMOE_PREFILL_PAIRS);
}

struct LayerLayout {
  Layout core;
  uint16_t *logits, *shared_logit, *shared_gate, *scores, *mass;
  uint32_t *inds, *routes;
  int4 *ptiles;        // 128-pair tiles of the prefill path
  int32_t *n_ptiles;
  int max_ptiles;
  uint16_t *xg;        // prefill: x rows gathered into bin order [n_total][H]
  int *ghist;          // prefill: per-chunk bin counts of the multi-CTA grouping
  uint64_t ghist_bytes;
  uint32_t *amax;      // batch-1 persistent kernel: activation row maxima
  RouterScratch rs;    // many-token router: fixed-point byte planes
  bool has_rs = false;
};

// Carves the layer workspace from `base` (null: a size probe).  Returns the
// bytes any base pointer needs (carves plus the alignment slack); `used`
// receives the bytes these carves take from this base.
uint64_t carve_layer(const FnMoELayerArgs *a, void *base, LayerLayout &LL, uint64_t *used = nullptr) {
  Carver cv(base);
  const int T = a->tokens, k = a->top_k, E = a->expert_count;
  const bool has_table = a->table.base != nullptr;
  const bool shared = a->shared_inter_size != 0;
  const int n_pairs = T * k;
  const int n_total = n_pairs + (shared ? T : 0);
  const int array_experts = has_table ? 0 : E;
  const int records = has_table ? static_cast<int>(a->table.records) : 0;
  const int n_bins = array_experts + records + (shared ? 1 : 0);
  LL.logits = cv.take<uint16_t>(static_cast<uint64_t>(T) * E);
  LL.shared_logit = cv.take<uint16_t>(T);
  LL.shared_gate = cv.take<uint16_t>(T);
  LL.scores = cv.take<uint16_t>(static_cast<uint64_t>(T) * k);
  LL.mass = cv.take<uint16_t>(T);
  LL.inds = cv.take<uint32_t>(static_cast<uint64_t>(T) * k);
  LL.routes = cv.take<uint32_t>(static_cast<uint64_t>(T) * k);
  carve_core(cv, LL.core, T, a->hidden_size, a->inter_size, a->group_size, n_total, n_bins, true);
  LL.max_ptiles = prefill_max_tiles(n_total, n_bins);
  LL.ptiles = cv.take<int4>(static_cast<uint64_t>(LL.max_ptiles));
  LL.n_ptiles = cv.take<int32_t>(4);
  LL.xg = layer_prefill(a) ? cv.take<uint16_t>(static_cast<uint64_t>(n_total) * a->hidden_size) : nullptr;
  LL.ghist_bytes = layer_prefill(a) ? static_cast<uint64_t>((n_total + 4095) / 4096) * n_bins * sizeof(int) : 0;
  LL.ghist = LL.ghist_bytes ? cv.take<int>(LL.ghist_bytes / sizeof(int)) : nullptr;
  LL.amax = cv.take<uint32_t>(32);
  {
    // many-token router: byte planes of the fixed points and row exponents
    const int R = E + (shared ? 1 : 0);
    LL.has_rs = carve_router(cv, T, R, static_cast<int>(a->hidden_size), LL.rs);
  }
  if (used != nullptr) *used = cv.used();
  return cv.off + kWorkspaceSlack;
}

}  // namespace

int fnmoe_moe_layer_workspace_size(const FnMoELayerArgs *args, uint64_t *bytes) {
  if (bytes == nullptr) return fail(FNMOE_ERR_NULL, "bytes is NULL");
  const int v = validate_layer(args);
  if (v != FNMOE_OK) return v;
  LayerLayout LL{};
  *bytes = carve_layer(args, nullptr, LL);
  return FNMOE_OK;
}

int fnmoe_moe_layer(const FnMoELayerArgs *a, void *stream) {
  const int v = validate_layer(a);
  if (v != FNMOE_OK) return v;
  std::string why;
  if (!device_ok(why)) return fail(FNMOE_ERR_DEVICE, why);
  LayerLayout LL{};
  const uint64_t need = carve_layer(a, nullptr, LL);
  uint64_t used = 0;
  if (a->workspace != nullptr) carve_layer(a, a->workspace, LL, &used);
  if (a->workspace == nullptr || a->workspace_bytes < used)
    return fail(FNMOE_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");

  const int T = a->tokens, k = a->top_k, E = a->expert_count;
  const int H = a->hidden_size, I = a->inter_size, G = a->group_size;
  const bool has_table = a->table.base != nullptr;
  const bool shared = a->shared_inter_size != 0;
  const int n_pairs = T * k;

  ExpertCallArgs call{};
  call.gate = {a->gate_weight, static_cast<const uint16_t *>(a->gate_scales), static_cast<const uint16_t *>(a->gate_biases)};
  call.up = {a->up_weight, static_cast<const uint16_t *>(a->up_scales), static_cast<const uint16_t *>(a->up_biases)};
  call.down = {a->down_weight, static_cast<const uint16_t *>(a->down_scales), static_cast<const uint16_t *>(a->down_biases)};
  call.sh_gate = {a->shared_gate_weight, static_cast<const uint16_t *>(a->shared_gate_scales), static_cast<const uint16_t *>(a->shared_gate_biases)};
  call.sh_up = {a->shared_up_weight, static_cast<const uint16_t *>(a->shared_up_scales), static_cast<const uint16_t *>(a->shared_up_biases)};
  call.sh_down = {a->shared_down_weight, static_cast<const uint16_t *>(a->shared_down_scales), static_cast<const uint16_t *>(a->shared_down_biases)};
  call.table.base = static_cast<const uint8_t *>(a->table.base);
  call.table.header = a->table.header_bytes;
  call.table.stride = a->table.record_stride;
  for (int i = 0; i < 9; ++i) call.table.off[i] = a->table.part_offset[i];
  call.table.records = has_table ? a->table.records : 0;
  call.array_experts = has_table ? 0 : E;
  call.tokens = T;
  call.slots = k;
  call.n_pairs = n_pairs;
  call.H = H;
  call.I = I;
  call.I_shared = shared ? static_cast<int>(a->shared_inter_size) : I;
  call.G = G;
  if (a->tiled.gate_up != nullptr) {
    call.tiled.gate_up = static_cast<const uint8_t *>(a->tiled.gate_up);
    call.tiled.down = static_cast<const uint8_t *>(a->tiled.down);
    call.tiled.gate_up_record = a->tiled.gate_up_record_bytes;
    call.tiled.down_record = a->tiled.down_record_bytes;
    call.tiled.records = a->tiled.records;
    call.tiled.has_shared = a->tiled.has_shared ? 1 : 0;
    if (!aligned(call.tiled.gate_up, 16) || !aligned(call.tiled.down, 16))
      return fail(FNMOE_ERR_VALUE, "tiled tables must start on 16-byte boundaries");
  }
  if (int rc = check_expert_alignment(call)) return rc;

  const int n_total_pairs = n_pairs + (shared ? T : 0);
  const bool prefill = prefill_supported(call) && layer_prefill(a);
  if ((a->flags & FNMOE_LAYER_FORCE_PREFILL) && !prefill_supported(call))
    return fail(FNMOE_ERR_UNSUPPORTED,
                "the prefill path needs tiled tables, group size 32 and hidden/inter multiples of 256");
  Layout &L = LL.core;
  uint16_t *logits = a->logits_out ? static_cast<uint16_t *>(a->logits_out) : LL.logits;
  uint32_t *inds = a->inds_out ? a->inds_out : LL.inds;
  uint16_t *scores = a->scores_out ? static_cast<uint16_t *>(a->scores_out) : LL.scores;

  // One token on tiled tables: the whole layer in one persistent kernel
  // (same arithmetic, same bits as the launches below).
  if (T == 1 && !prefill && call.tiled.gate_up != nullptr && a->table_routes_of_expert == nullptr &&
      !fused_disabled()) {
    FusedLayer f{};
    f.x = static_cast<const uint16_t *>(a->x);
    f.W = static_cast<const uint16_t *>(a->router_weight);
    f.wsg = shared ? static_cast<const uint16_t *>(a->shared_expert_gate) : nullptr;
    f.tiled = call.tiled;
    f.E = E;
    f.k = k;
    f.H = H;
    f.I = I;
    f.blend = a->renorm_blend;
    f.keep_threshold = a->keep_threshold;
    f.min_keep = static_cast<int>(a->min_keep);
    f.logits = logits;
    f.shared_logit = LL.shared_logit;
    f.inds = inds;
    f.scores = scores;
    f.mass = LL.mass;
    f.shared_gate = LL.shared_gate;
    f.act = L.act;
    e = grid_barrier_slot(a->workspace, &f.bar);
    if (e != cudaSuccess) return cuda_fail(e, "grid barrier slot");
    f.out = static_cast<uint16_t *>(a->output);
    f.amax = LL.amax;
    {
      Prof p("decode_layer", s);
      e = launch_decode_layer(f, G, s);
    }
    if (e == cudaSuccess) return FNMOE_OK;
    if (e != cudaErrorNotSupported) return cuda_fail(e, "decode layer");
  }

  // Small decode batches get the row fixed point of x from extra CTAs of the
  // router launch; otherwise it is a launch of its own.
  bool prep_done = false;
  {
    Prof p("router_logits", s);
    e = launch_router_logits(static_cast<const uint16_t *>(a->x), static_cast<const uint16_t *>(a->router_weight),
                             T, H, E, shared ? static_cast<const uint16_t *>(a->shared_expert_gate) : nullptr,
                             logits, LL.shared_logit, s, prefill ? nullptr : L.xl, prefill ? nullptr : L.xm, G,
                             &prep_done, LL.has_rs ? &LL.rs : nullptr);
  }
  if (e != cudaSuccess) return cuda_fail(e, "router logits");
  if (!prefill && !prep_done) {
    Prof p("prep_x", s);
    e = launch_prep_rows(static_cast<const uint16_t *>(a->x), T, H, G, L.xl, L.xm, s);
    if (e != cudaSuccess) return cuda_fail(e, "prep x");
  }
  e = cudaErrorNotSupported;
  if (T <= 8) {
    Prof p("route_group", s);
    e = launch_route_small(logits, T, E, k, a->renorm_blend, a->table_routes_of_expert, has_table ? 1 : 0, inds,
                           LL.routes, nullptr, scores, LL.mass, shared ? LL.shared_logit : nullptr,
                           shared ? LL.shared_gate : nullptr, shared ? T : 0, call.array_experts,
                           static_cast<int>(call.table.records), L.gv, s, a->keep_threshold,
                           static_cast<int>(a->min_keep), !prefill);
    if (e != cudaSuccess && e != cudaErrorNotSupported) return cuda_fail(e, "route_group");
  }
  if (e == cudaErrorNotSupported) {
    {
      Prof p("softmax_topk", s);
      e = launch_softmax_topk(logits, T, E, k, a->renorm_blend, a->table_routes_of_expert, has_table ? 1 : 0,
                              inds, LL.routes, nullptr, scores, LL.mass, shared ? LL.shared_logit : nullptr,
                              shared ? LL.shared_gate : nullptr, s, a->keep_threshold,
                              static_cast<int>(a->min_keep));
    }
    if (e != cudaSuccess) return cuda_fail(e, "softmax_topk");
    {
      Prof p("group", s);
      // the prefill GEMMs cut their own 128-pair tiles from the counts and
      // offsets: no 8-pair decode tiles (max_tiles 0 skips writing them)
      GroupView gv = L.gv;
      e = cudaErrorNotSupported;
      if (prefill) {
        gv.max_tiles = 0;
        e = launch_group_large(LL.routes, n_pairs, shared ? T : 0, call.array_experts,
                               static_cast<int>(call.table.records), gv, LL.ghist, LL.ghist_bytes, s);
        if (e != cudaSuccess && e != cudaErrorNotSupported) return cuda_fail(e, "group");
      }
      if (e == cudaErrorNotSupported)
        e = launch_group(LL.routes, n_pairs, shared ? T : 0, call.array_experts,
                         static_cast<int>(call.table.records), gv, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "group");
  }
  if (prefill) {
    {
      Prof p("prefill_tiles", s);
      e = launch_prefill_tiles(L.gv, LL.ptiles, LL.n_ptiles, LL.max_ptiles, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prefill tiles");
    {
      Prof p("gather_rows", s);
      e = launch_prefill_gather(call, L.gv, static_cast<const uint16_t *>(a->x), LL.xg, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prefill gather");
    {
      Prof p("gate_up", s);
      e = launch_prefill_gemm(true, call, L.gv, LL.ptiles, LL.n_ptiles, LL.max_ptiles, LL.xg, n_total_pairs,
                              L.act, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prefill gate_up");
    {
      Prof p("down", s);
      e = launch_prefill_gemm(false, call, L.gv, LL.ptiles, LL.n_ptiles, LL.max_ptiles, L.act, n_total_pairs,
                              L.d, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prefill down");
  } else {
    {
      Prof p("gate_up", s);
      e = launch_gate_up(call, L.gv, L.xl, L.xm, L.act, nullptr, nullptr, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "gate_up");
    {
      Prof p("prep_act", s);
      // dropped slots (adaptive keep) have no activation row: skipped
      e = launch_prep_rows(L.act, n_pairs + (shared ? T : 0), I, G, L.al, L.am, s, LL.routes, n_pairs);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prep act");
    {
      Prof p("down", s);
      e = launch_down(call, L.gv, L.al, L.am, L.d, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "down");
  }
  {
    Prof p("combine", s);
    e = launch_combine(L.d, LL.routes, scores, 0, T, k, H, shared ? kCombineParts : kCombineNone, nullptr,
                       shared ? L.d + static_cast<size_t>(n_pairs) * H : nullptr,
                       shared ? LL.shared_gate : nullptr, call.array_experts,
                       static_cast<int>(call.table.records), static_cast<uint16_t *>(a->output), s);
  }
  if (e != cudaSuccess) return cuda_fail(e, "combine");
  return FNMOE_OK;
}

int fnmoe_dequantize(const uint32_t *weight, const void *scales, const void *biases, void *out,
                     uint64_t rows, uint32_t in_width, uint32_t group_size, void *stream) {
  if (!weight || !scales || !biases || !out) return fail(FNMOE_ERR_NULL, "dequantize needs all pointers");
  if (group_size != 32 && group_size != 64) return fail(FNMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (in_width == 0 || in_width % group_size) return fail(FNMOE_ERR_SHAPE, "in_width must be group aligned");
  cudaError_t e = launch_dequant(weight, static_cast<const uint16_t *>(scales), static_cast<const uint16_t *>(biases),
                                 static_cast<uint16_t *>(out), rows, in_width, group_size,
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "dequantize");
}

int fnmoe_swiglu(const void *gate, const void *up, void *out, uint64_t n, void *stream) {
  if (!gate || !up || !out) return fail(FNMOE_ERR_NULL, "swiglu needs gate, up and out");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = ensure_exp_table(s);
  if (e != cudaSuccess) return cuda_fail(e, "exp table");
  e = launch_swiglu(static_cast<const uint16_t *>(gate), static_cast<const uint16_t *>(up),
                    static_cast<uint16_t *>(out), n, s);
  return e == cudaSuccess ? FNMOE_OK : cuda_fail(e, "swiglu");
}

int fnmoe_read_device_errors(uint32_t *flags, int clear) {
  if (flags == nullptr) return fail(FNMOE_ERR_NULL, "flags is NULL");
  uint32_t *p = device_error_word();
  if (p == nullptr) return fail(FNMOE_ERR_DEVICE, "device error word unavailable");
  cudaError_t e = cudaMemcpy(flags, p, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read device errors");
  if (clear) {
    e = cudaMemset(p, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "clear device errors");
  }
  // a bounded wait that gave up may have left a grid-barrier counter of the
  // batch-1 kernel mid-barrier: start them over (the device is idle here)
  if (*flags & kErrTimeout) {
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = reset_grid_barriers();
    if (e != cudaSuccess) return cuda_fail(e, "reset grid barriers");
  }
  return FNMOE_OK;
}

int fnmoe_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(g_prof_mutex);
  g_prof_on = on != 0;
  return FNMOE_OK;
}

int fnmoe_profile_read(char *buf, uint32_t max_len, int reset) {
  if (buf == nullptr || max_len == 0) return fail(FNMOE_ERR_NULL, "buf is NULL");
  std::lock_guard<std::mutex> lock(g_prof_mutex);
  std::map<std::string, std::pair<int, double>> agg;
  for (auto &r : g_prof) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.stop) == cudaSuccess && cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
      auto &v = agg[r.name];
      v.first += 1;
      v.second += ms;
    }
  }
  std::string text;
  for (auto &kv : agg) {
    char line[160];
    std::snprintf(line, sizeof(line), "%s %d %.6f\n", kv.first.c_str(), kv.second.first, kv.second.second);
    text += line;
  }
  if (reset) {
    for (auto &r : g_prof) {
      cudaEventDestroy(r.start);
      cudaEventDestroy(r.stop);
    }
    g_prof.clear();
  }
  std::strncpy(buf, text.c_str(), max_len - 1);
  buf[max_len - 1] = '\0';
  return FNMOE_OK;
}

int fnmoe_paged_decode_workspace_size(const FnPagedArgs *args, uint64_t *bytes) {
  return paged_workspace_size(args, bytes, g_last_error);
}

int fnmoe_paged_decode(const FnPagedArgs *args, void *stream) {
  return paged_decode(args, static_cast<cudaStream_t>(stream), g_last_error);
}

int fnmoe_rows_dequantize(const FnRowsArgs *args, void *stream) {
  return rows_dequant(args, static_cast<cudaStream_t>(stream), g_last_error);
}

int fnmoe_tiled_record_bytes(uint32_t hidden_size, uint32_t inter_size, uint32_t group_size,
                             uint64_t *gate_up_record_bytes, uint64_t *down_record_bytes) {
  if (!gate_up_record_bytes || !down_record_bytes) return fail(FNMOE_ERR_NULL, "output pointers are required");
  if (group_size != 32 && group_size != 64) return fail(FNMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (hidden_size == 0 || inter_size == 0 || hidden_size % group_size || inter_size % group_size)
    return fail(FNMOE_ERR_SHAPE, "Q4 projection inputs must be group aligned");
  if (inter_size % 8 || hidden_size % 16)
    return fail(FNMOE_ERR_SHAPE, "tiled tables need inter_size % 8 == 0 and hidden_size % 16 == 0");
  *gate_up_record_bytes = tiled_record_bytes(static_cast<int>(inter_size), static_cast<int>(hidden_size), true);
  *down_record_bytes = tiled_record_bytes(static_cast<int>(hidden_size), static_cast<int>(inter_size), false);
  return FNMOE_OK;
}

int fnmoe_tile_experts(const FnTileArgs *a, void *stream) {
  if (a == nullptr) return fail(FNMOE_ERR_NULL, "args is NULL");
  if (a->abi_version != FNMOE_ABI_VERSION) return fail(FNMOE_ERR_ABI, "abi_version mismatch");
  uint64_t gu = 0, dn = 0;
  if (int rc = fnmoe_tiled_record_bytes(a->hidden_size, a->inter_size, a->group_size, &gu, &dn)) return rc;
  if (a->experts == 0) return FNMOE_OK;
  if (!a->gate_weight || !a->gate_scales || !a->gate_biases || !a->up_weight || !a->up_scales || !a->up_biases ||
      !a->down_weight || !a->down_scales || !a->down_biases)
    return fail(FNMOE_ERR_NULL, "gate, up and down projections with scales and biases are required");
  if (!a->tiled.gate_up || !a->tiled.down) return fail(FNMOE_ERR_NULL, "destination tables are required");
  if (a->tiled.gate_up_record_bytes != gu || a->tiled.down_record_bytes != dn)
    return fail(FNMOE_ERR_SHAPE, "destination record sizes do not match hidden/inter sizes");
  if (static_cast<uint64_t>(a->first_record) + a->experts > a->tiled.records)
    return fail(FNMOE_ERR_SHAPE, "records past the end of the destination tables");
  std::string why;
  if (!device_ok(why)) return fail(FNMOE_ERR_DEVICE, why);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int H = static_cast<int>(a->hidden_size), I = static_cast<int>(a->inter_size);
  const int G = static_cast<int>(a->group_size), E = static_cast<int>(a->experts);
  uint8_t *gdst = static_cast<uint8_t *>(const_cast<void *>(a->tiled.gate_up)) + gu * a->first_record;
  uint8_t *ddst = static_cast<uint8_t *>(const_cast<void *>(a->tiled.down)) + dn * a->first_record;
  cudaError_t e = launch_tile_experts(a->gate_weight, a->up_weight, static_cast<const uint16_t *>(a->gate_scales),
                                      static_cast<const uint16_t *>(a->gate_biases),
                                      static_cast<const uint16_t *>(a->up_scales),
                                      static_cast<const uint16_t *>(a->up_biases), E, I, H, G, true, gdst, gu, s);
  if (e != cudaSuccess) return cuda_fail(e, "tile gate/up");
  e = launch_tile_experts(a->down_weight, a->down_weight, static_cast<const uint16_t *>(a->down_scales),
                          static_cast<const uint16_t *>(a->down_biases),
                          static_cast<const uint16_t *>(a->down_scales),
                          static_cast<const uint16_t *>(a->down_biases), E, H, I, G, false, ddst, dn, s);
  if (e != cudaSuccess) return cuda_fail(e, "tile down");
  return FNMOE_OK;
}

int fnmoe_ep_create(const FnEpConfig *config, void **handle) {
  std::string why;
  if (!device_ok(why)) return fail(FNMOE_ERR_DEVICE, why);
  return ep_create(config, handle, g_last_error);
}

int fnmoe_ep_ipc_handle(void *handle, void *out) { return ep_ipc_handle(handle, out, g_last_error); }

int fnmoe_ep_open_peers(void *handle, const void *handles) { return ep_open_peers(handle, handles, g_last_error); }

int fnmoe_ep_window(void *handle, FnEpWindow *window) { return ep_window(handle, window, g_last_error); }

int fnmoe_ep_dispatch(void *handle, const void *x, const uint32_t *inds, uint32_t tokens, void *stream) {
  Prof p("ep_dispatch", static_cast<cudaStream_t>(stream));
  return ep_dispatch(handle, x, inds, tokens, static_cast<cudaStream_t>(stream), g_last_error);
}

int fnmoe_ep_return_combine(void *handle, const void *scores, const void *shared_gate, uint32_t tokens, void *out,
                            void *stream) {
  Prof p("ep_return_combine", static_cast<cudaStream_t>(stream));
  return ep_return_combine(handle, scores, shared_gate, tokens, out, static_cast<cudaStream_t>(stream), g_last_error);
}

int fnmoe_ep_destroy(void *handle) { return ep_destroy(handle, g_last_error); }

}  // extern "C"
