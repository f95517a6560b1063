// decode_layer.cuh -- a batch-1 sparse-MoE layer as ONE persistent kernel.
//
// Included at the end of moe_kernels.cu (same translation unit): it reuses
// the expert kernels' block arithmetic (compute_block), the bfloat16 exp
// table and the device error word, so its results are bit-identical to the
// multi-launch layer (router -> top-k -> gate/up -> activation fixed point ->
// down -> combine), which the CPU oracle pins.
//
// Why one kernel: at batch 1 the layer moves ~24 MB (H2048/I512, top-10 +
// shared expert) -- under 4 us of HBM time -- but six dependent launches
// cost ~5 us each in launch/dependency latency plus first-byte latency,
// because the expert kernels cannot ask for weights before the routing
// kernel has finished.  Here every CTA (one per SM, co-resident: cooperative
// launch) runs three phases separated by two grid barriers:
//
//  A  row fixed point of x (shared memory), bulk copies of this CTA's
//     shared-expert gate/up row groups (routing-independent), the router
//     GEMV rows of this CTA (one row per warp, the exact integer dot product
//     of the row fixed points),
//     logits to global.                                          barrier 1
//  B  softmax / top-k / keep / renorm of the 512 logits, recomputed by
//     every CTA (identical arithmetic, so identical results -- no third
//     barrier), then the bulk copies of this CTA's routed gate/up row groups
//     and its down row groups of every routed expert are issued at once;
//     each warp folds one gate/up item (8 gate + 8 up rows over the whole
//     contraction, groups in canonical order) and writes its SwiGLU
//     activations to global.                                     barrier 2
//  C  row fixed point of the (k + 1) activation rows, then the down row
//     group of every expert (16 rows each) and the slot-ordered combine of
//     those 16 output rows in the same CTA -- no combine launch.
//
// Work items: gate/up item j = unit * (I/8) + row group, unit 0 the shared
// expert (when present) then the kept routed slots in slot order; CTA c takes
// items c, c + nCTA, ...; down row group dg (16 rows of H) goes to CTA
// dg mod nCTA.  Every wait is bounded: a grid barrier or mbarrier that gives
// up sets kErrTimeout, the CTA waits (bounded) for its copies in flight and
// returns; the outputs of that call are then invalid.

constexpr int kFusedThreads = 512;
constexpr int kFusedWarps = kFusedThreads / 32;
constexpr int kFusedMaxSlots = 16;              // gate/up items per CTA
constexpr int kFusedRowsPerGroup = 5;           // activation rows per fixed-point thread group (I <= 1024)
constexpr uint32_t kGridSpinLimit = 1u << 24;   // barrier polls (one L2 round trip each): ~1-2 s

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t atom_add_release_gpu(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Grid barrier over co-resident CTAs (one call per CTA per barrier).  The
// counter flips its top bit once per completed barrier: CTA 0 adds
// 2^31 - (nCTA - 1), every other CTA adds 1, so the arrivals sum to exactly
// 2^31 and each CTA waits until the top bit differs from the value its own
// add returned.  The low 31 bits are back to zero after every complete
// barrier, so a counter that starts at zero needs no reset between launches.
// Ordering: the CTA barrier orders the CTA's writes before thread 0's
// release add; a waiter's acquire load that sees the flip, then its CTA
// barrier, orders them before every later read of its CTA (L2-coherent:
// ld.cg / acquire).  The spin has no back-off: the wake-up latency is one
// L2 round trip.  Returns false (and flags kErrTimeout) if it gave up; the
// counter is then left mid-barrier (fnmoe_read_device_errors clears it).
__device__ __forceinline__ bool grid_sync(uint32_t *bar, uint32_t *err, int *s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t inc = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1u) : 1u;
    const uint32_t old = atom_add_release_gpu(bar, inc);
    int ok = 1;
    uint32_t spins = 0;
    while (((old ^ ld_acquire_gpu(bar)) & 0x80000000u) == 0u) {
      if (++spins >= kGridSpinLimit) {
        ok = 0;
        set_error(err, kErrTimeout);
        break;
      }
    }
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

// Bounded wait on an mbarrier phase; false (and kErrTimeout) if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity, uint32_t *err) {
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins >= kSpinLimit) {
      set_error(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// Row fixed point of one row of K bfloat16 values by a group of TPR threads
// (TPR a multiple of 32; this thread is tr of the group; named barrier
// `bar_id` spans the group), in prep_rows_body's layout and arithmetic --
// the same integer definition, so the same bits: limbs [K/G][2][G] fp16 in
// fragment order, meta [meta_pitch] floats.  A row in global memory is read
// through L2 (ld.cg): other CTAs of this kernel wrote it before a barrier.
template <int G, int SPT>
__device__ __forceinline__ void fixed_point_group(const uint16_t *row, bool from_global, int K, int tr, int TPR,
                                                  uint16_t *limbs, float *meta, uint32_t *err, int bar_id,
                                                  uint32_t *s_mx) {
  constexpr int LPG = G / 8;  // lanes per group
  const int lane = threadIdx.x & 31;
  const int Gc = K / G, slices = K / 8;
  uint4 v[SPT];
  uint32_t mx = 0;
  bool bad = false;
#pragma unroll
  for (int q = 0; q < SPT; ++q) {
    const int i = tr + q * TPR;
    v[q] = make_uint4(0u, 0u, 0u, 0u);
    if (i < slices)
      v[q] = from_global ? __ldcg(reinterpret_cast<const uint4 *>(row) + i) : reinterpret_cast<const uint4 *>(row)[i];
    const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t a = (w[e >> 1] >> (16 * (e & 1))) & 0x7FFFu;
      if (a >= 0x7F80u) bad = true;
      else mx = max(mx, a);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) set_error(err, kErrNonFinite);
  if (lane == 0) s_mx[tr >> 5] = mx;
  named_sync(bar_id, TPR);
  for (int q = 0; q < TPR / 32; ++q) mx = max(mx, s_mx[q]);
  int E = 0;
  if (mx != 0) E = (mx >> 7) ? static_cast<int>(mx >> 7) - 127 : (31 - __clz(static_cast<int>(mx))) - 133;
#pragma unroll
  for (int q = 0; q < SPT; ++q) {
    const int i = tr + q * TPR;
    int sx = 0;
    if (i < slices) {
      const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
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
      uint16_t *dst = limbs + static_cast<size_t>(g) * 2 * G + within;
      *reinterpret_cast<uint4 *>(dst) = make_uint4(half_pair(l0[0], l0[4]), half_pair(l0[1], l0[5]),
                                                   half_pair(l0[2], l0[6]), half_pair(l0[3], l0[7]));
      *reinterpret_cast<uint4 *>(dst + G) = make_uint4(half_pair(l1[0], l1[4]), half_pair(l1[1], l1[5]),
                                                       half_pair(l1[2], l1[6]), half_pair(l1[3], l1[7]));
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) sx += __shfl_xor_sync(0xFFFFFFFFu, sx, off);
    if (i < slices && (lane & (LPG - 1)) == 0) meta[(8 * i) / G] = __int2float_rn(sx);
  }
  if (tr == 0) {
    const int ai = meta_a_index(Gc);
    for (int g = Gc; g < ai; ++g) meta[g] = 0.0f;
    const int k = E - 22;
    const int ka = max(k, -126);
    meta[ai] = __int_as_float((ka + 127) << 23);          // A = 2^ka, normal
    meta[ai + 1] = __int_as_float((k - ka + 127) << 23);  // B = 2^(k-ka)
    meta[ai + 2] = 0.0f;
    meta[ai + 3] = 0.0f;
  }
}

// Exact per-group sums of one staged tiled block (row group x 128-byte
// block, fragment order) against one token's limbs: S = sum_i X_i q_i for
// the block's GPB groups of MMA rows r (A) and r + 8 (B), formed on the
// tensor cores exactly as k_expert_gemv does.  The sums are parked in the
// block's own packed-word area, whose words this warp has consumed:
// [group j][row r][A, B] float.  Every MMA column reads the same token, so
// lanes c = 0 store.
template <int G>
__device__ __forceinline__ void block_sums(uint32_t st, uint32_t xb, int b, int Gc, int r, int c) {
  constexpr int GPB = 2 * kBlkBytes / G;
  constexpr int QG = GPB / 2;
  constexpr int WB = G / 32;
  const uint32_t wq = st + (r * 4 + c) * 16;
  float SA[GPB], SB[GPB];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 wA4 = lds128(wq + (2 * h) * 512);
    const uint4 wB4 = lds128(wq + (2 * h + 1) * 512);
#pragma unroll
    for (int j = 0; j < QG; ++j) {
      const int jj = h * QG + j;
      const int g = b * GPB + jj;
      SA[jj] = SB[jj] = 0.0f;
      if (g < Gc) {
        uint32_t A0[WB][4], A1[WB][4];
#pragma unroll
        for (int wb = 0; wb < WB; ++wb)
          nibble_operands(word_at(wA4, j * WB + wb), word_at(wB4, j * WB + wb), A0[wb], A1[wb]);
        float C[4];
#pragma unroll
        for (int wb = 0; wb < WB; ++wb) {
          const uint4 v = lds128(xb + g * (4 * G) + wb * 64);
          if (wb == 0) mma_16816_z(C, A0[wb], v.x, v.y);
          else mma_16816(C, A0[wb], v.x, v.y);
          mma_16816(C, A1[wb], v.z, v.w);
        }
        SA[jj] = __fmaf_rn(C[0], 4096.0f, C[1]);
        SB[jj] = __fmaf_rn(C[2], 4096.0f, C[3]);
      }
    }
  }
  __syncwarp();  // every lane has read its words: the area is free
  if (c == 0) {
#pragma unroll
    for (int jj = 0; jj < GPB; ++jj)
      asm volatile("st.shared.v2.f32 [%0], {%1, %2};\n" ::"r"(st + (jj * 8 + r) * 8), "f"(SA[jj]), "f"(SB[jj])
                   : "memory");
  }
}

// Canonical fold of one MMA row (mrow 0-15 of a row group) over the staged
// blocks of an item: acc = fma(b_g, fl(SX_g), fma(s_g, S_g, acc)) for the
// groups in increasing order (group_step's two fmas), from -0.0.  The next
// block's sums, scales, biases and fl(SX) are loaded while the current one
// is folded, and groups past Gc leave acc unchanged (select, no branch).
template <int G>
struct FoldBlock {
  static constexpr int GPB = 2 * kBlkBytes / G;
  uint4 s8, b8;
  float S[GPB], F[GPB];
};

template <int G>
__device__ __forceinline__ void fold_load(uint32_t item, uint32_t sxa, int b, int mrow, FoldBlock<G> &d) {
  constexpr int GPB = FoldBlock<G>::GPB;
  const int side = mrow >> 3, r = mrow & 7;
  const uint32_t ch = item + b * kTileChunk;
  d.s8 = lds128(ch + kTileW + mrow * 32);
  d.b8 = lds128(ch + kTileW + mrow * 32 + 16);
#pragma unroll
  for (int j = 0; j < GPB; ++j) d.S[j] = __uint_as_float(lds32(ch + (j * 8 + r) * 8 + side * 4));
#pragma unroll
  for (int j4 = 0; j4 < GPB / 4; ++j4) {
    const uint4 f = lds128(sxa + (b * GPB + 4 * j4) * 4);  // fl(SX) rows are padded: in bounds
    d.F[4 * j4] = __uint_as_float(f.x);
    d.F[4 * j4 + 1] = __uint_as_float(f.y);
    d.F[4 * j4 + 2] = __uint_as_float(f.z);
    d.F[4 * j4 + 3] = __uint_as_float(f.w);
  }
}

template <int G>
__device__ __forceinline__ float fold_row(const uint8_t *item, int nblk, int Gc, int mrow, const float *sx) {
  constexpr int GPB = FoldBlock<G>::GPB;
  const uint32_t it = smem_u32(item), sxa = smem_u32(sx);
  FoldBlock<G> cur, nxt;
  fold_load<G>(it, sxa, 0, mrow, cur);
  float acc = -0.0f;
  for (int b = 0; b < nblk; ++b) {
    if (b + 1 < nblk) fold_load<G>(it, sxa, b + 1, mrow, nxt);
#pragma unroll
    for (int j = 0; j < GPB; ++j) {
      const int sh = 16 * (j & 1);
      const float sc = bf16_to_f32(static_cast<uint16_t>(word_at(cur.s8, j >> 1) >> sh));
      const float bi = bf16_to_f32(static_cast<uint16_t>(word_at(cur.b8, j >> 1) >> sh));
      const float na = __fmaf_rn(bi, cur.F[j], __fmaf_rn(sc, cur.S[j], acc));
      acc = (b * GPB + j < Gc) ? na : acc;
    }
    cur = nxt;
  }
  return acc;
}

template <int G>
__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_layer(FusedLayer p, uint32_t *err) {
  constexpr int GPB = 2 * kBlkBytes / G;  // groups per 128-byte block
  (void)GPB;
  extern __shared__ __align__(128) uint8_t fsm[];
  __shared__ uint64_t s_bar[kFusedMaxSlots + 1];  // ring slots, then the down stage
  __shared__ int s_flag;
  __shared__ int s_dead;
  __shared__ uint32_t s_idx[kCombineMaxSlots];
  __shared__ float s_score[kCombineMaxSlots];
  __shared__ float s_red[kFusedWarps];
  __shared__ uint32_t s_mx[8][8];
  __shared__ uint32_t s_rmx[8];     // router row half maxima (warps 0-7)
  __shared__ uint32_t s_xmx[8];     // maxima of x by eighths (warps 0-7)
  __shared__ long long s_rsum[8];   // router row half sums (warps 0-7)
  __shared__ int s_keep;
  __shared__ float s_sg;
  __shared__ uint32_t s_armed;    // ring slots armed (bit i)
  __shared__ uint32_t s_dphase;   // down-stage arms so far

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, c = lane & 3;
  const int NB = gridDim.x, cta = blockIdx.x;
  const int H = p.H, I = p.I, E = p.E, k = p.k;
  const bool has_sh = p.wsg != nullptr;
  const int n_rg = I / 8;    // gate/up row groups (8 gate + 8 up rows)
  const int n_dg = H / 16;   // down row groups
  const int nblk_h = (H / 2 + kBlkBytes - 1) / kBlkBytes;
  const int nblk_i = (I / 2 + kBlkBytes - 1) / kBlkBytes;
  const uint32_t gu_item = static_cast<uint32_t>(nblk_h) * kTileChunk;
  const uint32_t dn_item = static_cast<uint32_t>(nblk_i) * kTileChunk;
  const XStage xsh = xstage_geom(H, G);
  const XStage xsi = xstage_geom(I, G);

  uint16_t *xs = reinterpret_cast<uint16_t *>(fsm + p.off_x);
  int *xqs = reinterpret_cast<int *>(fsm + p.off_xq);
  uint8_t *xl = fsm + p.off_xl;
  float *xm = reinterpret_cast<float *>(fsm + p.off_xm);
  float *soft = reinterpret_cast<float *>(fsm + p.off_soft);
  float *dsm = reinterpret_cast<float *>(fsm + p.off_d);
  uint8_t *ring = fsm + p.off_ring;
  uint8_t *dstage = fsm + p.off_down;
  uint8_t *al = fsm + p.off_al;
  uint8_t *am = fsm + p.off_am;

  if (tid == 0) {
    for (int i = 0; i <= p.nslot; ++i) mbar_init(&s_bar[i], 1);
    mbar_init_fence();
    s_dead = 0;
    s_armed = 0;
    s_dphase = 0;
  }
  __syncthreads();

  // record of a unit (0 = shared expert when present, then the kept slots)
  auto unit_record = [&](int q) -> uint32_t {
    if (has_sh) {
      if (q == 0) return p.tiled.records - 1;
      --q;
    }
    return s_idx[q];
  };
  auto unit_row = [&](int q) -> int {  // activation row of a unit
    if (has_sh) {
      if (q == 0) return k;
      --q;
    }
    return q;
  };
  auto issue_gu = [&](int slot, int j) {  // one lane: item j into ring slot `slot`
    const int q = j / n_rg, rg = j - q * n_rg;
    const uint8_t *src = p.tiled.gate_up + static_cast<size_t>(unit_record(q)) * p.tiled.gate_up_record +
                         static_cast<size_t>(rg) * gu_item;
    fence_proxy_async();
    mbar_expect_tx(&s_bar[slot], gu_item);
    bulk_g2s(ring + static_cast<size_t>(slot) * gu_item, src, gu_item, &s_bar[slot]);
  };
  // one warp: row group dg of every unit into the down stage
  auto issue_down = [&](int dg, int n_units) {
    if (lane == 0) {
      fence_proxy_async();
      mbar_expect_tx(&s_bar[p.nslot], static_cast<unsigned>(n_units) * dn_item);
    }
    __syncwarp();
    for (int q = lane; q < n_units; q += 32) {
      fence_proxy_async();
      bulk_g2s(dstage + static_cast<size_t>(q) * dn_item,
               p.tiled.down + static_cast<size_t>(unit_record(q)) * p.tiled.down_record +
                   static_cast<size_t>(dg) * dn_item,
               dn_item, &s_bar[p.nslot]);
    }
    if (lane == 0) ++s_dphase;
  };
  // Wait (bounded) for every copy this CTA issued before leaving early.
  auto drain = [&]() {
    __syncthreads();
    if (tid == 0) {
      for (int i = 0; i < p.nslot; ++i)
        if (s_armed & (1u << i)) mbar_wait_bounded(&s_bar[i], 0, err);
      if (s_dphase > 0) mbar_wait_bounded(&s_bar[p.nslot], (s_dphase - 1) & 1, err);
    }
    __syncthreads();
  };

  // ---------------- phase A ----------------
  // Constant data first -- the shared expert's gate/up row groups of this
  // CTA (routing-independent), its down rows into L2, and this warp's
  // router row -- then wait for the previous kernel of the stream (under
  // programmatic dependent launch this kernel may start while it runs).
  if (warp == 0 && has_sh) {
    const int j = cta + NB * lane;
    const bool mine = lane < p.nslot && j < n_rg;
    if (mine) issue_gu(lane, j);
    const unsigned armed = __ballot_sync(0xFFFFFFFFu, mine);
    if (lane == 0) s_armed = armed;
    for (int dg = cta + NB * lane; dg < n_dg; dg += NB * 32)
      bulk_prefetch_l2(p.tiled.down + static_cast<size_t>(p.tiled.records - 1) * p.tiled.down_record +
                           static_cast<size_t>(dg) * dn_item,
                       dn_item);
  }
  // Router rows: warps 0-7 in pairs, pair q = warp / 2 owns row cta + NB * q
  // (E + 1 <= 4 * nCTA; row E is the shared gate row), each warp of a pair
  // half of the row's 8-element chunks.  Integer sums combine exactly, so
  // the halves add in shared memory.
  const int nchunks = H / 8;
  const int hc = (nchunks + 1) / 2;             // chunks per half (<= 256: H <= 4096)
  const int half = warp & 1;
  const int row = cta + NB * (warp >> 1);
  const bool router_warp = warp < 8 && row < E + (has_sh ? 1 : 0);
  const int c_end = min(nchunks, (half + 1) * hc);
  uint4 wv[8];
  if (router_warp) {
    const uint16_t *wrow = row < E ? p.W + static_cast<size_t>(row) * H : p.wsg;
    bool bad = false;
    uint32_t mw = 0;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int cidx = half * hc + lane + 32 * m;
      wv[m] = (cidx < c_end) ? ldg_u128(reinterpret_cast<const uint4 *>(wrow + cidx * 8)) : make_uint4(0, 0, 0, 0);
      mw = max(mw, max_mag8(wv[m], bad));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mw = max(mw, __shfl_xor_sync(0xFFFFFFFFu, mw, off));
    if (lane == 0) s_rmx[warp] = mw;  // the router row's half maximum (constant data: before the wait)
  }
  pdl_trigger();
  pdl_wait();
  // per-unit activation maxima: zeroed here, raised by the gate/up CTAs
  // after barrier 1, read after barrier 2
  if (cta == 0 && tid < kCombineMaxSlots + 1) p.amax[tid] = 0u;
  // x (an input of the call) into shared memory
  for (int i = tid; i < H / 8; i += kFusedThreads)
    reinterpret_cast<uint4 *>(xs)[i] = reinterpret_cast<const uint4 *>(p.x)[i];
  __syncthreads();
  if (warp >= 8) {
    // row fixed point of x: warps 8-15 (named barrier 1)
    const int tr = tid - 256;
    if (H / 8 <= 256)
      fixed_point_group<G, 1>(xs, false, H, tr, 256, reinterpret_cast<uint16_t *>(xl), xm, err, 1, s_mx[0]);
    else
      fixed_point_group<G, 2>(xs, false, H, tr, 256, reinterpret_cast<uint16_t *>(xl), xm, err, 1, s_mx[0]);
  } else {
    // exact integer dot product of the row fixed points (k_router_logits'
    // arithmetic).  x's maximum: each of warps 0-7 takes an eighth of x
    // (named barrier 2 over the 256 router-warp threads).
    bool bad = false;
    uint32_t mxx = 0;
    for (int c = warp * 32 + lane; c < nchunks; c += 256)
      mxx = max(mxx, max_mag8(reinterpret_cast<const uint4 *>(xs)[c], bad));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mxx = max(mxx, __shfl_xor_sync(0xFFFFFFFFu, mxx, off));
    if (lane == 0) s_xmx[warp] = mxx;
    named_sync(2, 256);
    uint32_t mx_all = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) mx_all = max(mx_all, s_xmx[w]);
    const int ex = row_exponent(mx_all);
    // x's fixed point, once per CTA: each of warps 0-7 converts an eighth
    {
      const FixScale sx = fix_scale(ex, kRouterXBits);
      for (int c = warp * 32 + lane; c < nchunks; c += 256) {
        const uint4 v = reinterpret_cast<const uint4 *>(xs)[c];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        int q8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q8[i] = fixed_qf((u[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, sx);
        reinterpret_cast<int4 *>(xqs)[2 * c] = make_int4(q8[0], q8[1], q8[2], q8[3]);
        reinterpret_cast<int4 *>(xqs)[2 * c + 1] = make_int4(q8[4], q8[5], q8[6], q8[7]);
      }
    }
    named_sync(2, 256);
    if (router_warp) {
      const int ew = row_exponent(max(s_rmx[warp & ~1], s_rmx[warp | 1]));
      const FixScale sw = fix_scale(ew, kRouterWBits);
      long long a = 0;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int cidx = half * hc + lane + 32 * m;
        if (cidx < c_end) {
          const int4 x0 = reinterpret_cast<const int4 *>(xqs)[2 * cidx];
          const int4 x1 = reinterpret_cast<const int4 *>(xqs)[2 * cidx + 1];
          const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          const uint32_t wu[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w};
#pragma unroll
          for (int i = 0; i < 8; ++i)
            a += static_cast<long long>(fixed_qf((wu[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, sw)) * xv[i];
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, off);
      if (lane == 0) s_rsum[warp] = a;
      __syncwarp();
      // the pair's halves meet: a barrier over just the pair's 64 threads
      asm volatile("bar.sync %0, 64;\n" ::"r"(3 + (warp >> 1)) : "memory");
      if (half == 0 && lane == 0) {
        const uint16_t bits = router_logit_bits(s_rsum[warp] + s_rsum[warp + 1], ex, ew);
        if (row < E) p.logits[row] = bits;
        else p.shared_logit[0] = bits;
      }
    }
  }
  if (!grid_sync(p.bar, err, &s_flag)) {
    drain();
    return;
  }

  // ---------------- phase B: routing (every CTA, same arithmetic) ----------------
  const int per = (E + 31) / 32;
  float lmax = -INFINITY;
  for (int i = tid; i < E; i += kFusedThreads) {
    const float l = bf16_to_f32(__ldcg(p.logits + i));
    soft[i] = l;
    lmax = fmaxf(lmax, l);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, off));
  if (lane == 0) s_red[warp] = lmax;
  __syncthreads();
  float M = s_red[0];
#pragma unroll
  for (int w = 1; w < kFusedWarps; ++w) M = fmaxf(M, s_red[w]);
  for (int i = tid; i < E; i += kFusedThreads)
    soft[i] = __double2float_rn(exp(static_cast<double>(__fsub_rn(soft[i], M))));
  __syncthreads();
  if (warp == 0) {
    float sum = -0.0f;  // canonical order: lane chains over m, then the xor butterfly
    for (int m = 0; m < per; ++m)
      if (lane + 32 * m < E) sum = __fadd_rn(sum, soft[lane + 32 * m]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, off));
    if (lane == 0) s_red[0] = sum;
  }
  __syncthreads();
  // top-k, level 1: each warp forms the keys of its slice in registers and
  // takes their k largest, one redux.sync per pick (keys are unique and
  // nonzero; 0 = none); level 2 (warp 0) picks the k largest of the 16
  // candidate lists in the same way -- the order the serial selection of
  // k_route_small gives.
  uint32_t *cand = reinterpret_cast<uint32_t *>(soft) + ((E + 31) & ~31);
  {
    const float S = s_red[0];
    const int chunk = (E + kFusedWarps - 1) / kFusedWarps;  // <= 64 (E <= 1024)
    const int lo = warp * chunk, hi = min(E, lo + chunk);
    auto key_of = [&](int i) -> uint32_t {
      if (i >= hi) return 0u;
      const uint32_t pb = f32_to_bf16(__fdiv_rn(soft[i], S));
      return (pb << 16) | (0xFFFFu - static_cast<uint32_t>(i));
    };
    uint32_t k0 = key_of(lo + lane);
    uint32_t k1 = key_of(lo + 32 + lane);
    for (int q = 0; q < k; ++q) {
      const uint32_t best = __reduce_max_sync(0xFFFFFFFFu, max(k0, k1));
      if (k0 == best) k0 = 0u;
      if (k1 == best) k1 = 0u;
      if (lane == 0) cand[warp * k + q] = best;
    }
  }
  __syncthreads();
  if (warp == 0) {
    const int nc = kFusedWarps * k;  // <= 256
    uint32_t key[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) key[m] = (lane + 32 * m < nc) ? cand[lane + 32 * m] : 0u;
    float acc = 0.0f, sel = 0.0f;
    uint32_t idx = 0;
    for (int q = 0; q < k; ++q) {
      uint32_t best = 0u;
#pragma unroll
      for (int m = 0; m < 8; ++m) best = max(best, key[m]);
      best = __reduce_max_sync(0xFFFFFFFFu, best);
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (key[m] == best) key[m] = 0u;
      const float pr = bf16_to_f32(static_cast<uint16_t>(best >> 16));
      if (lane == q) {
        sel = pr;
        idx = 0xFFFFu - (best & 0xFFFFu);
      }
      acc = __fadd_rn(acc, pr);
    }
    const float topm = round_bf16(acc);
    const int keep = keep_count([&](int s) { return __shfl_sync(0xFFFFFFFFu, sel, s); }, k, p.keep_threshold,
                                p.min_keep);
    float kept = 0.0f;
    for (int s = 0; s < keep; ++s) kept = __fadd_rn(kept, __shfl_sync(0xFFFFFFFFu, sel, s));
    const float selected = round_bf16(kept);
    const uint32_t idx0 = __shfl_sync(0xFFFFFFFFu, idx, 0);
    const float bl = round_bf16(p.blend);
    const float normalizer = badd(topm, bmul(bl, bsub(selected, topm)));
    if (lane < k) {
      const bool live = lane < keep;
      const uint16_t sc = live ? f32_to_bf16(__fdiv_rn(sel, normalizer)) : 0;
      s_idx[lane] = live ? idx : idx0;
      s_score[lane] = bf16_to_f32(sc);
      if (cta == 0) {
        p.inds[lane] = live ? idx : idx0;
        p.scores[lane] = sc;
      }
    }
    if (lane == 0) {
      s_keep = keep;
      if (cta == 0) p.mass[0] = f32_to_bf16(topm);
    }
  }
  __syncthreads();
  const int keep = s_keep;
  const int n_units = (has_sh ? 1 : 0) + keep;
  const int n_items = n_units * n_rg;
  int n_my = 0;
  while (n_my < p.nslot && cta + NB * n_my < n_items) ++n_my;
  const bool has_dg = cta < n_dg;
  if (warp == 0) {
    const int j = cta + NB * lane;
    const bool mine = lane < n_my && !(has_sh && j < n_rg);  // shared items are in flight
    if (mine) issue_gu(lane, j);
    const unsigned armed = __ballot_sync(0xFFFFFFFFu, mine);
    if (lane == 0) s_armed |= armed;
  } else if (warp == 1) {
    if (has_dg && !p.alias) issue_down(cta, n_units);
    // the shared expert's sigmoid gate, needed only by the combine: its
    // loads overlap the expert data's arrival instead of the routing
    if (lane == 0) {
      s_sg = has_sh ? sigmoid_bf16_direct(bf16_to_f32(__ldcg(p.shared_logit))) : 0.0f;
      if (cta == 0 && has_sh) p.shared_gate[0] = f32_to_bf16(s_sg);
    }
  } else if (warp == 2) {
    // down rows of this CTA's row groups that are not staged yet: into L2
    const int first = p.alias ? cta : cta + NB;
    const int q0 = has_sh ? 1 : 0;
    const int per_dg = n_units - q0;
    for (int dg = first; dg < n_dg && per_dg > 0; dg += NB)
      for (int q = q0 + lane; q < n_units; q += 32)
        bulk_prefetch_l2(p.tiled.down + static_cast<size_t>(unit_record(q)) * p.tiled.down_record +
                             static_cast<size_t>(dg) * dn_item,
                         dn_item);
  }
  __syncthreads();  // s_armed / s_dphase

  // gate/up: (item, block) units over the warps -- exact group sums
  {
    const uint32_t xb = smem_u32(xl) + (r & 1) * (G * 2) + c * 16;  // one token: every MMA column reads it
    const int units = n_my * nblk_h;
    for (int u = warp; u < units; u += kFusedWarps) {
      const int i = u / nblk_h, b = u - i * nblk_h;
      if (!mbar_wait_bounded(&s_bar[i], 0, err)) {
        s_dead = 1;
        continue;
      }
      block_sums<G>(smem_u32(ring + static_cast<size_t>(i) * gu_item + static_cast<size_t>(b) * kTileChunk), xb, b,
                    xsh.Gc, r, c);
    }
  }
  __syncthreads();
  // canonical fold: one thread per (item, MMA row); gate (rows 0-7) and up
  // (rows 8-15) of a row meet in lanes t and t ^ 8 for the SwiGLU
  if (!s_dead && tid < ((n_my * 16 + 31) & ~31)) {
    const int i = tid >> 4, mrow = tid & 15;
    const bool live = i < n_my;
    float y = 0.0f;
    if (live) {
      const float acc = fold_row<G>(ring + static_cast<size_t>(i) * gu_item, nblk_h, xsh.Gc, mrow, xm);
      const float2 ab = *reinterpret_cast<const float2 *>(xm + xsh.a_off / 4);
      y = round_bf16(__fmul_rn(__fmul_rn(acc, ab.x), ab.y));
    }
    const float other = __shfl_xor_sync(0xFFFFFFFFu, y, 8);
    // the row group's largest finite activation magnitude (bfloat16
    // magnitudes order like their bit patterns) goes to the unit's max word
    const int j = cta + NB * i;
    const int q = j / n_rg, rg = j - q * n_rg;
    uint32_t mag = 0u;
    if (live && mrow < 8) {
      const uint16_t a = f32_to_bf16(swiglu_bf16_direct(y, other));
      p.act[static_cast<size_t>(unit_row(q)) * I + rg * 8 + mrow] = a;
      mag = a & 0x7FFFu;
      if (mag >= 0x7F80u) {
        set_error(err, kErrNonFinite);
        mag = 0u;
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) mag = max(mag, __shfl_xor_sync(0xFFFFFFFFu, mag, off));
    if (live && mrow == 0) atomicMax(p.amax + unit_row(q), mag);
  }
  if (p.alias) {
    __syncthreads();  // the ring is free: stage this CTA's first down row group there
    if (warp == 1 && has_dg && !s_dead) issue_down(cta, n_units);
  }
  if (!grid_sync(p.bar, err, &s_flag) || s_dead) {
    drain();
    return;
  }

  // ---------------- phase C: down + combine ----------------
  if (!has_dg) return;  // nothing in flight: no down stage was armed
  {
    // row fixed point of the units' activation rows from the published row
    // maxima: groups of TPR threads, group rl owns rows rl, rl + rpc, ...
    // (<= kFusedRowsPerGroup); every load is issued before any row is done
    const int slices = I / 8;
    const int TPR = (slices + 31) & ~31;
    const int rpc = min(8, kFusedThreads / TPR);
    const int rl = tid / TPR, tr = tid - rl * TPR;
    const int nr = rl < rpc && rl < n_units ? (n_units - rl + rpc - 1) / rpc : 0;
    if (nr > 0) {
      constexpr int LPG = G / 8;
      const int Gc = xsi.Gc;
      uint4 v[kFusedRowsPerGroup];
      uint32_t mx[kFusedRowsPerGroup];
#pragma unroll
      for (int m = 0; m < kFusedRowsPerGroup; ++m) {
        v[m] = make_uint4(0u, 0u, 0u, 0u);
        mx[m] = 0u;
        if (m < nr) {
          const int row = unit_row(rl + m * rpc);
          mx[m] = __ldcg(p.amax + row);
          if (tr < slices) v[m] = __ldcg(reinterpret_cast<const uint4 *>(p.act + static_cast<size_t>(row) * I) + tr);
        }
      }
#pragma unroll
      for (int m = 0; m < kFusedRowsPerGroup; ++m) {
        if (m >= nr) break;  // uniform over the group
        const uint32_t x = mx[m];
        const int q = rl + m * rpc;
        uint16_t *limbs = reinterpret_cast<uint16_t *>(al + static_cast<size_t>(q) * xsi.Xrow);
        float *meta = reinterpret_cast<float *>(am + static_cast<size_t>(q) * xsi.Mp);
        int E = 0;
        if (x != 0) E = (x >> 7) ? static_cast<int>(x >> 7) - 127 : (31 - __clz(static_cast<int>(x))) - 133;
        int sx = 0;
        if (tr < slices) {
          const uint32_t w[4] = {v[m].x, v[m].y, v[m].z, v[m].w};
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
          const int g = (8 * tr) / G;
          const int within = (8 * tr) - g * G;
          uint16_t *dst = limbs + static_cast<size_t>(g) * 2 * G + within;
          *reinterpret_cast<uint4 *>(dst) = make_uint4(half_pair(l0[0], l0[4]), half_pair(l0[1], l0[5]),
                                                       half_pair(l0[2], l0[6]), half_pair(l0[3], l0[7]));
          *reinterpret_cast<uint4 *>(dst + G) = make_uint4(half_pair(l1[0], l1[4]), half_pair(l1[1], l1[5]),
                                                           half_pair(l1[2], l1[6]), half_pair(l1[3], l1[7]));
        }
#pragma unroll
        for (int off = 1; off < LPG; off <<= 1) sx += __shfl_xor_sync(0xFFFFFFFFu, sx, off);
        if (tr < slices && (lane & (LPG - 1)) == 0) meta[(8 * tr) / G] = __int2float_rn(sx);
        if (tr == 0) {
          const int ai = meta_a_index(Gc);
          for (int g = Gc; g < ai; ++g) meta[g] = 0.0f;
          const int kk = E - 22;
          const int ka = max(kk, -126);
          meta[ai] = __int_as_float((ka + 127) << 23);
          meta[ai + 1] = __int_as_float((kk - ka + 127) << 23);
          meta[ai + 2] = 0.0f;
          meta[ai + 3] = 0.0f;
        }
      }
    }
    __syncthreads();
  }
  int t = 0;
  for (int dg = cta; dg < n_dg; dg += NB, ++t) {
    if (t > 0) {
      __syncthreads();  // the stage is free again
      if (warp == 1) issue_down(dg, n_units);
      __syncthreads();
    }
    if (!mbar_wait_bounded(&s_bar[p.nslot], t & 1, err)) s_dead = 1;
    __syncthreads();
    if (s_dead) {
      drain();
      return;
    }
    const int units = n_units * nblk_i;
    for (int u = warp; u < units; u += kFusedWarps) {
      const int q = u / nblk_i, b = u - q * nblk_i;
      const uint32_t xb = smem_u32(al + static_cast<size_t>(q) * xsi.Xrow) + (r & 1) * (G * 2) + c * 16;
      block_sums<G>(smem_u32(dstage + static_cast<size_t>(q) * dn_item + static_cast<size_t>(b) * kTileChunk), xb,
                    b, xsi.Gc, r, c);
    }
    __syncthreads();
    if (tid < n_units * 16) {
      const int q = tid >> 4, mrow = tid & 15;
      const float *mq = reinterpret_cast<const float *>(am + static_cast<size_t>(q) * xsi.Mp);
      const float acc = fold_row<G>(dstage + static_cast<size_t>(q) * dn_item, nblk_i, xsi.Gc, mrow, mq);
      const float2 ab = *reinterpret_cast<const float2 *>(mq + xsi.a_off / 4);
      dsm[q * 16 + mrow] = round_bf16(__fmul_rn(__fmul_rn(acc, ab.x), ab.y));
    }
    __syncthreads();
    if (tid < 16) {
      // slot-ordered float32 combine (no fused multiply-add), then the gated
      // shared expert: k_combine's kCombineParts arithmetic
      const int q0 = has_sh ? 1 : 0;
      float acc = 0.0f;
      for (int s = 0; s < keep; ++s) acc = __fadd_rn(acc, __fmul_rn(dsm[(q0 + s) * 16 + tid], s_score[s]));
      const float routed = round_bf16(acc);
      const float res = has_sh ? __fadd_rn(routed, bmul(dsm[tid], s_sg)) : routed;
      p.out[dg * 16 + tid] = f32_to_bf16(res);
    }
  }
}

// Bytes of dynamic shared memory and the carve of k_decode_layer for these
// sizes on `sms` CTAs; false when the fused kernel does not apply.
inline bool fused_layer_geometry(FusedLayer &p, int sms, int G, size_t limit, size_t *smem) {
  const int H = p.H, I = p.I, E = p.E, k = p.k;
  if (k < 1 || k > kCombineMaxSlots || E < k || E > 1024 || H % 256 || H > 4096 || I % 16 || I > 1024)
    return false;
  const int units = k + (p.wsg ? 1 : 0);
  const int n_rg = I / 8;
  const int nblk_h = (H / 2 + kBlkBytes - 1) / kBlkBytes;
  const int nblk_i = (I / 2 + kBlkBytes - 1) / kBlkBytes;
  const size_t gu_item = static_cast<size_t>(nblk_h) * kTileChunk;
  const size_t dn_item = static_cast<size_t>(nblk_i) * kTileChunk;
  const XStage xsh = xstage_geom(H, G), xsi = xstage_geom(I, G);
  const int nslot = (units * n_rg + sms - 1) / sms;
  if (nslot > kFusedMaxSlots || E + 1 > 4 * sms) return false;
  auto up = [](size_t v) { return (v + 127) & ~static_cast<size_t>(127); };
  size_t off = 0;
  p.off_x = static_cast<int>(off);
  off = up(off + static_cast<size_t>(H) * 2);
  p.off_xq = static_cast<int>(off);  // x's router fixed point (int32)
  off = up(off + static_cast<size_t>(H) * 4);
  p.off_xl = static_cast<int>(off);
  off = up(off + static_cast<size_t>(xsh.Xrow));
  p.off_xm = static_cast<int>(off);
  off = up(off + static_cast<size_t>(xsh.Mp));
  p.off_soft = static_cast<int>(off);
  off = up(off + (static_cast<size_t>((E + 31) & ~31) + 16 * kCombineMaxSlots) * 4);
  p.off_d = static_cast<int>(off);
  off = up(off + static_cast<size_t>(units) * 16 * 4);
  p.off_ring = static_cast<int>(off);
  const size_t ring = static_cast<size_t>(nslot) * gu_item;
  const size_t tail = up(static_cast<size_t>(units) * dn_item) + up(static_cast<size_t>(units) * xsi.Xrow) +
                      up(static_cast<size_t>(units) * xsi.Mp);
  size_t total;
  if (off + ring + tail <= limit) {
    p.alias = 0;
    size_t o = off + up(ring);
    p.off_down = static_cast<int>(o);
    o = up(o + static_cast<size_t>(units) * dn_item);
    p.off_al = static_cast<int>(o);
    o = up(o + static_cast<size_t>(units) * xsi.Xrow);
    p.off_am = static_cast<int>(o);
    total = o + static_cast<size_t>(units) * xsi.Mp;
  } else {
    p.alias = 1;
    size_t o = off;
    p.off_down = static_cast<int>(o);
    o = up(o + static_cast<size_t>(units) * dn_item);
    p.off_al = static_cast<int>(o);
    o = up(o + static_cast<size_t>(units) * xsi.Xrow);
    p.off_am = static_cast<int>(o);
    total = std::max(o + static_cast<size_t>(units) * xsi.Mp, off + ring);
  }
  if (total > limit) return false;
  p.nslot = nslot;
  *smem = total;
  return true;
}

// Grid-barrier counters of k_decode_layer: library-owned (zero at module
// load), one per workspace pointer that has run the kernel.  A workspace is
// never used by two overlapping calls, so neither is its counter.
constexpr int kGridBarSlots = 4096;
__device__ uint32_t g_grid_bar[kGridBarSlots];

namespace {
std::mutex g_bar_mutex;
std::map<std::pair<int, uintptr_t>, int> g_bar_slot;  // (device, workspace) -> slot
int g_bar_next[64] = {0};
}  // namespace

// Counter of the workspace `key` on the current device; slots are handed
// out round robin (the oldest binding is dropped when they run out).
cudaError_t grid_barrier_slot(const void *key, uint32_t **bar) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void *base = nullptr;
  e = cudaGetSymbolAddress(&base, g_grid_bar);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_bar_mutex);
  const auto k = std::make_pair(dev, reinterpret_cast<uintptr_t>(key));
  auto it = g_bar_slot.find(k);
  int slot;
  if (it != g_bar_slot.end()) {
    slot = it->second;
  } else {
    slot = g_bar_next[dev & 63]++ % kGridBarSlots;
    for (auto jt = g_bar_slot.begin(); jt != g_bar_slot.end(); ++jt)
      if (jt->first.first == dev && jt->second == slot) {
        g_bar_slot.erase(jt);
        break;
      }
    g_bar_slot[k] = slot;
  }
  *bar = static_cast<uint32_t *>(base) + slot;
  return cudaSuccess;
}

// After a bounded wait gave up, a counter may be left mid-barrier: zero them
// all (the caller has synchronised the device) and forget the bindings.
cudaError_t reset_grid_barriers() {
  void *base = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&base, g_grid_bar);
  if (e != cudaSuccess) return e;
  e = cudaMemset(base, 0, sizeof(uint32_t) * kGridBarSlots);
  std::lock_guard<std::mutex> lock(g_bar_mutex);
  g_bar_slot.clear();
  return e;
}

cudaError_t launch_decode_layer(FusedLayer p, int G, cudaStream_t s) {
  if (G != 32 && G != 64) return cudaErrorNotSupported;
  if (p.tiled.gate_up == nullptr || p.tiled.down == nullptr) return cudaErrorNotSupported;
  if ((p.wsg != nullptr) != (p.tiled.has_shared != 0)) return cudaErrorNotSupported;
  const DeviceInfo di = device_info();
  size_t smem = 0;
  constexpr size_t kLimit = 227 * 1024 - 2048;  // static shared memory of the kernel stays below 2 KB
  if (!fused_layer_geometry(p, di.sms, G, kLimit, &smem)) return cudaErrorNotSupported;
  auto kernel = G == 32 ? k_decode_layer<32> : k_decode_layer<64>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kFusedThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorNotSupported;
  // cooperative: the launch fails instead of starting fewer CTAs than the
  // grid barriers wait for
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(di.sms);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kernel, p, device_error_word());
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
