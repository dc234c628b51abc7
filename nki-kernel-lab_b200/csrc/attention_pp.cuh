// attention_pp.cuh - the single-query-tile flash kernel with two softmax warp groups that
// take alternate key tiles ("ping-pong"). Included by attention.cu after the shared
// definitions (work units, plans, TMEM helpers); same parameters, work plan, split-KV
// partial layout and combine kernel as attn_fwd_bf16_kernel.
//
// Reference numerics (nkilab/kernels/attention.py:204-246): the running row max is updated
// on every key tile, m(G) = max(m(G-1), rowmax(S(G))), and P(G) = exp(scale*S(G) - m(G)) is
// rounded to bf16 against it before P.V; O and l are multiplied by exp(m_old - m_new).
//
//   warps 0-3  softmax group 0: key tiles with even global tile count G (S buffer 0, O
//              accumulator 0). Warp w owns TMEM lane quadrant w: one thread per query row,
//              all 128 keys of the row
//   warps 4-7  softmax group 1: odd G (S buffer 1, O accumulator 1)
//   warp 8     TMA producer of Q (one buffer per unit) and K (2-deep ring)
//   warp 9     TMEM allocator + single-thread MMA issuer
//   warp 10    TMA producer of V (3-deep ring)
//   warp 11    idle (fills the third warp group for the register split)
//   TMEM       S 0 [0,128), S 1 [128,256), O_0 [256, 256+D), O_1 [256+D, 256+2D)
//   smem       Q, K ring, V ring, P (bf16, the K-major 128-byte-swizzled layout of the A
//              operand, written by the group of the tile once the previous tile's P.V has
//              read it; it also stages the output tile)
//
// A group loads S(G) from TMEM and releases the buffer at once, so S(G+2) = Q K(G+2)^T is
// computed while the group exponentiates; P goes to shared memory and P.V reads it from
// there. The MMA warp issues S(G+3) ahead of P(G).V(G), the order in which the groups
// release and fill their buffers. The group of tile G takes m(G-1) from the other group
// through shared memory (an mbarrier per direction and lane quadrant) once that group's
// exponentials are done, so the two groups' exp2 phases on the MUFU pipe alternate instead
// of overlapping. Each O_b holds its group's tiles against the group's latest max and is
// multiplied by exp(m_prev - m(G)) before P(G).V(G) adds to it, once P(G-1).V(G-1) (which
// read the P buffer, and follows the group's own previous P.V) has completed. The V ring is
// three deep: a V tile can only be loaded once the P.V two tiles back has completed, and
// loads land about a microsecond after they are issued while the tensor core runs. The epilogue adds the two accumulators, each scaled to the unit's final
// max: products summed in another fp32 order than the reference's single accumulator,
// every P rounding the reference's.

// 384 threads. The register file is split by setmaxnreg: launched at 168 per thread
// (384 x 168 = 64512), the softmax warps take 224 and the third warp group (producers,
// MMA, idle) drops to 56: 256 x 224 + 128 x 56 = 64512. One thread holds a 128-score row.
constexpr int kPPThreads = 384;
constexpr int kPPVProducerWarp = 10;
__device__ __forceinline__ void pp_regs_softmax() { asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory"); }
__device__ __forceinline__ void pp_regs_other() { asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory"); }

template <int D>
struct PPSmem {
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kPBytes = kTile * kTile * 2;
  uint8_t q[kTileBytes];     // Q of the current unit
  uint8_t k[2][kTileBytes];  // key ring, K-major
  uint8_t v[3][kTileBytes];  // value ring, N-major for P.V
  uint8_t p[kPBytes];        // P: [2 x 64 keys][128 rows][128 B], swizzled; also output staging
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[3], v_empty[3];
  uint64_t s_full[2];  // S(G) in TMEM buffer G & 1
  uint64_t s_free[2];  // the group has loaded S(G) (128 threads)
  uint64_t p_full[2];  // P(G) in shared memory and O corrected (128 threads)
  uint64_t pv_step;    // one phase per P.V (it has read P)
  uint64_t pv_done;    // one phase per unit: its last P.V complete
  uint64_t o_free;     // both accumulators read (all 256 softmax threads)
  uint64_t mma_done;
  uint64_t hand[2][4];  // [publishing group][lane quadrant]: m published (32 lanes)
  uint64_t ep[4];       // per lane quadrant: both groups' (max, sum) written (64 lanes)
  uint64_t stg[4];      // per lane quadrant: both halves of the output rows staged (64 lanes)
  uint64_t stg_read[4];  // per lane quadrant: its staged rows have been read by the TMA store
  float mh[kTile];      // running max after the latest tile, handed to the other group
  float xm[2][kTile];   // [group][row]: the group's final max of the unit (-inf: no tile)
  float xl[2][kTile];   // [group][row]: its row sum against that max
  uint32_t tmem_base;
  int abort;
};

// Wait by every lane (each with acquire semantics on the data the arriving threads
// published), then agree across the warp so it stays converged for the tcgen05 .sync.aligned
// instructions that follow.
__device__ __forceinline__ bool lanes_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  const bool ok = mbar_wait(bar, parity, abort, &g_attn_dev_error, code);
  return __all_sync(0xffffffffu, ok);
}

// max128 (four max3 chains over a 128-score row): attention_pair.cuh.

// P = 2^(s * scale_log2 - m) for the 128 scores in v, packed as bf16 pairs into v[0..64)
// (pair (c, c+1) lands in v[c/2], a score already consumed); returns the fp32 row sum.
__device__ __forceinline__ float exp_pack128(uint32_t* v, float scale_log2, float neg_m) {
  f32x2 rs[2];  // four fp32 chains: (even pairs, odd pairs) x (even scores, odd scores)
  exp_pack<128, 2>(v, scale_log2, neg_m, rs);
  return (f2_lo(rs[0]) + f2_lo(rs[1])) + (f2_hi(rs[0]) + f2_hi(rs[1]));
}

// Drain helper for the producers' abort path: wait (bounded) for an armed load to land.
__device__ __forceinline__ void pp_drain(uint64_t* bar, int armed, uint64_t t0) {
  if (armed >= 0)
    while (!mbar_try_wait(bar, (uint32_t)armed) && globaltimer() - t0 < kWaitTimeoutNs) {}
}

template <int D>
__global__ void __launch_bounds__(kPPThreads, 1)
attn_fwd_pp_bf16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                        const __grid_constant__ AttnArgs args, const __grid_constant__ PeerOut peers) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicCAS(&g_attn_dev_error, 0u, 40u);
    return;
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  auto& s = *reinterpret_cast<PPSmem<D>*>(smem_raw);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kOCol0 = 2 * kTile;  // O_0 at [256, 256+D), O_1 at [256+D, 256+2D)
  constexpr uint32_t kIdescS = idesc_bf16_f32(kTile, kTile, false, false);
  constexpr uint32_t kIdescPV = idesc_bf16_f32(kTile, D, false, true);
  constexpr uint32_t kTileBytes = kTile * D * 2;
  constexpr int kSub = D / 64;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float scale_log2 = args.scale_log2;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_free[i], kEngineThreads / 2);
      mbar_init(&s.p_full[i], kEngineThreads / 2);
      for (int q = 0; q < 4; ++q) mbar_init(&s.hand[i][q], 32);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    mbar_init(&s.pv_step, 1);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&s.ep[q], 64);
      mbar_init(&s.stg[q], 64);
      mbar_init(&s.stg_read[q], 1);
    }
    mbar_init(&s.pv_done, 1);
    mbar_init(&s.o_free, kEngineThreads);
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_o);
  }
  if (warp == kMmaWarp) tmem_alloc(&s.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // Programmatic dependent launch: nothing in global memory is touched before the previous
  // kernel of the stream has completed; the producer only asks L2 to prefetch the first
  // unit's tiles (a prefetch warms L2, the point of coherence, so it is safe while that
  // kernel still writes them).
  if (warp == kProducerWarp && elect_one()) {
    UnitRun u0;
    if (next_unit(args, 0, u0)) {
      for (int c = 0; c < kSub; ++c) {
        tma_prefetch_3d(&map_q, c * 64, u0.qt * kTile, u0.head);
        tma_prefetch_3d(&map_k, c * 64, u0.j0 * kTile, u0.kv_head);
        tma_prefetch_3d(&map_v, c * 64, u0.j0 * kTile, u0.kv_head);
        if (u0.n > 1) tma_prefetch_3d(&map_k, c * 64, (u0.j0 + 1) * kTile, u0.kv_head);
      }
    }
  }
  __syncwarp();
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == kProducerWarp) {
    pp_regs_other();
    // ------------------------------------------------ Q and K producer
    if (elect_one()) {
      uint32_t kc = 0, qc = 0;
      int k_armed[2] = {-1, -1}, q_armed = -1;
      bool ok = true;
      auto load_k = [&](int kt, int kvh) -> bool {
        const int ks = kc & 1;
        if (!mbar_wait(&s.k_empty[ks], ((kc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 11)) return false;
        mbar_arrive_expect_tx(&s.k_full[ks], kTileBytes);
        k_armed[ks] = (int)((kc >> 1) & 1u);
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.k[ks] + c * (kTile * 128), &map_k, &s.k_full[ks], c * 64, kt * kTile, kvh);
        ++kc;
        return true;
      };
      UnitRun un;
      for (int i = 0; ok && next_unit(args, i, un); ++i) {
        ok = load_k(un.j0, un.kv_head);
        // Q: its buffer is free once the previous unit's last S has been computed
        if (ok && !mbar_wait(&s.q_empty, (qc & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 10)) ok = false;
        if (ok) {
          mbar_arrive_expect_tx(&s.q_full, kTileBytes);
          q_armed = (int)(qc & 1u);
          for (int c = 0; c < kSub; ++c)
            tma_load_3d(s.q + c * (kTile * 128), &map_q, &s.q_full, c * 64, un.qt * kTile, un.head);
          ++qc;
        }
        for (int t = 1; ok && t < un.n; ++t) ok = load_k(un.j0 + t, un.kv_head);
      }
      if (!ok) {  // let issued copies land before shared memory is released
        const uint64_t t0 = globaltimer();
        pp_drain(&s.q_full, q_armed, t0);
        for (int b = 0; b < 2; ++b) pp_drain(&s.k_full[b], k_armed[b], t0);
      }
    }
    __syncwarp();
  } else if (warp == kPPVProducerWarp) {
    pp_regs_other();
    // ------------------------------------------------ V producer
    if (elect_one()) {
      uint32_t vc = 0;
      int v_armed[3] = {-1, -1, -1};
      bool ok = true;
      UnitRun un;
      for (int i = 0; ok && next_unit(args, i, un); ++i) {
        for (int t = 0; t < un.n; ++t) {
          const int vs = (int)(vc % 3);
          const uint32_t vph = (vc / 3) & 1u;
          if (!mbar_wait(&s.v_empty[vs], vph ^ 1u, &s.abort, &g_attn_dev_error, 12)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.v_full[vs], kTileBytes);
          v_armed[vs] = (int)vph;
          for (int c = 0; c < kSub; ++c)
            tma_load_3d(s.v[vs] + c * (kTile * 128), &map_v, &s.v_full[vs], c * 64, (un.j0 + t) * kTile, un.kv_head);
          ++vc;
        }
      }
      if (!ok) {
        const uint64_t t0 = globaltimer();
        for (int b = 0; b < 3; ++b) pp_drain(&s.v_full[b], v_armed[b], t0);
      }
    }
    __syncwarp();
  } else if (warp > kMmaWarp) {
    pp_regs_other();  // idle warp of the third warp group
  } else if (warp == kMmaWarp) {
    pp_regs_other();
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint64_t q_desc = smem_desc_sw128(smem_u32(s.q), 16, 1024);
      const uint64_t k_desc0 = smem_desc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t k_desc1 = smem_desc_sw128(smem_u32(s.k[1]), 16, 1024);
      const uint64_t v_desc0 = smem_desc_sw128(smem_u32(s.v[0]), kTile * 128, 1024);
      const uint64_t p_desc = smem_desc_sw128(smem_u32(s.p), 16, 1024);
      constexpr uint32_t kVSlot = (uint32_t)(kTileBytes >> 4);  // descriptor address step per V slot
      bool ok = true;
      // S cursor: the next score tile to compute (global tile gs, tile ts of unit us)
      UnitRun us;
      int is = 0, ts = 0;
      bool s_more = next_unit(args, 0, us);
      uint32_t gs = 0, kc = 0, qc = 0;
      // P.V cursor: the next P.V (global tile gp, tile tp of unit up)
      UnitRun up;
      int ip = 0, tp = 0;
      bool p_more = next_unit(args, 0, up);
      uint32_t gp = 0, vc = 0, uc = 0;
      auto issue_s = [&]() -> bool {
        const int b = gs & 1;
        if (ts == 0 && !mbar_wait(&s.q_full, qc & 1u, &s.abort, &g_attn_dev_error, 20)) return false;
        if (gs >= 2 && !mbar_wait(&s.s_free[b], ((gs - 2) >> 1) & 1u, &s.abort, &g_attn_dev_error, 26)) return false;
        if (!mbar_wait(&s.k_full[kc & 1], (kc >> 1) & 1u, &s.abort, &g_attn_dev_error, 21)) return false;
        tc_fence_after();
        const uint64_t kd = (kc & 1) ? k_desc1 : k_desc0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4);
          mma_bf16_ss(tmem + (uint32_t)(b * kTile), q_desc + off, kd + off, kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full[b]);
        mma_commit(&s.k_empty[kc & 1]);
        ++kc;
        ++gs;
        if (++ts == us.n) {  // the unit's last S: its Q buffer is free once that has completed
          mma_commit(&s.q_empty);
          ++qc;
          ts = 0;
          s_more = next_unit(args, ++is, us);
        }
        return true;
      };
      auto issue_pv = [&]() -> bool {
        const int b = gp & 1;
        const uint32_t vs = vc % 3;
        if (!mbar_wait(&s.v_full[vs], (vc / 3) & 1u, &s.abort, &g_attn_dev_error, 24)) return false;
        // the first P.V of a unit overwrites an accumulator the previous epilogue reads
        if (tp == 0 && !mbar_wait(&s.o_free, (uc & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 23)) return false;
        if (!mbar_wait(&s.p_full[b], (gp >> 1) & 1u, &s.abort, &g_attn_dev_error, 22)) return false;
        tc_fence_after();
        const uint64_t vd = v_desc0 + vs * kVSlot;
        // a group's first tile of the unit overwrites its accumulator
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4);
          mma_bf16_ss(tmem + kOCol0 + (uint32_t)(b * D), p_desc + off, vd + (uint32_t)(kk * 128), kIdescPV,
                      (tp >= 2 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&s.v_empty[vs]);
        mma_commit(&s.pv_step);
        ++vc;
        ++gp;
        if (++tp == up.n) {
          mma_commit(&s.pv_done);
          ++uc;
          tp = 0;
          p_more = next_unit(args, ++ip, up);
        }
        return true;
      };
      // S(G+3) ahead of P(G).V(G): a group releases its S buffer early in its tile and
      // fills its P buffer at the end, so the buffers free up in this order. An S whose
      // buffer is released by a tile of a later unit than P.V's waits for that P.V: the
      // group reaches that tile only after the epilogue of P.V's unit.
      while (ok && p_more) {
        const uint32_t gp_end = gp - (uint32_t)tp + (uint32_t)up.n;  // first tile after P.V's unit
        while (ok && s_more && gs <= gp + 3 && (gs < 2 || gs - 2 < gp_end)) ok = issue_s();
        if (ok) ok = issue_pv();
      }
      mma_commit(&s.mma_done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
    }
    __syncwarp();
  } else {
    pp_regs_softmax();
    // ------------------------------------------------ softmax groups (warps 0-7)
    const int qd = warp & 3;
    const int grp = warp >> 2;
    const int r = qd * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + (uint32_t)(grp * kTile);
    const uint32_t o_own = tmem + lane_off + kOCol0 + (uint32_t)(grp * D);
    const uint32_t o_half = tmem + lane_off + kOCol0 + (uint32_t)(grp * (D / 2));  // + b * D: accumulator b
    const int sw = r & 7;
    uint8_t* p_row = s.p + r * 128;  // this row of P (+ 64-key half * 16 KB)
    const bool quad_lead = grp == 0 && lane == 0;  // stores its quadrant's output rows
    bool stored_any = false;
    uint32_t gt = 0, uc = 0, ncons = 0, nstaged = 0;  // nstaged: units stored from shared memory
    bool staged_rows = false;  // group 1: the last unit's rows of this quadrant were staged in P
    // A group-1 warp writes this quadrant's rows of P (scores or output staging) only after
    // the TMA store has read the rows staged there at the end of the previous stored unit
    // (group 0's warp of the quadrant issues that store and waits for it itself).
    auto wait_staged = [&]() -> bool {
      if (!staged_rows) return true;
      staged_rows = false;
      return lanes_wait(&s.stg_read[qd], (nstaged - 1u) & 1u, &s.abort, 38);
    };
    bool ok = true;
    UnitRun un;
    for (int i = 0; ok && next_unit(args, i, un); ++i) {
      const int u = un.u;
      const int qt = un.qt;
      float m_own = -INFINITY, l_own = 0.f;  // the group's latest max (log2 domain), row sum against it
      bool any = false;                      // the group has had a tile of this unit
      for (int t = 0; t < un.n; ++t) {
        const uint32_t G = gt + (uint32_t)t;
        if ((int)(G & 1u) != grp) continue;
        if (!warp_wait(&s.s_full[grp], (G >> 1) & 1u, &s.abort, 31)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
        tmem_wait_ld();
        reg_fence<128>(v);
        tc_fence_before();
        mbar_arrive(&s.s_free[grp]);  // S(G+2) may be computed into this buffer
        if (un.j0 + t == qt) {  // diagonal tile: keys above the diagonal are masked
          // The row index goes through an opaque move on every diagonal tile: otherwise the
          // compiler hoists the 128 loop-invariant comparisons out of the tile loop and keeps
          // their results live across it, spilling the score row.
          int lim;
          asm volatile("mov.b32 %0, %1;" : "=r"(lim) : "r"(r));
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > lim) v[c] = 0xff800000u;  // -inf
        }
        float mx = max128(v) * scale_log2;  // key 0 of a unit's first tile is never masked: finite
        if (t > 0) {  // m(G-1) from the other group
          if (!lanes_wait(&s.hand[grp ^ 1][qd], ncons & 1u, &s.abort, 34)) { ok = false; break; }
          ++ncons;
          mx = fmaxf(mx, s.mh[r]);
        }
        float factor = 1.f;
        if (any && mx > m_own) factor = fast_exp2(m_own - mx);
        m_own = mx;
        const float rs = exp_pack128(v, scale_log2, -mx);
        // m(G) for the other group's tile G+1, handed over once this group's exponentials
        // are done: the other group's exp phase then follows this one instead of sharing
        // the MUFU pipe with it
        if (t + 1 < un.n) {
          s.mh[r] = mx;
          mbar_arrive(&s.hand[grp][qd]);
        }
        // P is free (and O_grp holds the group's previous tiles) once P(G-1).V(G-1) has
        // completed
        if (G >= 1 && !lanes_wait(&s.pv_step, (G - 1u) & 1u, &s.abort, 37)) { ok = false; break; }
        if (!wait_staged()) { ok = false; break; }
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int g = 0; g < 8; ++g)
            *reinterpret_cast<uint4*>(p_row + c * (kTile * 128) + ((g ^ sw) * 16)) =
                make_uint4(v[c * 32 + g * 4], v[c * 32 + g * 4 + 1], v[c * 32 + g * 4 + 2], v[c * 32 + g * 4 + 3]);
        fence_proxy_async_smem();  // P is read by the tensor core (async proxy)
        if (any && __any_sync(0xffffffffu, factor != 1.f)) {
          // O_own *= factor before P(G).V(G) accumulates into it, 64 columns per TMEM
          // round trip in the registers the packing freed.
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            tmem_ld32(o_own + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[64]));
            tmem_ld32(o_own + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[96]));
            tmem_wait_ld();
            reg_fence<64>(v + 64);
#pragma unroll
            for (int k2 = 64; k2 < 128; k2 += 2) {  // two columns per mul.rn.f32x2
              const f32x2 o2 = f2_mul(f2_pack_bits(v[k2], v[k2 + 1]), f2_pack(factor, factor));
              v[k2] = (uint32_t)o2;
              v[k2 + 1] = (uint32_t)(o2 >> 32);
            }
            tmem_st32(o_own + c * 64, v + 64);
            tmem_st32(o_own + c * 64 + 32, v + 96);
            tmem_wait_st();  // before the registers take the next columns
          }
          tc_fence_before();
        }
        mbar_arrive(&s.p_full[grp]);
        l_own = l_own * factor + rs;
        any = true;
      }
      if (!ok) break;
      // ---------------- epilogue: O = (O_0 * f_0 + O_1 * f_1) / l, each group half the columns
      s.xm[grp][r] = any ? m_own : -INFINITY;
      s.xl[grp][r] = l_own;
      mbar_arrive(&s.ep[qd]);
      if (!warp_wait(&s.pv_done, uc & 1u, &s.abort, 33)) { ok = false; break; }
      if (!lanes_wait(&s.ep[qd], uc & 1u, &s.abort, 35)) { ok = false; break; }
      tc_fence_after();
      const bool has0 = un.n >= 2 || (gt & 1u) == 0u;  // group 0 had a tile of this unit
      const bool has1 = un.n >= 2 || (gt & 1u) == 1u;
      const float m0 = s.xm[0][r], m1 = s.xm[1][r];
      const float mf = fmaxf(m0, m1);
      const float f0 = has0 ? fast_exp2(m0 - mf) : 0.f;
      const float f1 = has1 ? fast_exp2(m1 - mf) : 0.f;
      const float lt = (has0 ? s.xl[0][r] * f0 : 0.f) + (has1 ? s.xl[1][r] * f1 : 0.f);
      const float linv = 1.0f / lt;
      const float g0 = f0 * linv, g1 = f1 * linv;
      uint32_t w[D / 2];  // this group's half of the output columns
      {
        // both accumulators are loaded; one that had no tile of this unit holds stale
        // values, which the selects below drop
        uint32_t a0[D / 2], a1[D / 2];
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tmem_ld32(o_half + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&a0[c * 32]));
          tmem_ld32(o_half + (uint32_t)D + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&a1[c * 32]));
        }
        tmem_wait_ld();
        reg_fence<D / 2>(a0);
        reg_fence<D / 2>(a1);
#pragma unroll
        for (int k2 = 0; k2 < D / 2; ++k2) {
          const float x0 = has0 ? __uint_as_float(a0[k2]) * g0 : 0.f;
          const float x1 = has1 ? __uint_as_float(a1[k2]) * g1 : 0.f;
          w[k2] = __float_as_uint(x0 + x1);
        }
      }
      tc_fence_before();
      mbar_arrive(&s.o_free);  // the next unit's first P.V may overwrite the accumulators
      if (un.split) {
        // Split query tile: this chunk's O / sum in fp32 and its (max, sum); the combine
        // kernel merges the chunks once this kernel has completed.
        float4* op = reinterpret_cast<float4*>(args.ws + args.ws_o_off) + (size_t)u * (kTile * D / 4) + r;
#pragma unroll
        for (int g4 = 0; g4 < D / 8; ++g4)  // layout [col/4][row][4]: a warp stores 512 contiguous bytes
          op[(size_t)(grp * (D / 8) + g4) * kTile] =
              make_float4(__uint_as_float(w[4 * g4]), __uint_as_float(w[4 * g4 + 1]), __uint_as_float(w[4 * g4 + 2]),
                          __uint_as_float(w[4 * g4 + 3]));
        if (grp == 0) {
          float* st = reinterpret_cast<float*>(args.ws + args.ws_stats_off) + (size_t)u * 2 * kTile;
          st[r] = mf;
          st[kTile + r] = lt;
        }
      } else {
        // Stage the bf16 output rows in P (every P.V of the unit has completed; the next P
        // rows of this quadrant are written only after its store has read them) in the
        // 128-byte-swizzled layout of the output map; one TMA store per 64 columns.
        if (!wait_staged()) { ok = false; break; }
#pragma unroll
        for (int g2 = 0; g2 < D / 16; ++g2) {
          const int g = grp * (D / 16) + g2;  // 16-byte chunk of the output row
          float f[8];
#pragma unroll
          for (int k2 = 0; k2 < 8; ++k2) f[k2] = __uint_as_float(w[8 * g2 + k2]);
          uint8_t* rowp = s.p + (g / 8) * (kTile * 128) + r * 128;
          *reinterpret_cast<uint4*>(rowp + (((g & 7) ^ sw) * 16)) = pack16<bf16>(f);
        }
        fence_proxy_async_smem();
        mbar_arrive(&s.stg[qd]);
        const int row0 = qt * kTile + qd * 32;
        if (quad_lead) {
          // both warps of the quadrant have staged their halves of its 32 rows
          if (!mbar_wait(&s.stg[qd], nstaged & 1u, &s.abort, &g_attn_dev_error, 36)) ok = false;
          if (ok && row0 < args.seq) {
            const int oh = un.head + peers.head_offset;
#pragma unroll
            for (int c = 0; c < kSub; ++c)
              tma_store_3d(&map_o, s.p + c * (kTile * 128) + qd * 32 * 128, c * 64, row0, oh);
            for (int p = 0; p < peers.n; ++p)  // the same staged rows into every peer's buffer
#pragma unroll
              for (int c = 0; c < kSub; ++c)
                tma_store_3d(&peers.map[p], s.p + c * (kTile * 128) + qd * 32 * 128, c * 64, row0, oh);
            tma_store_commit();
            tma_store_wait_read();
            stored_any = true;
          }
          mbar_arrive(&s.stg_read[qd]);  // the quadrant's staged rows may be overwritten
        }
        ++nstaged;
        staged_rows = grp == 1;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      gt += (uint32_t)un.n;
      ++uc;
    }
    if (stored_any) tma_store_wait_all();  // every output store, local and remote, has completed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}
