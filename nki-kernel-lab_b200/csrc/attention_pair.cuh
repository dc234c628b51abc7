// attention_pair.cuh - the bf16 causal attention kernel with two query tiles per CTA.
// Included by attention.cu (it uses that file's helpers, combine kernel and constants).
//
// Reference: nkilab/kernels/attention.py:280-325 (flash_attention_pipelined, ILP = 2):
// two independent query tiles interleaved so one tile's tensor-core work fills the gaps
// while the other tile's online softmax runs. The reference's arithmetic, step for step
// (attention.py:204-246): fp32 scores, the running row max m updated on every key tile,
// P = exp(scale * s - m) rounded to bf16 relative to that running max, the correction
// exp(m_old - m_new) applied to l and to O whenever the max grows, O * (1/l) rounded once.
// The exponent is taken in the log2 domain (scale * log2(e) folded into one FMA before a
// hardware exp2).
//
// Work unit: (head, query-tile pair p = tiles A = 2p and B = 2p + 1, chunk [j0, j0 + n)
// of the pair's causal key range [0, 2p + 2)). Tile A uses key tiles j <= 2p, so it
// takes nA = min(n, 2p + 1 - j0) >= 1 of the chunk's tiles (the planner never makes a
// chunk holding only key tile 2p + 1); tile B takes all n. K and V tiles are loaded once
// for both query tiles.
//
// Warp roles (512 threads; register split by setmaxnreg, 2 x 168 + 2 x 88 per thread =
// the 128 x 512 the block launches with):
//   warps 0-3    softmax engine of tile A: thread r owns score row r (TMEM lane r), so
//                a row's max and sum need no exchange between threads
//   warps 4-7    softmax engine of tile B
//   warps 8-11   correction and epilogue of both tiles, in the MMA issuer's order: per key
//                tile, the new running max of every row (published by the engines) and,
//                where it grew, O rescaled in TMEM between P.V(j-1) and P.V(j), off the
//                engines' critical path; at a unit's end O from TMEM, * 1/l, bf16, staged
//                in the tile's Q buffer and TMA-stored per lane quadrant (or fp32
//                partials + (max, sum) to the workspace for a split pair)
//   warp 12      TMA producer: Q pair per unit (double buffered), K and V through one
//                3-deep ring in consumption order K(j0), V(j0), K(j0+1), V(j0+1), ...
//   warp 13      TMEM allocator + single-thread tcgen05.mma issuer, per key tile j:
//                P.V_A(j), S_A(j+1), P.V_B(j), S_B(j+1) -- while engine A exponentiates
//                tile j+1 the tensor core runs B's products, and the other way round
//   warps 14-15  idle
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [384,384+D); P
// (bf16 pairs) overwrites the first 64 columns of its S buffer and is read from there by
// the TS-form P.V product. Because one thread issues every MMA and they complete in issue
// order, the commit of S_T(j+1) also covers P.V_T(j): once an engine has seen S_T(j+1) and
// published its new row maxima, O_T already holds every earlier product and the
// correction warps may rescale it.

constexpr int kPairThreads = 512;
constexpr int kPairEpiWarp0 = 8;
constexpr int kPairProducerWarp = 12;
constexpr int kPairMmaWarp = 13;
constexpr int kPairRing = 3;
constexpr int kMaxPairSched = 1024;

template <int D>
struct PairSmem {
  static constexpr int kTileBytes = kTile * D * 2;
  uint8_t q[2][2][kTileBytes];      // [Q buffer][tile A/B]: D/64 sub-tiles of [128 rows x 128 B]; output staging
  uint8_t kv[kPairRing][kTileBytes];  // K (K-major) and V (N-major for P.V) tiles, in consumption order
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kPairRing], kv_empty[kPairRing];
  uint64_t s_full[2];      // per tile: S(j) in TMEM
  uint64_t p_full[2];      // per tile: P(j) written (all 128 engine threads)
  uint64_t o_ready[2];     // per tile: the unit's last P.V (and every MMA before it) complete
  uint64_t corr_full[2][4];  // per tile, lane quadrant and key step: new row maxima in row_m (its engine warp)
  uint64_t corr_done[2];   // per tile and key step: O corrected, previous O read (4 correction warps)
  uint64_t stats_full[2];  // per tile: row sums of the unit in row_l (4 engine warps)
  uint64_t mma_done;
  float row_m[2][kTile], row_l[2][kTile];
  uint32_t tmem_base;
  int abort;
};

template <int D>
constexpr size_t pair_smem_bytes() {
  return sizeof(PairSmem<D>);
}

struct PairArgs {
  unsigned char* ws;  // NULL when no pair is split
  int heads, pairs, kv_group, seq;
  float scale_log2;
  size_t ws_stats_off, ws_o_off;
  int n_ctas_listed;  // > 0: cta_off / unit give each CTA's units; 0: round-robin, no split
  int units;          // round-robin plans: number of units (heads * pairs)
  uint16_t cta_off[kMaxCtas + 1];
  // x = head | kv head << 16, y = pair | j0 << 16, z = n | chunks << 16, w = workspace slot
  // of tile A's partial (0xffffffff: the unit covers its pair's whole key range)
  uint4 unit[kMaxPairSched];
};

struct PairRun {
  int head, kv_head, p, j0, n, nA, n_e;
  uint32_t slot_a;  // 0xffffffff: not split
};

__device__ __forceinline__ bool pair_next_unit(const PairArgs& a, int i, PairRun& r) {
  if (a.n_ctas_listed > 0) {
    const int k = a.cta_off[blockIdx.x] + i;
    if (k >= a.cta_off[blockIdx.x + 1]) return false;
    const uint4 d = a.unit[k];
    r.head = (int)(d.x & 0xffffu);
    r.kv_head = (int)(d.x >> 16);
    r.p = (int)(d.y & 0xffffu);
    r.j0 = (int)(d.y >> 16);
    r.n = (int)(d.z & 0xffffu);
    r.n_e = (int)(d.z >> 16);
    r.slot_a = d.w;
  } else {
    const int u = (int)blockIdx.x + i * (int)gridDim.x;
    if (u >= a.units) return false;
    r.head = u % a.heads;
    r.kv_head = r.head / a.kv_group;
    r.p = a.pairs - 1 - u / a.heads;  // longest pairs first
    r.j0 = 0;
    r.n = 2 * r.p + 2;
    r.n_e = 1;
    r.slot_a = 0xffffffffu;
  }
  r.nA = min(r.n, 2 * r.p + 1 - r.j0);
  return true;
}

__device__ __forceinline__ void set_max_regs_inc168() { asm volatile("setmaxnreg.inc.sync.aligned.u32 168;\n" ::: "memory"); }
__device__ __forceinline__ void set_max_regs_dec88() { asm volatile("setmaxnreg.dec.sync.aligned.u32 88;\n" ::: "memory"); }

// Max of 128 fp32 scores held as bits.
__device__ __forceinline__ float max128(const uint32_t* v) {
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < 128; c += 8)
#pragma unroll
    for (int a = 0; a < 4; ++a) mx[a] = max3f(mx[a], __uint_as_float(v[c + 2 * a]), __uint_as_float(v[c + 2 * a + 1]));
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

template <int D>
__global__ void __launch_bounds__(kPairThreads, 1)
attn_fwd_pair_bf16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                          const __grid_constant__ PairArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicCAS(&g_attn_dev_error, 0u, 41u);
    return;
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the combine kernel may be scheduled
  auto& s = *reinterpret_cast<PairSmem<D>*>(smem_raw);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kIdescS = idesc_bf16_f32(kTile, kTile, false, false);
  constexpr uint32_t kIdescPV = idesc_bf16_f32(kTile, D, false, true);
  constexpr uint32_t kTileBytes = kTile * D * 2;
  constexpr int kSub = D / 64;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 8);  // 4 epilogue warps x 2 tiles
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], kTile);
      mbar_init(&s.o_ready[i], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&s.corr_full[i][q], 1);
      mbar_init(&s.corr_done[i], 4);
      mbar_init(&s.stats_full[i], 4);
    }
    for (int i = 0; i < kPairRing; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == kPairProducerWarp && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_o);
  }
  if (warp == kPairMmaWarp) tmem_alloc(&s.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // Programmatic dependent launch: nothing in global memory is touched before the
  // previous kernel of the stream has completed; the L2 prefetch of the first unit's
  // tiles only warms L2 (the point of coherence), so it is safe before the wait.
  if (warp == kPairProducerWarp && elect_one()) {
    PairRun u0;
    if (pair_next_unit(args, 0, u0)) {
      for (int c = 0; c < kSub; ++c) {
        tma_prefetch_3d(&map_q, c * 64, 2 * u0.p * kTile, u0.head);
        tma_prefetch_3d(&map_q, c * 64, (2 * u0.p + 1) * kTile, u0.head);
        tma_prefetch_3d(&map_k, c * 64, u0.j0 * kTile, u0.kv_head);
        tma_prefetch_3d(&map_v, c * 64, u0.j0 * kTile, u0.kv_head);
      }
    }
  }
  __syncwarp();
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp < kPairEpiWarp0) {
    set_max_regs_inc168();
    // ------------------------------------------------ softmax engines (warps 0-7)
    const int T = warp >> 2;   // 0: tile A, 1: tile B
    const int qd = warp & 3;   // TMEM lane quadrant
    const int r = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + (uint32_t)(T * kTile);
    const float scale_log2 = args.scale_log2;
    uint32_t sc = 0;  // key steps of this tile so far (s_full, corr_full, corr_done, p_full phases)
    bool ok = true;
    PairRun un;
    for (int i = 0; ok && pair_next_unit(args, i, un); ++i) {
      const int nT = T == 0 ? un.nA : un.n;
      const int diag = 2 * un.p + T;  // this tile's diagonal key tile
      float m = -INFINITY, l = 0.f;
      for (int t = 0; t < nT; ++t, ++sc) {
        if (!warp_wait(&s.s_full[T], sc & 1u, &s.abort, 51)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
        tmem_wait_ld();
        reg_fence<128>(v);
        if (un.j0 + t == diag) {  // diagonal tile: keys after the query are masked
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > r) v[c] = __float_as_uint(-INFINITY);
        }
        // running max (attention.py:224-227); key 0 of a unit's first tile is never
        // masked, so the max is finite from the first tile on
        const float mx = max128(v) * scale_log2;
        const float m_new = t == 0 ? mx : fmaxf(m, mx);
        const float factor = (t > 0 && m_new > m) ? fast_exp2(m - m_new) : 1.f;  // :232-233
        s.row_m[T][r] = m_new;  // for the correction warps (which compute the same factor)
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.corr_full[T][qd]);
        m = m_new;
        const float neg_m = -m;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int c = 0; c < 128; c += 2) {  // :228-231
          const float p0 = fast_exp2(fmaf(__uint_as_float(v[c]), scale_log2, neg_m));
          const float p1 = fast_exp2(fmaf(__uint_as_float(v[c + 1]), scale_log2, neg_m));
          rs0 += p0;
          rs1 += p1;
          __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
          v[c >> 1] = *reinterpret_cast<uint32_t*>(&h2);
        }
        tmem_st32(s_addr, v);            // P: keys 0..63 as bf16 pairs in columns 0..31
        tmem_st32(s_addr + 32, v + 32);  // keys 64..127 in columns 32..63
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s.p_full[T]);
        l = l * factor + (rs0 + rs1);  // :234-236
      }
      if (!ok) break;
      // The unit's row sums for the epilogue. The correction warps finish the previous
      // unit's epilogue (which reads row_l) before they handle this unit's first key
      // step, so waiting for their last step of this unit makes the single buffer safe.
      if (!warp_wait(&s.corr_done[T], (sc - 1) & 1u, &s.abort, 52)) { ok = false; break; }
      s.row_l[T][r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.stats_full[T]);
    }
  } else if (warp < kPairProducerWarp) {
    set_max_regs_dec88();
    // ------------------------------------------------ correction + epilogue (warps 8-11)
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const int sw = r & 7;
    uint32_t fc[2] = {0, 0};  // key steps per tile (corr_full / corr_done phases)
    float m_old[2] = {0.f, 0.f};
    bool ok = true;
    bool stored = false;
    // Epilogue of tile T of unit `pu` (the uc-th unit of this CTA): O / l -> output, or the
    // split chunk's fp32 partial and (max, sum). Frees the Q buffer (no staging) or lets the
    // producer refill it once the staged tile has been stored.
    auto epilogue = [&](int T, const PairRun& pu, uint32_t uc) -> bool {
      if (!warp_wait(&s.o_ready[T], uc & 1u, &s.abort, 53)) return false;
      if (!warp_wait(&s.stats_full[T], uc & 1u, &s.abort, 54)) return false;
      __syncwarp();  // orders the engine's row_l writes before every lane's reads
      tc_fence_after();
      const float lt = s.row_l[T][r];
      const float mr = T == 0 ? m_old[0] : m_old[1];
      const float linv = 1.0f / lt;  // attention.py:137-142
      const uint32_t o_addr = tmem + lane_off + (uint32_t)((2 + T) * kTile);
      const int qb = uc & 1;
      if (pu.slot_a != 0xffffffffu) {
        // this chunk's O / sum in fp32 (layout [col/4][row][4]) and its (max, sum)
        const uint32_t slot = pu.slot_a + (uint32_t)(T * pu.n_e * args.heads);
        float4* op = reinterpret_cast<float4*>(args.ws + args.ws_o_off) + (size_t)slot * (kTile * D / 4) + r;
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          uint32_t w[16];
          tmem_ld16(o_addr + c * 16, w);
          tmem_wait_ld();
          reg_fence<16>(w);
#pragma unroll
          for (int g = 0; g < 4; ++g)
            op[(size_t)(4 * c + g) * kTile] =
                make_float4(__uint_as_float(w[4 * g]) * linv, __uint_as_float(w[4 * g + 1]) * linv,
                            __uint_as_float(w[4 * g + 2]) * linv, __uint_as_float(w[4 * g + 3]) * linv);
        }
        float* st = reinterpret_cast<float*>(args.ws + args.ws_stats_off) + (size_t)slot * 2 * kTile;
        st[r] = mr;
        st[kTile + r] = lt;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.q_empty[qb]);  // no staging: the Q buffer is free once the MMAs are done
      } else {
        uint8_t* stage = s.q[qb][T];
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          uint32_t w[16];
          tmem_ld16(o_addr + c * 16, w);
          tmem_wait_ld();
          reg_fence<16>(w);
#pragma unroll
          for (int g2 = 0; g2 < 2; ++g2) {
            const int g = 2 * c + g2;  // 16-byte chunk of the output row
            float f[8];
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) f[k2] = __uint_as_float(w[8 * g2 + k2]) * linv;
            uint8_t* rowp = stage + (g / 8) * (kTile * 128) + r * 128;
            *reinterpret_cast<uint4*>(rowp + (((g & 7) ^ sw) * 16)) = pack16<bf16>(f);
          }
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int row0 = (2 * pu.p + T) * kTile + qd * 32;
#pragma unroll
          for (int c = 0; c < kSub; ++c)
            tma_store_3d(&map_o, stage + c * (kTile * 128) + qd * 32 * 128, c * 64, row0, pu.head);
          tma_store_commit();
          tma_store_wait_read();
          stored = true;
          mbar_arrive(&s.q_empty[qb]);
        }
        __syncwarp();
      }
      return true;
    };
    PairRun un, prev;
    uint32_t uc = 0;
    for (int i = 0; ok && pair_next_unit(args, i, un); ++i, ++uc) {
      for (int t = 0; ok && t < un.n; ++t) {
        for (int T = 0; T < 2; ++T) {
          if (t >= (T == 0 ? un.nA : un.n)) continue;
          // the previous unit's epilogue of this tile comes before this unit's first
          // step: P.V(0) of this unit overwrites O, and waits for corr_done(0)
          if (t == 0 && i > 0 && !epilogue(T, prev, uc - 1)) { ok = false; break; }
          if (!warp_wait(&s.corr_full[T][qd], fc[T] & 1u, &s.abort, 55)) { ok = false; break; }
          __syncwarp();
          const float m_new = s.row_m[T][r];
          const bool grow = t > 0 && m_new > m_old[T];
          if (__any_sync(0xffffffffu, grow)) {
            // O_T *= exp(m_old - m_new) (attention.py:243-245), between P.V(t-1) and P.V(t)
            tc_fence_after();
            const float factor = grow ? fast_exp2(m_old[T] - m_new) : 1.f;
            const uint32_t o_addr = tmem + lane_off + (uint32_t)((2 + T) * kTile);
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t w[32];
              tmem_ld32(o_addr + c * 32, w);
              tmem_wait_ld();
              reg_fence<32>(w);
#pragma unroll
              for (int k2 = 0; k2 < 32; ++k2) w[k2] = __float_as_uint(__uint_as_float(w[k2]) * factor);
              tmem_st32(o_addr + c * 32, w);
            }
            tmem_wait_st();
          }
          m_old[T] = m_new;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.corr_done[T]);
          ++fc[T];
        }
      }
      prev = un;
    }
    if (ok && uc > 0)
      for (int T = 0; T < 2 && ok; ++T) ok = epilogue(T, prev, uc - 1);
    if (stored) tma_store_wait_all();
  } else {
    set_max_regs_dec88();
    if (warp == kPairProducerWarp) {
      // ------------------------------------------------ TMA producer
      if (elect_one()) {
        uint32_t qc = 0, kc = 0;
        int q_armed[2] = {-1, -1};
        int kv_armed[kPairRing] = {-1, -1, -1};
        bool ok = true;
        auto load_kv = [&](const CUtensorMap* map, int kt, int kvh) -> bool {
          const int st = (int)(kc % kPairRing);
          const uint32_t ph = (kc / kPairRing) & 1u;
          if (!mbar_wait(&s.kv_empty[st], ph ^ 1u, &s.abort, &g_attn_dev_error, 61)) return false;
          mbar_arrive_expect_tx(&s.kv_full[st], kTileBytes);
          kv_armed[st] = (int)ph;
          for (int c = 0; c < kSub; ++c)
            tma_load_3d(s.kv[st] + c * (kTile * 128), map, &s.kv_full[st], c * 64, kt * kTile, kvh);
          ++kc;
          return true;
        };
        // Q of unit i + 1 is loaded while unit i streams its K and V: as soon as its
        // buffer (that of unit i - 1) has been released by the epilogue, checked before
        // every K/V load, and at the latest after unit i's last one.
        auto load_q = [&](const PairRun& u) {
          const int qb = qc & 1;
          mbar_arrive_expect_tx(&s.q_full[qb], 2 * kTileBytes);
          q_armed[qb] = (int)((qc >> 1) & 1u);
          for (int T = 0; T < 2; ++T)
            for (int c = 0; c < kSub; ++c)
              tma_load_3d(s.q[qb][T] + c * (kTile * 128), &map_q, &s.q_full[qb], c * 64, (2 * u.p + T) * kTile,
                          u.head);
          ++qc;
        };
        auto q_free = [&]() { return mbar_try_wait(&s.q_empty[qc & 1], ((qc >> 1) & 1u) ^ 1u); };
        PairRun un, nx;
        bool have = pair_next_unit(args, 0, un);
        if (have) load_q(un);  // both buffers start free
        for (int i = 0; ok && have; ++i) {
          const bool has_next = pair_next_unit(args, i + 1, nx);
          bool q_pending = has_next;
          for (int t = 0; ok && t < un.n; ++t) {
            if (q_pending && q_free()) { load_q(nx); q_pending = false; }
            ok = load_kv(&map_k, un.j0 + t, un.kv_head);
            if (ok && q_pending && q_free()) { load_q(nx); q_pending = false; }
            if (ok) ok = load_kv(&map_v, un.j0 + t, un.kv_head);
          }
          if (ok && q_pending) {
            if (!mbar_wait(&s.q_empty[qc & 1], ((qc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 60)) { ok = false; break; }
            load_q(nx);
          }
          un = nx;
          have = has_next;
        }
        if (!ok) {  // let issued copies land before shared memory is released
          const uint64_t t0 = globaltimer();
          for (int b = 0; b < 2; ++b)
            if (q_armed[b] >= 0)
              while (!mbar_try_wait(&s.q_full[b], (uint32_t)q_armed[b]) && globaltimer() - t0 < kWaitTimeoutNs) {}
          for (int b = 0; b < kPairRing; ++b)
            if (kv_armed[b] >= 0)
              while (!mbar_try_wait(&s.kv_full[b], (uint32_t)kv_armed[b]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        }
      }
      __syncwarp();
    } else if (warp == kPairMmaWarp) {
      // ------------------------------------------------ MMA issuer
      if (elect_one()) {
        uint32_t qc = 0, kc = 0, sc[2] = {0, 0};
        bool ok = true;
        auto kv_wait = [&](uint32_t idx) -> bool {
          return mbar_wait(&s.kv_full[idx % kPairRing], (idx / kPairRing) & 1u, &s.abort, &g_attn_dev_error, 71);
        };
        auto kv_desc = [&](uint32_t idx, uint32_t lbo) {
          return smem_desc_sw128(smem_u32(s.kv[idx % kPairRing]), lbo, 1024);
        };
        PairRun un;
        for (int i = 0; ok && pair_next_unit(args, i, un); ++i) {
          const int qb = qc & 1;
          if (!mbar_wait(&s.q_full[qb], (qc >> 1) & 1u, &s.abort, &g_attn_dev_error, 70)) { ok = false; break; }
          ++qc;
          const uint64_t qdesc[2] = {smem_desc_sw128(smem_u32(s.q[qb][0]), 16, 1024),
                                     smem_desc_sw128(smem_u32(s.q[qb][1]), 16, 1024)};
          // S_T = Q_T K^T into TMEM buffer T, from ring entry idx
          auto issue_s = [&](int T, uint32_t idx) {
            const uint64_t kd = kv_desc(idx, 16);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4);
              mma_bf16_ss(tmem + (uint32_t)(T * kTile), qdesc[T] + off, kd + off, kIdescS, kk > 0 ? 1u : 0u);
            }
            mma_commit(&s.s_full[T]);
          };
          // O_T += P_T V from ring entry idx
          auto issue_pv = [&](int T, uint32_t idx, int t) {
            const uint64_t vd = kv_desc(idx, kTile * 128);
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              mma_bf16_ts(tmem + (uint32_t)((2 + T) * kTile), tmem + (uint32_t)(T * kTile + kk * 8),
                          vd + (uint32_t)(kk * 128), kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
          };
          const uint32_t k0 = kc;  // ring index of K(j0); V(j0 + t) at k0 + 2t + 1, K(j0 + t) at k0 + 2t
          if (!kv_wait(k0)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, k0);
          issue_s(1, k0);
          mma_commit(&s.kv_empty[k0 % kPairRing]);
          for (int t = 0; ok && t < un.n; ++t) {
            const uint32_t vi = k0 + 2 * t + 1, ki = k0 + 2 * t + 2;
            if (!kv_wait(vi)) { ok = false; break; }
            for (int T = 0; T < 2; ++T) {
              const int nT = T == 0 ? un.nA : un.n;
              if (t >= nT) continue;
              // corr_done: O rescaled for this step (and, at t == 0, the previous unit's O read)
              if (!mbar_wait(&s.corr_done[T], sc[T] & 1u, &s.abort, &g_attn_dev_error, 72)) { ok = false; break; }
              if (!mbar_wait(&s.p_full[T], sc[T] & 1u, &s.abort, &g_attn_dev_error, 73)) { ok = false; break; }
              tc_fence_after();
              ++sc[T];
              issue_pv(T, vi, t);
              if (T == 1) mma_commit(&s.kv_empty[vi % kPairRing]);  // V(t) read by both tiles
              if (t == nT - 1) mma_commit(&s.o_ready[T]);
              if (t + 1 < nT) {
                if (T == 0 || t + 1 >= un.nA) {  // K(t+1) not yet waited for
                  if (!kv_wait(ki)) { ok = false; break; }
                  tc_fence_after();
                }
                issue_s(T, ki);
                if (T == 1) mma_commit(&s.kv_empty[ki % kPairRing]);  // K(t+1) read by both tiles
              }
            }
          }
          if (!ok) break;
          kc += 2 * (uint32_t)un.n;
        }
        mma_commit(&s.mma_done);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
      }
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kPairMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}
