// attention.cu - causal scaled-dot-product attention O = softmax(Q K^T * scale + mask) V.
//
// Reference algorithms (Nags-gk/nki-kernel-lab):
//   flash family   nkilab/kernels/attention.py:92-176 (_flash_tile_update, flash_attention),
//                  :204-325 (balanced / pipelined variants, same numerics)
//   causal mask    nkilab/kernels/attention.py:28-32 (keep where q - k >= 0; diagonal tiles only)
//   naive          nkilab/kernels/attention.py:35-89 (scores and probs materialised in HBM)
// Numerics kept from the reference: 128 x 128 score tiles, fp32 scores / running max /
// running sum / output accumulator, P rounded to the input dtype before P.V (:228,
// dtype=vdtype), key tiles after the diagonal skipped (:166), final O * (1/l) rounded
// once (:137-142). The running max is kept in the log2 domain (scale * log2(e) folded
// into one FMA before a hardware exp2); mathematically the same exp(scale*s - m).
//
// bf16 kernel (sm_100a), one CTA per (head, 128-query tile), heavy tiles first:
//   warps 0-7  softmax. Thread = (query row, half): row r = 32*(warp%4) + lane is its
//              TMEM lane; half = warp/4 owns score columns [64*half, 64*half + 64) and
//              output columns [D/2*half, D/2*(half+1)). Per key tile: one tcgen05.ld
//              batch of its 64 S columns, row max exchanged with the other half through
//              shared memory (mbarrier-synchronised), exp2 with the scale folded into
//              one FMA, P (bf16) into its 64-key sub-tile of a double-buffered shared P
//              tile (UMMA K-major 128-byte swizzle), then O(j-1) = O(j-2)*corr + P(j-1).V
//              from TMEM (deferred one tile, so the tensor core runs P.V(j-1) and S(j+1)
//              while softmax(j) runs). Row sums stay per half until the end.
//   warp 8     TMA producer: Q once, K and V tiles through separate 2-deep rings
//   warp 9     TMEM allocator + single-thread tcgen05.mma issuer
//   TMEM       S double buffer (2 x 128 fp32 columns) + P.V double buffer (2 x d)
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace nkl {
namespace {

__device__ unsigned int g_attn_dev_error = 0;

using namespace sm100;

constexpr int kTile = 128;  // query / key tile, as the reference's T (attention.py:24)
constexpr int kSoftmaxThreads = 256;
constexpr int kAttnThreads = kSoftmaxThreads + 64;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
struct AttnSmem {
  static constexpr int kQBytes = kTile * D * 2;
  uint8_t q[kQBytes];              // D/64 sub-tiles of [128 rows x 128 B]
  uint8_t k[2][kQBytes];           // key tiles, K-major (head_dim contiguous)
  uint8_t v[2][kQBytes];           // value tiles, N-major for the P.V product
  uint8_t p[2][kTile * kTile * 2];  // P double buffer, each 2 sub-tiles of [128 rows x 64 keys]
  float red[2][2][kTile];          // [slot][half][row]: row-max exchange, then the final row sums
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_full[2], pv_free[2];
  uint64_t xchg[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

template <int D>
constexpr size_t attn_smem_bytes() {
  return sizeof(AttnSmem<D>);
}

// Wait by lane 0, then broadcast, so the whole warp stays converged for the
// .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, &g_attn_dev_error, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// ---- split-KV work units
// A unit is (head, query tile qt, key chunk k): key tiles [k*C, min((k+1)*C, qt+1)) of
// the causal range of query tile qt, for a chunk size C chosen on the host so that
// there are enough units to fill every SM. Units are numbered head-fastest, query
// tiles in descending order (longest first), chunks ascending, so the block scheduler
// hands the largest units out first. Query tiles split into several chunks write
// partial (O, running max, row sum) to the workspace; the chunk that finishes last
// combines them in chunk order, so the result does not depend on finish order.

// sum_{s=1..n} ceil(s / C): number of units of query tiles 0..n-1.
__host__ __device__ __forceinline__ int units_below(int n, int C) {
  const int a = n / C, b = n % C;
  return C * a * (a + 1) / 2 + b * (a + 1);
}

// Unit index within a head -> (query tile, chunk).
__device__ __forceinline__ void decode_unit(int u, int q_tiles, int C, int& qt, int& chunk) {
  const int total = units_below(q_tiles, C);
  int lo = 0, hi = q_tiles - 1;  // smallest qt with units_below(qt + 1) >= total - u
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (units_below(mid + 1, C) >= total - u) hi = mid;
    else lo = mid + 1;
  }
  qt = lo;
  chunk = u - (total - units_below(qt + 1, C));
}

struct AttnArgs {
  bf16* out;
  unsigned char* ws;     // NULL when every query tile is a single unit
  int heads, seq, q_tiles, chunk, units_per_head;
  float scale_log2;
  size_t ws_stats_off, ws_o_off;  // byte offsets of the partial (m, l) and O regions
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_fwd_bf16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                     const AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicCAS(&g_attn_dev_error, 0u, 40u);
    return;
  }
  auto& s = *reinterpret_cast<AttnSmem<D>*>(smem_raw);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kSCol0 = 0;               // S buffers at columns [0,128) and [128,256)
  constexpr uint32_t kPVCol0 = 2 * kTile;      // P.V buffers at [256, 256+D) and [256+D, 256+2D)
  constexpr uint32_t kIdescS = idesc_bf16_f32(kTile, kTile, false, false);
  constexpr uint32_t kIdescPV = idesc_bf16_f32(kTile, D, false, true);
  constexpr uint32_t kTileBytes = kTile * D * 2;
  constexpr int kSub = D / 64;  // 64-column (128-byte) sub-tiles per Q/K/V tile
  constexpr int kHalfD = D / 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = args.heads;
  const float scale_log2 = args.scale_log2;
  const int head = (int)(blockIdx.x % (unsigned)heads);
  int qt, chunk;
  decode_unit((int)(blockIdx.x / (unsigned)heads), args.q_tiles, args.chunk, qt, chunk);
  const int n_chunks = (qt + args.chunk) / args.chunk;  // ceil((qt + 1) / C)
  const int j0 = chunk * args.chunk;                    // first key tile of this unit
  const int n_kv = min(args.chunk, qt + 1 - j0);         // causal: tiles after qt are fully masked
  const int q0 = qt * kTile;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], kSoftmaxThreads);
      mbar_init(&s.pv_full[i], 1);
      mbar_init(&s.pv_free[i], kSoftmaxThreads);
      mbar_init(&s.xchg[i], kSoftmaxThreads);
    }
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

  if (warp == kProducerWarp) {
    // ------------------------------------------------ TMA producer
    if (elect_one()) {
      int k_armed[2] = {-1, -1}, v_armed[2] = {-1, -1};
      bool ok = true;
      mbar_arrive_expect_tx(&s.q_full, kTileBytes);
      for (int c = 0; c < kSub; ++c) tma_load_3d(s.q + c * (kTile * 128), &map_q, &s.q_full, c * 64, q0, head);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1u, &s.abort, &g_attn_dev_error, 11)) { ok = false; break; }
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        k_armed[st] = (int)ph;
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.k[st] + c * (kTile * 128), &map_k, &s.k_full[st], c * 64, (j0 + j) * kTile, head);
        if (!mbar_wait(&s.v_empty[st], ph ^ 1u, &s.abort, &g_attn_dev_error, 12)) { ok = false; break; }
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        v_armed[st] = (int)ph;
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.v[st] + c * (kTile * 128), &map_v, &s.v_full[st], c * 64, (j0 + j) * kTile, head);
      }
      if (!ok) {  // let issued copies land before shared memory is released
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&s.q_full, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
        for (int i = 0; i < 2; ++i) {
          if (k_armed[i] >= 0)
            while (!mbar_try_wait(&s.k_full[i], (uint32_t)k_armed[i]) && globaltimer() - t0 < kWaitTimeoutNs) {}
          if (v_armed[i] >= 0)
            while (!mbar_try_wait(&s.v_full[i], (uint32_t)v_armed[i]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      bool ok = mbar_wait(&s.q_full, 0, &s.abort, &g_attn_dev_error, 21);
      const uint32_t q_base = smem_u32(s.q);
      // S(j) = Q K(j)^T into S buffer j&1.
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&s.k_full[st], (uint32_t)(j >> 1) & 1u, &s.abort, &g_attn_dev_error, 22)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * (kTile * 128) + (kk & 3) * 32);
          mma_bf16_ss(tmem + kSCol0 + (uint32_t)(st * kTile), smem_desc_sw128(q_base + off, 16, 1024),
                      smem_desc_sw128(k_base + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.k_empty[st]);
        mma_commit(&s.s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_kv > 1) ok = issue_s(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int b = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        // p_full(b) also means the softmax warps finished reading S buffer b.
        if (!mbar_wait(&s.p_full[b], ph, &s.abort, &g_attn_dev_error, 23)) { ok = false; break; }
        if (!mbar_wait(&s.v_full[b], ph, &s.abort, &g_attn_dev_error, 24)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&s.pv_free[b], ph ^ 1u, &s.abort, &g_attn_dev_error, 25)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_base = smem_u32(s.p[b]);
        const uint32_t v_base = smem_u32(s.v[b]);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t a_off = (uint32_t)((kk >> 2) * (kTile * 128) + (kk & 3) * 32);
          const uint32_t b_off = (uint32_t)(kk * 2048);
          mma_bf16_ss(tmem + kPVCol0 + (uint32_t)(b * D), smem_desc_sw128(p_base + a_off, 16, 1024),
                      smem_desc_sw128(v_base + b_off, kTile * 128, 1024), kIdescPV, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.v_empty[b]);
        mma_commit(&s.pv_full[b]);
        if (j + 2 < n_kv) ok = issue_s(j + 2);
      }
      mma_commit(&s.mma_done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
    }
  } else {
    // ------------------------------------------------ softmax (warps 0..7)
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int c0 = half * 64;  // first score column of this thread
    float2 o[kHalfD / 2];
#pragma unroll
    for (int i = 0; i < kHalfD / 2; ++i) o[i] = make_float2(0.f, 0.f);
    float m = -INFINITY, l = 0.f, corr_prev = 0.f;
    bool ok = true;
    const int sw = r & 7;
    const float2 sc2 = make_float2(scale_log2, scale_log2);

    // One key tile: row max, exp2, row sum and the bf16 P sub-tile. The diagonal tile
    // (the only one with masked keys) is a separate instantiation so the others carry
    // no per-element predicates.
    auto softmax_tile = [&](auto diag_tag, const uint32_t (&v)[64], int b, float& corr_out) -> bool {
      constexpr bool kDiag = decltype(diag_tag)::value;
      const uint32_t ph = 0;  // unused; phases are passed through the waits below
      (void)ph;
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 64; e += 8) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          float x0 = __uint_as_float(v[e + 2 * a]), x1 = __uint_as_float(v[e + 2 * a + 1]);
          if constexpr (kDiag) {
            if (c0 + e + 2 * a > r) x0 = -INFINITY;
            if (c0 + e + 2 * a + 1 > r) x1 = -INFINITY;
          }
          float t;
          asm("max.f32 %0, %1, %2, %3;" : "=f"(t) : "f"(mx[a]), "f"(x0), "f"(x1));
          mx[a] = t;
        }
      }
      float pm;
      asm("max.f32 %0, %1, %2, %3;" : "=f"(pm) : "f"(mx[0]), "f"(mx[1]), "f"(mx[2]));
      pm = fmaxf(pm, mx[3]);
      s.red[b][half][r] = pm;
      mbar_arrive(&s.xchg[b]);
      return true;
    };
    auto exp_tile = [&](auto diag_tag, const uint32_t (&v)[64], int b, float m_new) -> float {
      constexpr bool kDiag = decltype(diag_tag)::value;
      const float2 nm2 = make_float2(-m_new, -m_new);
      float2 rs[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint8_t* p_row = s.p[b] + half * (kTile * 128) + r * 128;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const int c = q * 8 + e;
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])), sc2, nm2);
          float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          if constexpr (kDiag) {
            if (c0 + c > r) p.x = 0.f;
            if (c0 + c + 1 > r) p.y = 0.f;
          }
          rs[(e >> 1) & 1] = __fadd2_rn(rs[(e >> 1) & 1], p);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(p.x, p.y);
          pk[e >> 1] = *reinterpret_cast<uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(p_row + ((q ^ sw) * 16)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      const float2 t = __fadd2_rn(rs[0], rs[1]);
      return t.x + t.y;
    };
    auto update_o = [&](int pb, float corr) {
      const uint32_t pv_addr = tmem + lane_off + kPVCol0 + (uint32_t)(pb * D + half * kHalfD);
      uint32_t w[kHalfD];
#pragma unroll
      for (int c = 0; c < kHalfD / 32; ++c) tmem_ld32(pv_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&w[c * 32]));
      tmem_wait_ld();
      const float2 c2 = make_float2(corr, corr);
#pragma unroll
      for (int e = 0; e < kHalfD / 2; ++e)
        o[e] = __ffma2_rn(o[e], c2, make_float2(__uint_as_float(w[2 * e]), __uint_as_float(w[2 * e + 1])));
    };

    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      const bool diag = (j0 + j == qt);
      if (!warp_wait(&s.s_full[b], ph, &s.abort, 31)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[64];
      {
        const uint32_t s_addr = tmem + lane_off + kSCol0 + (uint32_t)(b * kTile + c0);
        tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
      }
      float corr_unused = 0.f;
      if (diag) softmax_tile(std::true_type{}, v, b, corr_unused);
      else softmax_tile(std::false_type{}, v, b, corr_unused);
      if (!warp_wait(&s.xchg[b], ph, &s.abort, 32)) { ok = false; break; }
      const float mx = fmaxf(s.red[b][0][r], s.red[b][1][r]);
      const float m_new = fmaxf(m, mx * scale_log2);
      const float corr = fast_exp2(m - m_new);
      const float rs = diag ? exp_tile(std::true_type{}, v, b, m_new) : exp_tile(std::false_type{}, v, b, m_new);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&s.p_full[b]);
      l = l * corr + rs;
      // O(j-1) = O(j-2) * corr(j-1) + P(j-1).V(j-1), this thread's D/2 output columns
      if (j >= 1) {
        const int pb = (j - 1) & 1;
        if (!warp_wait(&s.pv_full[pb], (uint32_t)((j - 1) >> 1) & 1u, &s.abort, 33)) { ok = false; break; }
        tc_fence_after();
        update_o(pb, corr_prev);
        tc_fence_before();
        mbar_arrive(&s.pv_free[pb]);
      }
      corr_prev = corr;
      m = m_new;
    }
    if (ok) {
      const int pb = (n_kv - 1) & 1;
      ok = warp_wait(&s.pv_full[pb], (uint32_t)((n_kv - 1) >> 1) & 1u, &s.abort, 34);
      if (ok) {
        tc_fence_after();
        update_o(pb, corr_prev);
        // total row sum = the two halves' partial sums (same running max)
        const int fb = n_kv & 1;
        s.red[fb][half][r] = l;
        mbar_arrive(&s.xchg[fb]);
        ok = warp_wait(&s.xchg[fb], (uint32_t)(n_kv >> 1) & 1u, &s.abort, 35);
      }
      const int fb = n_kv & 1;
      float l_tot = 0.f;
      if (ok) l_tot = s.red[fb][0][r] + s.red[fb][1][r];
      bool write_out = ok;
      int xi = n_kv + 1;  // next use of the xchg barriers (one phase per use, alternating slots)
      if (ok && n_chunks > 1) {
        // ---- split query tile: publish this chunk's partial, the last chunk combines
        const int unit = (int)blockIdx.x;
        float* st_m = reinterpret_cast<float*>(args.ws + args.ws_stats_off) + (size_t)unit * 2 * kTile;
        float* o_part = reinterpret_cast<float*>(args.ws + args.ws_o_off) + (size_t)unit * kTile * D;
        // layout [col/4][row][4]: a warp's 32 rows store 512 contiguous bytes per instruction
        float4* op = reinterpret_cast<float4*>(o_part) + (size_t)(half * kHalfD / 4) * kTile + r;
#pragma unroll
        for (int g = 0; g < kHalfD / 4; ++g)
          op[(size_t)g * kTile] = make_float4(o[2 * g].x, o[2 * g].y, o[2 * g + 1].x, o[2 * g + 1].y);
        if (half == 0) {
          st_m[r] = m;
          st_m[kTile + r] = l_tot;
        }
        __threadfence();
        int* counter = reinterpret_cast<int*>(args.ws) + head * args.q_tiles + qt;
        const int sb = xi & 1;
        mbar_arrive(&s.xchg[sb]);
        ok = warp_wait(&s.xchg[sb], (uint32_t)(xi >> 1) & 1u, &s.abort, 36);
        ++xi;
        if (ok && threadIdx.x == 0) s.red[sb][0][0] = (float)atomicAdd(counter, 1);
        if (ok) {
          mbar_arrive(&s.xchg[xi & 1]);
          ok = warp_wait(&s.xchg[xi & 1], (uint32_t)(xi >> 1) & 1u, &s.abort, 37);
          ++xi;
        }
        write_out = ok && (int)s.red[sb][0][0] == n_chunks - 1;
        if (write_out) {
          __threadfence();
          const int base_unit = (int)(blockIdx.x / (unsigned)heads) - chunk;  // unit index (per head) of chunk 0
          const float* ws_stats = reinterpret_cast<const float*>(args.ws + args.ws_stats_off);
          const float* ws_o = reinterpret_cast<const float*>(args.ws + args.ws_o_off);
          float mmax = -INFINITY;
          for (int c = 0; c < n_chunks; ++c) {
            const size_t uc = (size_t)(base_unit + c) * heads + head;
            const float mc = (c == chunk) ? m : __ldcg(ws_stats + uc * 2 * kTile + r);
            mmax = fmaxf(mmax, mc);
          }
          float2 acc[kHalfD / 2];
#pragma unroll
          for (int e = 0; e < kHalfD / 2; ++e) acc[e] = make_float2(0.f, 0.f);
          float lsum = 0.f;
          for (int c = 0; c < n_chunks; ++c) {
            const size_t uc = (size_t)(base_unit + c) * heads + head;
            float mc, lc;
            if (c == chunk) {
              mc = m;
              lc = l_tot;
            } else {
              mc = __ldcg(ws_stats + uc * 2 * kTile + r);
              lc = __ldcg(ws_stats + uc * 2 * kTile + kTile + r);
            }
            const float w = fast_exp2(mc - mmax);
            lsum = fmaf(w, lc, lsum);
            const float2 w2 = make_float2(w, w);
            if (c == chunk) {
#pragma unroll
              for (int e = 0; e < kHalfD / 2; ++e) acc[e] = __ffma2_rn(o[e], w2, acc[e]);
            } else {
              const float4* src =
                  reinterpret_cast<const float4*>(ws_o + uc * kTile * D) + (size_t)(half * kHalfD / 4) * kTile + r;
#pragma unroll
              for (int e = 0; e < kHalfD / 4; ++e) {
                const float4 t = __ldcg(src + (size_t)e * kTile);
                acc[2 * e] = __ffma2_rn(make_float2(t.x, t.y), w2, acc[2 * e]);
                acc[2 * e + 1] = __ffma2_rn(make_float2(t.z, t.w), w2, acc[2 * e + 1]);
              }
            }
          }
#pragma unroll
          for (int e = 0; e < kHalfD / 2; ++e) o[e] = acc[e];
          l_tot = lsum;
          if (threadIdx.x == 0) *counter = 0;  // ready for the next launch on this workspace
        }
      }
      if (write_out) {
        // Stage the bf16 output tile in the Q buffer (free: every MMA has completed) in
        // the 128-byte-swizzled layout of the output tensor map, then one TMA store per
        // 64-column sub-tile; rows past seq are clipped by the TMA unit.
        const float linv = 1.0f / l_tot;
        const int col0 = half * kHalfD;
        uint8_t* orow = s.q + (col0 / 64) * (kTile * 128) + r * 128;
#pragma unroll
        for (int c = 0; c < kHalfD / 8; ++c) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            f[2 * e] = o[c * 4 + e].x * linv;
            f[2 * e + 1] = o[c * 4 + e].y * linv;
          }
          const int ch = ((col0 % 64) / 8 + c) ^ sw;
          *reinterpret_cast<uint4*>(orow + ch * 16) = pack16<bf16>(f);
        }
        fence_proxy_async_smem();
        mbar_arrive(&s.xchg[xi & 1]);
        const bool staged = warp_wait(&s.xchg[xi & 1], (uint32_t)(xi >> 1) & 1u, &s.abort, 38);
        if (staged && threadIdx.x == 0) {
#pragma unroll
          for (int c = 0; c < kSub; ++c) tma_store_3d(&map_o, s.q + c * (kTile * 128), c * 64, q0, head);
          tma_store_commit();
          tma_store_wait_read();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ fp32 exact flash kernel
// CUDA-core flash attention for fp32 inputs (the reference's fp32 tests need 2e-5
// absolute agreement with PyTorch SDPA, beyond TF32 tensor cores). A block of 4 warps
// owns 16 query rows (4 per warp); key/value tiles of 32 rows are staged in shared
// memory; lane k scores key k, lane c accumulates output columns c, c+32, ...

constexpr int kF32Rows = 16;
constexpr int kF32Keys = 32;

__global__ void __launch_bounds__(128)
attn_fwd_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    float* __restrict__ out, int seq, int d, float scale) {
  __shared__ float ks[kF32Keys][129];
  __shared__ float vs[kF32Keys][128];
  __shared__ float qs[kF32Rows][128];
  const int head = blockIdx.y;
  const int r0 = blockIdx.x * kF32Rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qh = q + (int64_t)head * seq * d;
  const float* kh = k + (int64_t)head * seq * d;
  const float* vh = v + (int64_t)head * seq * d;
  for (int i = threadIdx.x; i < kF32Rows * d; i += 128) {
    const int rr = i / d, cc = i % d;
    qs[rr][cc] = (r0 + rr < seq) ? qh[(int64_t)(r0 + rr) * d + cc] : 0.f;
  }
  float o[4][4];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[i][c] = 0.f;
  }
  const int last_row = min(r0 + kF32Rows, seq) - 1;
  for (int k0 = 0; k0 <= last_row; k0 += kF32Keys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kF32Keys * d; i += 128) {
      const int rr = i / d, cc = i % d;
      const bool in = k0 + rr < seq;
      ks[rr][cc] = in ? kh[(int64_t)(k0 + rr) * d + cc] : 0.f;
      vs[rr][cc] = in ? vh[(int64_t)(k0 + rr) * d + cc] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = warp * 4 + i;
      const int row = r0 + rl;
      float sc = 0.f;
      for (int c = 0; c < d; ++c) sc = fmaf(qs[rl][c], ks[lane][c], sc);
      const int key = k0 + lane;
      const bool valid = key <= row && key < seq;
      const float x = valid ? sc * scale : -INFINITY;
      const float m_new = fmaxf(m[i], warp_max(x));
      const float p = valid ? expf(x - m_new) : 0.f;
      const float corr = expf(m[i] - m_new);
      l[i] = l[i] * corr + warp_sum(p);
#pragma unroll
      for (int c = 0; c < 4; ++c) o[i][c] *= corr;
      for (int kk = 0; kk < kF32Keys; ++kk) {
        const float pk = __shfl_sync(0xffffffffu, p, kk);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int col = lane + 32 * c;
          if (col < d) o[i][c] = fmaf(pk, vs[kk][col], o[i][c]);
        }
      }
      m[i] = m_new;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = r0 + warp * 4 + i;
    if (row >= seq) continue;
    const float linv = 1.0f / l[i];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = lane + 32 * c;
      if (col < d) out[((int64_t)head * seq + row) * d + col] = o[i][c] * linv;
    }
  }
}

// ------------------------------------------------------------------ naive 3-pass path
// attention.py:35-89: pass 1 writes masked fp32 scores, pass 2 normalises full rows
// into probabilities of the input dtype, pass 3 multiplies the full S x S
// probability matrix by V. Plain tiled CUDA-core kernels, fp32 accumulation.

constexpr int kNT = 64;  // output tile
constexpr int kNK = 16;  // reduction step

// C[h] = A[h] (M x K) * op(B[h]) with op(B) = B^T when b_is_nk (B stored N x K).
template <typename TA, typename TC, bool kScores>
__global__ void __launch_bounds__(256)
naive_bmm_kernel(const TA* __restrict__ A, const TA* __restrict__ B, TC* __restrict__ C, int M, int N, int K,
                 float scale) {
  __shared__ float As[kNK][kNT + 4];
  __shared__ float Bs[kNK][kNT + 4];
  const int h = blockIdx.z;
  const TA* Ah = A + (int64_t)h * M * K;
  const TA* Bh = B + (int64_t)h * N * K;
  TC* Ch = C + (int64_t)h * M * N;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kNT, n0 = blockIdx.x * kNT;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kNK) {
    for (int i = threadIdx.x; i < kNT * kNK; i += 256) {
      const int rr = i / kNK, kk = i % kNK;
      const int gm = m0 + rr, gk = k0 + kk;
      As[kk][rr] = (gm < M && gk < K) ? to_f32(Ah[(int64_t)gm * K + gk]) : 0.f;
      if (kScores) {  // B = keys [N x K]
        const int gn = n0 + rr;
        Bs[kk][rr] = (gn < N && gk < K) ? to_f32(Bh[(int64_t)gn * K + gk]) : 0.f;
      } else {        // B = values [K x N]
        const int kr = i / kNT, cn = i % kNT;
        const int gk2 = k0 + kr, gn = n0 + cn;
        Bs[kr][cn] = (gk2 < K && gn < N) ? to_f32(Bh[(int64_t)gk2 * N + gn]) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kNK; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(As[kk][ty * 4 + i], Bs[kk][tx * 4 + j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      if (kScores) {
        const float sc = acc[i][j] * scale;
        Ch[(int64_t)gm * N + gn] = from_f32<TC>(gm - gn >= 0 ? sc : -3.0e38f);  // attention.py:25,28-32
      } else {
        Ch[(int64_t)gm * N + gn] = from_f32<TC>(acc[i][j]);
      }
    }
  }
}

// One block per score row: nmax = -max, e = exp(row + nmax), p = e * (1/sum e).
template <typename TP>
__global__ void __launch_bounds__(256)
naive_softmax_kernel(const float* __restrict__ scores, TP* __restrict__ probs, int n) {
  __shared__ float red[9];
  const float* row = scores + (int64_t)blockIdx.x * n;
  TP* prow = probs + (int64_t)blockIdx.x * n;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < n; c += 256) mx = fmaxf(mx, row[c]);
  mx = warp_max(mx);
  if (lane == 0) red[w] = mx;
  __syncthreads();
  if (w == 0) {
    float t = warp_max(lane < 8 ? red[lane] : -INFINITY);
    if (lane == 0) red[8] = t;
  }
  __syncthreads();
  const float nmax = -red[8];
  __syncthreads();
  float sm = 0.f;
  for (int c = threadIdx.x; c < n; c += 256) sm += expf(row[c] + nmax);
  sm = warp_sum(sm);
  if (lane == 0) red[w] = sm;
  __syncthreads();
  if (w == 0) {
    float t = warp_sum(lane < 8 ? red[lane] : 0.f);
    if (lane == 0) red[8] = t;
  }
  __syncthreads();
  const float rinv = 1.0f / red[8];
  for (int c = threadIdx.x; c < n; c += 256) prow[c] = from_f32<TP>(expf(row[c] + nmax) * rinv);
}

// ------------------------------------------------------------------ host

int make_qkv_map(CUtensorMap* m, const void* base, int heads, int seq, int d, const char* what) {
  const uint64_t dims[3] = {(uint64_t)d, (uint64_t)seq, (uint64_t)heads};
  const uint64_t strides[2] = {(uint64_t)d * 2, (uint64_t)seq * d * 2};
  const uint32_t box[3] = {64, (uint32_t)kTile, 1};
  return make_tensor_map_bf16(m, base, 3, dims, strides, box, what);
}

// Work decomposition shared by the workspace-size query and the launch.
struct AttnPlan {
  int q_tiles = 0, chunk = 0, units_per_head = 0;
  size_t stats_off = 0, o_off = 0, ws_bytes = 0;  // ws_bytes == 0: no split, no workspace
};

inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

AttnPlan plan_attention(int heads, int seq, int d, bool split) {
  AttnPlan p;
  p.q_tiles = (seq + kTile - 1) / kTile;
  p.chunk = p.q_tiles;
  if (split) {
    // halve the chunk until there are at least two units per SM (or chunks of 2 tiles)
    const int target = 2 * sm_count();
    while (p.chunk > 2 && heads * units_below(p.q_tiles, p.chunk) < target) p.chunk = (p.chunk + 1) / 2;
  }
  p.units_per_head = units_below(p.q_tiles, p.chunk);
  if (p.chunk < p.q_tiles) {
    const size_t units = (size_t)heads * p.units_per_head;
    p.stats_off = round256((size_t)heads * p.q_tiles * sizeof(int));
    p.o_off = p.stats_off + round256(units * 2 * kTile * sizeof(float));
    p.ws_bytes = p.o_off + units * kTile * (size_t)d * sizeof(float);
  }
  return p;
}

template <int D>
int launch_attn_bf16(const void* q, const void* k, const void* v, void* out, int heads, int seq, float scale,
                     void* ws, size_t ws_bytes, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo;
  int rc = make_qkv_map(&mq, q, heads, seq, D, "nkl_attention(q)");
  if (!rc) rc = make_qkv_map(&mk, k, heads, seq, D, "nkl_attention(k)");
  if (!rc) rc = make_qkv_map(&mv, v, heads, seq, D, "nkl_attention(v)");
  if (!rc) rc = make_qkv_map(&mo, out, heads, seq, D, "nkl_attention(out)");
  if (rc) return rc;
  AttnPlan plan = plan_attention(heads, seq, D, ws != nullptr);
  if (ws != nullptr && plan.ws_bytes > 0 && ws_bytes < plan.ws_bytes)
    return fail(NKL_ERR_ARG, "nkl_attention_ws: workspace %zu B < required %zu B", ws_bytes, plan.ws_bytes);
  if (plan.ws_bytes == 0) ws = nullptr;
  constexpr size_t smem = attn_smem_bytes<D>();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_bf16_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "nkl_attention: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  AttnArgs a;
  a.out = static_cast<bf16*>(out);
  a.ws = static_cast<unsigned char*>(ws);
  a.heads = heads;
  a.seq = seq;
  a.q_tiles = plan.q_tiles;
  a.chunk = plan.chunk;
  a.units_per_head = plan.units_per_head;
  a.scale_log2 = scale * kLog2e;
  a.ws_stats_off = plan.stats_off;
  a.ws_o_off = plan.o_off;
  const unsigned grid = (unsigned)(heads * plan.units_per_head);
  attn_fwd_bf16_kernel<D><<<grid, kAttnThreads, smem, st>>>(mq, mk, mv, mo, a);
  return check_launch("nkl_attention");
}

int check_attn(const char* op, int64_t heads, int64_t seq, int64_t d, int dtype) {
  if (!valid_dtype(dtype)) return fail(NKL_ERR_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (heads < 0 || seq < 0 || d < 1 || d > 128)
    return fail(NKL_ERR_SHAPE, "%s: need heads >= 0, seq >= 0, 1 <= head_dim <= 128 (got %lld, %lld, %lld)", op,
                (long long)heads, (long long)seq, (long long)d);
  if (heads > 65535 || seq > (1 << 24)) return fail(NKL_ERR_SHAPE, "%s: heads or seq too large", op);
  return NKL_OK;
}

}  // namespace

int attention_read_and_clear_device_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_dev_error, sizeof(v)) != cudaSuccess) return -1;
  if (v && cudaMemcpyToSymbol(g_attn_dev_error, &zero, sizeof(zero)) != cudaSuccess) return -1;
  return (int)v;
}

}  // namespace nkl

using namespace nkl;

extern "C" int nkl_attention(const void* q, const void* k, const void* v, void* out, int64_t heads, int64_t seq,
                             int64_t head_dim, float scale, int dtype, void* stream) {
  int rc = check_attn("nkl_attention", heads, seq, head_dim, dtype);
  if (rc) return rc;
  if (heads == 0 || seq == 0) return NKL_OK;
  if (!q || !k || !v || !out) return fail(NKL_ERR_ARG, "nkl_attention: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NKL_FLOAT32) {
    dim3 grid((unsigned)((seq + kF32Rows - 1) / kF32Rows), (unsigned)heads);
    attn_fwd_f32_kernel<<<grid, 128, 0, st>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                              static_cast<const float*>(v), static_cast<float*>(out), (int)seq,
                                              (int)head_dim, scale);
    return check_launch("nkl_attention");
  }
  if (head_dim != 64 && head_dim != 128)
    return fail(NKL_ERR_SHAPE, "nkl_attention: bf16 head_dim must be 64 or 128 (got %lld); pad on the host",
                (long long)head_dim);
  if (!is_aligned(q, 16) || !is_aligned(k, 16) || !is_aligned(v, 16) || !is_aligned(out, 16))
    return fail(NKL_ERR_ALIGN, "nkl_attention: bf16 tensors must be 16-byte aligned");
  if (head_dim == 64) return launch_attn_bf16<64>(q, k, v, out, (int)heads, (int)seq, scale, nullptr, 0, st);
  return launch_attn_bf16<128>(q, k, v, out, (int)heads, (int)seq, scale, nullptr, 0, st);
}

extern "C" size_t nkl_attention_workspace_size(int64_t heads, int64_t seq, int64_t head_dim, int dtype) {
  if (dtype != NKL_BFLOAT16 || heads <= 0 || seq <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  if (heads > 65535 || seq > (1 << 24)) return 0;
  return plan_attention((int)heads, (int)seq, (int)head_dim, true).ws_bytes;
}

extern "C" int nkl_attention_ws(const void* q, const void* k, const void* v, void* out, void* workspace,
                                size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim, float scale,
                                int dtype, void* stream) {
  if (workspace == nullptr || dtype != NKL_BFLOAT16)
    return nkl_attention(q, k, v, out, heads, seq, head_dim, scale, dtype, stream);
  int rc = check_attn("nkl_attention_ws", heads, seq, head_dim, dtype);
  if (rc) return rc;
  if (heads == 0 || seq == 0) return NKL_OK;
  if (!q || !k || !v || !out) return fail(NKL_ERR_ARG, "nkl_attention_ws: NULL pointer");
  if (head_dim != 64 && head_dim != 128)
    return fail(NKL_ERR_SHAPE, "nkl_attention_ws: bf16 head_dim must be 64 or 128 (got %lld); pad on the host",
                (long long)head_dim);
  if (!is_aligned(q, 16) || !is_aligned(k, 16) || !is_aligned(v, 16) || !is_aligned(out, 16))
    return fail(NKL_ERR_ALIGN, "nkl_attention_ws: bf16 tensors must be 16-byte aligned");
  if (!is_aligned(workspace, 256)) return fail(NKL_ERR_ALIGN, "nkl_attention_ws: workspace not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    return launch_attn_bf16<64>(q, k, v, out, (int)heads, (int)seq, scale, workspace, workspace_bytes, st);
  return launch_attn_bf16<128>(q, k, v, out, (int)heads, (int)seq, scale, workspace, workspace_bytes, st);
}

extern "C" size_t nkl_attention_naive_workspace_size(int64_t heads, int64_t seq, int dtype) {
  if (heads <= 0 || seq <= 0 || !valid_dtype(dtype)) return 0;
  const size_t n = (size_t)heads * (size_t)seq * (size_t)seq;
  const size_t scores = (n * 4 + 255) & ~size_t(255);
  return scores + ((n * dtype_size(dtype) + 255) & ~size_t(255));
}

extern "C" int nkl_attention_naive(const void* q, const void* k, const void* v, void* out, void* workspace,
                                   size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim, float scale,
                                   int dtype, void* stream) {
  int rc = check_attn("nkl_attention_naive", heads, seq, head_dim, dtype);
  if (rc) return rc;
  if (heads == 0 || seq == 0) return NKL_OK;
  if (!q || !k || !v || !out || !workspace) return fail(NKL_ERR_ARG, "nkl_attention_naive: NULL pointer");
  const size_t need = nkl_attention_naive_workspace_size(heads, seq, dtype);
  if (workspace_bytes < need)
    return fail(NKL_ERR_ARG, "nkl_attention_naive: workspace %zu B < required %zu B", workspace_bytes, need);
  if (!is_aligned(workspace, 256)) return fail(NKL_ERR_ALIGN, "nkl_attention_naive: workspace not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t n = (size_t)heads * (size_t)seq * (size_t)seq;
  float* scores = static_cast<float*>(workspace);
  void* probs = static_cast<char*>(workspace) + ((n * 4 + 255) & ~size_t(255));
  const int S = (int)seq, d = (int)head_dim, H = (int)heads;
  dim3 g1((unsigned)((S + kNT - 1) / kNT), (unsigned)((S + kNT - 1) / kNT), (unsigned)H);
  dim3 g3((unsigned)((d + kNT - 1) / kNT), (unsigned)((S + kNT - 1) / kNT), (unsigned)H);
  if (dtype == NKL_FLOAT32) {
    naive_bmm_kernel<float, float, true><<<g1, 256, 0, st>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                                             scores, S, S, d, scale);
    naive_softmax_kernel<float><<<(unsigned)(H * S), 256, 0, st>>>(scores, static_cast<float*>(probs), S);
    naive_bmm_kernel<float, float, false><<<g3, 256, 0, st>>>(static_cast<const float*>(probs),
                                                              static_cast<const float*>(v), static_cast<float*>(out), S,
                                                              d, S, 1.f);
  } else {
    naive_bmm_kernel<bf16, float, true><<<g1, 256, 0, st>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                                            scores, S, S, d, scale);
    naive_softmax_kernel<bf16><<<(unsigned)(H * S), 256, 0, st>>>(scores, static_cast<bf16*>(probs), S);
    naive_bmm_kernel<bf16, bf16, false><<<g3, 256, 0, st>>>(static_cast<const bf16*>(probs),
                                                            static_cast<const bf16*>(v), static_cast<bf16*>(out), S, d,
                                                            S, 1.f);
  }
  return check_launch("nkl_attention_naive");
}
