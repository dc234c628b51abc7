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
// The reference rescales O on every key tile; here O is rescaled only when a row's
// running max grows by more than 2^8 (P values stay <= 256, exact in fp32 and
// relatively exact in bf16), which gives the same softmax up to rounding.
//
// bf16 kernel (sm_100a): persistent, one CTA per SM, two softmax engines per CTA.
//   work unit  (head, query-tile pair 2p / 2p+1, chunk of the causal key range); the
//              host orders units longest first and assigns them to CTAs greedily
//              (LPT); query tiles whose key range is split over several units write
//              partial (O, max, sum) to a workspace and the chunk that finishes last
//              combines them in chunk order (result independent of finish order)
//   warps 0-3  engine 0 (query tile 2p), warps 4-7 engine 1 (tile 2p+1); thread =
//              query row = TMEM lane. Per key tile: tcgen05.ld of the 128 scores, row
//              max, lazy rescale of O in TMEM, exp2 with the scale folded into one FMA,
//              P (bf16 pairs) written back over the score columns with tcgen05.st
//   warp 8     TMA producer: Q of both engines per unit, K and V tiles through 2-deep
//              rings shared by the engines
//   warp 9     TMEM allocator + single-thread tcgen05.mma issuer, interleaving the
//              engines: S_e = Q_e K^T (smem x smem), O_e += P_e V (P from TMEM)
//   TMEM       S/P of engine 0 [0,128), engine 1 [128,256), O_0 [256,256+d), O_1 after
//   epilogue   O from TMEM, * 1/l, bf16, staged in the engine's Q buffer, TMA store
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <vector>

#include <cuda_fp16.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace nkl {
namespace {

__device__ unsigned int g_attn_dev_error = 0;

using namespace sm100;

constexpr int kTile = 128;  // query / key tile, as the reference's T (attention.py:24)
constexpr int kEngineThreads = 128;
constexpr int kAttnThreads = 2 * kEngineThreads + 64;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the row max grows by > 2^8
constexpr int kMaxCtas = 192;         // schedule table capacity (>= SMs of any sm_100 part)
constexpr int kMaxSched = 1024;       // units listed explicitly; more units: round-robin
constexpr int kMaxChunks = 4;         // a query tile's key range is split into at most 4 units

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

template <int D>
struct AttnSmem {
  static constexpr int kTileBytes = kTile * D * 2;
  uint8_t q[2][kTileBytes];  // per engine: D/64 sub-tiles of [128 rows x 128 B]; output staging
  uint8_t k[2][kTileBytes];  // key ring, K-major (head_dim contiguous)
  uint8_t v[2][kTileBytes];  // value ring, N-major for the P.V product
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2], pv_done[2], o_free[2];
  uint64_t eng_sync[2];  // engine-local barrier (128 arrivals) for the epilogue
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int flag[2];
};

template <int D>
constexpr size_t attn_smem_bytes() {
  return sizeof(AttnSmem<D>);
}

// ---- split-KV work units over query-tile pairs
struct AttnArgs {
  unsigned char* ws;  // NULL when no query tile is split
  int heads, q_tiles, pairs, chunk, units;
  float scale_log2;
  size_t ws_stats_off, ws_o_off;  // byte offsets of the partial (max, sum) and O regions
  int n_ctas_listed;              // > 0: cta_off / unit_list give each CTA's units
  uint16_t cta_off[kMaxCtas + 1];
  uint16_t unit_list[kMaxSched];
};

struct Unit {
  int head, pm, chunk, n_chunks, j0, n, v0;  // v0: per-head index of this pair's chunk 0
};

__host__ __device__ __forceinline__ int pair_tiles(int pm, int q_tiles) {
  return (2 * pm + 2 < q_tiles) ? 2 * pm + 2 : q_tiles;
}

// Unit index -> (head, pair, chunk). Units run head-fastest; pairs longest first; chunks ascending.
__host__ __device__ __forceinline__ Unit decode_unit(int u, int heads, int pairs, int q_tiles, int C) {
  Unit r;
  r.head = u % heads;
  int v = u / heads, base = 0;
  for (int pm = pairs - 1; pm >= 0; --pm) {
    const int nt = pair_tiles(pm, q_tiles);
    const int c = (nt + C - 1) / C;
    if (v < base + c) {
      r.pm = pm;
      r.chunk = v - base;
      r.n_chunks = c;
      r.j0 = r.chunk * C;
      r.n = (C < nt - r.j0) ? C : nt - r.j0;
      r.v0 = base;
      return r;
    }
    base += c;
  }
  r.pm = -1;
  return r;
}

// Wait by lane 0, then broadcast, so the whole warp stays converged for the
// .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, &g_attn_dev_error, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ int unit_of(const AttnArgs& a, int i, int& u) {
  if (a.n_ctas_listed > 0) {
    const int k = a.cta_off[blockIdx.x] + i;
    if (k >= a.cta_off[blockIdx.x + 1]) return 0;
    u = a.unit_list[k];
    return 1;
  }
  u = (int)blockIdx.x + i * (int)gridDim.x;
  return u < a.units;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_fwd_bf16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                     const __grid_constant__ AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicCAS(&g_attn_dev_error, 0u, 40u);
    return;
  }
  auto& s = *reinterpret_cast<AttnSmem<D>*>(smem_raw);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kOCol0 = 2 * kTile;  // O_e at 256 + e*D
  constexpr uint32_t kIdescS = idesc_bf16_f32(kTile, kTile, false, false);
  constexpr uint32_t kIdescPV = idesc_bf16_f32(kTile, D, false, true);
  constexpr uint32_t kTileBytes = kTile * D * 2;
  constexpr int kSub = D / 64;  // 64-column (128-byte) sub-tiles per Q/K/V tile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = args.heads, q_tiles = args.q_tiles;
  const float scale_log2 = args.scale_log2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], kEngineThreads);
      mbar_init(&s.pv_done[i], 1);
      mbar_init(&s.o_free[i], kEngineThreads);
      mbar_init(&s.eng_sync[i], kEngineThreads);
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
      uint32_t kc = 0, vc = 0, qc[2] = {0, 0};
      int k_armed[2] = {-1, -1}, v_armed[2] = {-1, -1}, q_armed[2] = {-1, -1};
      bool ok = true;
      int u;
      // Per unit: K/V tile 0 first (their slots free up as soon as the previous unit's
      // MMAs consume them), then the engines' Q tiles (their buffers free up only after
      // the previous unit's output has been staged and stored), then the remaining K/V.
      auto load_kv = [&](const Unit& un, int t) -> bool {
        const int j = un.j0 + t;
        const int ks = kc & 1;
        if (!mbar_wait(&s.k_empty[ks], ((kc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 11)) return false;
        mbar_arrive_expect_tx(&s.k_full[ks], kTileBytes);
        k_armed[ks] = (int)((kc >> 1) & 1u);
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.k[ks] + c * (kTile * 128), &map_k, &s.k_full[ks], c * 64, j * kTile, un.head);
        ++kc;
        const int vs = vc & 1;
        if (!mbar_wait(&s.v_empty[vs], ((vc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 12)) return false;
        mbar_arrive_expect_tx(&s.v_full[vs], kTileBytes);
        v_armed[vs] = (int)((vc >> 1) & 1u);
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.v[vs] + c * (kTile * 128), &map_v, &s.v_full[vs], c * 64, j * kTile, un.head);
        ++vc;
        return true;
      };
      for (int i = 0; ok && unit_of(args, i, u); ++i) {
        const Unit un = decode_unit(u, heads, args.pairs, q_tiles, args.chunk);
        ok = load_kv(un, 0);
        for (int e = 0; e < 2 && ok; ++e) {
          const int qe = 2 * un.pm + e;
          if (qe >= q_tiles || qe < un.j0) continue;  // engine has no query tile / no key in this unit
          if (!mbar_wait(&s.q_empty[e], (qc[e] & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 10)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.q_full[e], kTileBytes);
          q_armed[e] = (int)(qc[e] & 1u);
          for (int c = 0; c < kSub; ++c)
            tma_load_3d(s.q[e] + c * (kTile * 128), &map_q, &s.q_full[e], c * 64, qe * kTile, un.head);
          ++qc[e];
        }
        for (int t = 1; t < un.n && ok; ++t) ok = load_kv(un, t);
      }
      if (!ok) {  // let issued copies land before shared memory is released
        const uint64_t t0 = globaltimer();
        for (int e = 0; e < 2; ++e) {
          if (q_armed[e] >= 0)
            while (!mbar_try_wait(&s.q_full[e], (uint32_t)q_armed[e]) && globaltimer() - t0 < kWaitTimeoutNs) {}
          if (k_armed[e] >= 0)
            while (!mbar_try_wait(&s.k_full[e], (uint32_t)k_armed[e]) && globaltimer() - t0 < kWaitTimeoutNs) {}
          if (v_armed[e] >= 0)
            while (!mbar_try_wait(&s.v_full[e], (uint32_t)v_armed[e]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      uint32_t kc = 0, vc = 0, qc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0};
      const uint64_t q_desc0 = smem_desc_sw128(smem_u32(s.q[0]), 16, 1024);
      const uint64_t q_desc1 = smem_desc_sw128(smem_u32(s.q[1]), 16, 1024);
      const uint64_t k_desc0 = smem_desc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t k_desc1 = smem_desc_sw128(smem_u32(s.k[1]), 16, 1024);
      const uint64_t v_desc0 = smem_desc_sw128(smem_u32(s.v[0]), kTile * 128, 1024);
      const uint64_t v_desc1 = smem_desc_sw128(smem_u32(s.v[1]), kTile * 128, 1024);
      bool ok = true;
      // S_e = Q_e K^T for the K stage ks
      auto issue_s = [&](int e, int ks) {
        const uint64_t qd = e ? q_desc1 : q_desc0;
        const uint64_t kd = ks ? k_desc1 : k_desc0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4);
          mma_bf16_ss(tmem + (uint32_t)(e * kTile), qd + off, kd + off, kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full[e]);
      };
      int u;
      for (int i = 0; ok && unit_of(args, i, u); ++i) {
        const Unit un = decode_unit(u, heads, args.pairs, q_tiles, args.chunk);
        int na[2];  // key tiles of this unit each engine takes part in
        for (int e = 0; e < 2; ++e) {
          const int qe = 2 * un.pm + e;
          na[e] = (qe >= q_tiles) ? 0 : max(0, min(un.n, qe + 1 - un.j0));
        }
        for (int e = 0; e < 2 && ok; ++e) {
          if (!na[e]) continue;
          ok = mbar_wait(&s.q_full[e], qc[e] & 1u, &s.abort, &g_attn_dev_error, 20);
          ++qc[e];
        }
        if (!ok) break;
        // S for tile 0
        {
          const int ks = kc & 1;
          if (!mbar_wait(&s.k_full[ks], (kc >> 1) & 1u, &s.abort, &g_attn_dev_error, 21)) break;
          tc_fence_after();
          for (int e = 0; e < 2; ++e)
            if (na[e] > 0) issue_s(e, ks);
          mma_commit(&s.k_empty[ks]);
        }
        for (int t = 0; t < un.n && ok; ++t) {
          const uint32_t kn = kc + (uint32_t)t + 1;  // ring index of the next K tile
          const uint32_t vi = vc + (uint32_t)t;
          const int vs = vi & 1;
          bool v_ready = false, k_ready = false;
          for (int e = 0; e < 2 && ok; ++e) {
            if (t >= na[e]) continue;
            if (!mbar_wait(&s.p_full[e], pc[e] & 1u, &s.abort, &g_attn_dev_error, 22)) { ok = false; break; }
            ++pc[e];
            if (t == 0 && !mbar_wait(&s.o_free[e], (oc[e] & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 23)) {
              ok = false;
              break;
            }
            if (!v_ready) {
              if (!mbar_wait(&s.v_full[vs], (vi >> 1) & 1u, &s.abort, &g_attn_dev_error, 24)) { ok = false; break; }
              v_ready = true;
            }
            tc_fence_after();
            const uint64_t vd = vs ? v_desc1 : v_desc0;
            const uint32_t p_tmem = tmem + (uint32_t)(e * kTile);
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              mma_bf16_ts(tmem + kOCol0 + (uint32_t)(e * D), p_tmem + (uint32_t)(kk * 8), vd + (uint32_t)(kk * 128),
                          kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
            if (t == na[e] - 1) {
              mma_commit(&s.pv_done[e]);
              ++oc[e];
            }
            if (t + 1 < na[e]) {  // next S of this engine, right behind its P.V (S/P columns reused)
              if (!k_ready) {
                if (!mbar_wait(&s.k_full[kn & 1], (kn >> 1) & 1u, &s.abort, &g_attn_dev_error, 25)) {
                  ok = false;
                  break;
                }
                k_ready = true;
                tc_fence_after();
              }
              issue_s(e, kn & 1);
            }
          }
          if (!ok) break;
          mma_commit(&s.v_empty[vs]);
          if (k_ready) mma_commit(&s.k_empty[kn & 1]);
        }
        kc += (uint32_t)un.n;
        vc += (uint32_t)un.n;
      }
      // Every MMA issued by this thread has completed once mma_done flips.
      mma_commit(&s.mma_done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
    }
  } else {
    // ------------------------------------------------ softmax engines (warps 0-3, 4-7)
    const int e = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + (uint32_t)(e * kTile);
    const uint32_t o_addr = tmem + lane_off + kOCol0 + (uint32_t)(e * D);
    const int sw = r & 7;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    uint32_t sc = 0, dc = 0, xc = 0;
    bool ok = true;
    int u;
    for (int i = 0; ok && unit_of(args, i, u); ++i) {
      const Unit un = decode_unit(u, heads, args.pairs, q_tiles, args.chunk);
      const int qe = 2 * un.pm + e;
      const int na = (qe >= q_tiles) ? 0 : max(0, min(un.n, qe + 1 - un.j0));
      if (na == 0) continue;
      float m_ref = -INFINITY, l = 0.f;
      for (int t = 0; t < na; ++t) {
        const int j = un.j0 + t;
        if (!warp_wait(&s.s_full[e], sc & 1u, &s.abort, 31)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        const bool diag = (j == qe);
        // all 128 scores of the row in one TMEM load batch
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
        tmem_wait_ld();
        if (diag) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > r) v[c] = __float_as_uint(-INFINITY);
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            float tm;
            asm("max.f32 %0, %1, %2, %3;"
                : "=f"(tm)
                : "f"(mx[a]), "f"(__uint_as_float(v[c + 2 * a])), "f"(__uint_as_float(v[c + 2 * a + 1])));
            mx[a] = tm;
          }
        }
        float rmax;
        asm("max.f32 %0, %1, %2, %3;" : "=f"(rmax) : "f"(mx[0]), "f"(mx[1]), "f"(mx[2]));
        rmax = fmaxf(rmax, mx[3]) * scale_log2;
        // lazy rescale: move the reference max only when it grew by more than 2^8
        float factor = 1.f;
        if (t == 0) {
          m_ref = rmax;
        } else if (rmax > m_ref + kRescaleLog2) {
          factor = fast_exp2(m_ref - rmax);
          m_ref = rmax;
        }
        if (__any_sync(0xffffffffu, factor != 1.f)) {
          // O holds P.V of tiles < t, complete: S(t) was issued after them. Rescale in TMEM.
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {  // 16 columns at a time: the scores stay in registers
            uint32_t w[16];
            tmem_ld16(o_addr + c * 16, w);
            tmem_wait_ld();
#pragma unroll
            for (int k2 = 0; k2 < 16; ++k2) w[k2] = __float_as_uint(__uint_as_float(w[k2]) * factor);
            tmem_st16(o_addr + c * 16, w);
          }
          tmem_wait_st();
        }
        // P = exp2(s * scale_log2 - m_ref) as bf16 pairs, packed in place: the pair of
        // keys (c, c+1) lands in v[c/2], a score already consumed (masked keys give 0)
        const float2 nm2 = make_float2(-m_ref, -m_ref);
        float2 rs[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])), sc2, nm2);
          const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          rs[(c >> 1) & 1] = __fadd2_rn(rs[(c >> 1) & 1], p);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(p.x, p.y);
          v[c >> 1] = *reinterpret_cast<uint32_t*>(&h2);
        }
        tmem_st32(s_addr, v);
        tmem_st32(s_addr + 32, v + 32);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s.p_full[e]);
        const float2 rsum = __fadd2_rn(rs[0], rs[1]);
        l = l * factor + (rsum.x + rsum.y);
      }
      if (!ok) break;
      // ---------------- epilogue: O (complete after the unit's last P.V) -> output or partial
      if (!warp_wait(&s.pv_done[e], dc & 1u, &s.abort, 33)) { ok = false; break; }
      ++dc;
      tc_fence_after();
      bool write_out = true;
      float linv = 1.0f / l;
      if (un.n_chunks > 1) {
        // Split query tile: publish this chunk's partial -- its running max, row sum and
        // O / sum in fp16 (a weighted mean of V rows, rounded 2^-11 relative, far below
        // the bf16 output's 2^-8) -- and let the chunk that finishes last combine.
        const int slot = u * 2 + e;
        float* st_m = reinterpret_cast<float*>(args.ws + args.ws_stats_off) + (size_t)slot * 2 * kTile;
        uint4* op = reinterpret_cast<uint4*>(args.ws + args.ws_o_off) + (size_t)slot * (kTile * D / 8) + r;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t w[32];
          tmem_ld32(o_addr + c * 32, w);
          tmem_wait_ld();
#pragma unroll
          for (int g = 0; g < 4; ++g) {  // layout [col/8][row][8]: a warp stores 512 contiguous bytes
            uint32_t hv[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
              __half2 h = __floats2half2_rn(__uint_as_float(w[8 * g + 2 * k2]) * linv,
                                            __uint_as_float(w[8 * g + 2 * k2 + 1]) * linv);
              hv[k2] = *reinterpret_cast<uint32_t*>(&h);
            }
            op[(size_t)(c * 4 + g) * kTile] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&s.o_free[e]);  // the next unit's first P.V may overwrite O_e
        st_m[r] = m_ref;
        st_m[kTile + r] = l;
        __threadfence();
        mbar_arrive(&s.eng_sync[e]);
        if (!warp_wait(&s.eng_sync[e], xc & 1u, &s.abort, 36)) { ok = false; break; }
        ++xc;
        int* counter = reinterpret_cast<int*>(args.ws) + un.head * q_tiles + qe;
        if ((threadIdx.x & (kEngineThreads - 1)) == 0) s.flag[e] = atomicAdd(counter, 1);
        mbar_arrive(&s.eng_sync[e]);
        if (!warp_wait(&s.eng_sync[e], xc & 1u, &s.abort, 37)) { ok = false; break; }
        ++xc;
        int n_e = 0;  // chunks of this pair that cover keys of engine e's query tile
        for (int c = 0; c < un.n_chunks; ++c)
          if (c * args.chunk <= qe) ++n_e;
        write_out = (s.flag[e] == n_e - 1);
        if (write_out) {
          // Combine every chunk's partial, this one's included, read back in chunk order:
          // the sum does not depend on which chunk finished last.
          __threadfence();
          const float* ws_stats = reinterpret_cast<const float*>(args.ws + args.ws_stats_off);
          const uint4* ws_o = reinterpret_cast<const uint4*>(args.ws + args.ws_o_off);
          float mc[kMaxChunks], lc[kMaxChunks];
          size_t sl[kMaxChunks];
          float mmax = -INFINITY;
#pragma unroll
          for (int c = 0; c < kMaxChunks; ++c) {
            sl[c] = (size_t)(((un.v0 + min(c, n_e - 1)) * heads + un.head) * 2 + e);
            mc[c] = c < n_e ? __ldcg(ws_stats + sl[c] * 2 * kTile + r) : -INFINITY;
            lc[c] = c < n_e ? __ldcg(ws_stats + sl[c] * 2 * kTile + kTile + r) : 0.f;
            mmax = fmaxf(mmax, mc[c]);
          }
          float wc[kMaxChunks], lsum = 0.f;
#pragma unroll
          for (int c = 0; c < kMaxChunks; ++c) {
            wc[c] = c < n_e ? fast_exp2(mc[c] - mmax) * lc[c] : 0.f;
            lsum += wc[c];
          }
          const float inv = 1.0f / lsum;
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            uint4 t[kMaxChunks][4];  // every chunk's 32 columns of this row, loads all in flight
#pragma unroll
            for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
              for (int g = 0; g < 4; ++g)
                t[c][g] = c < n_e ? __ldcg(ws_o + sl[c] * (kTile * D / 8) + (size_t)(cc * 4 + g) * kTile + r)
                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int c = 0; c < kMaxChunks; ++c) {
                const __half2* h = reinterpret_cast<const __half2*>(&t[c][g]);
#pragma unroll
                for (int k2 = 0; k2 < 4; ++k2) {
                  const float2 x = __half22float2(h[k2]);
                  f[2 * k2] = fmaf(x.x, wc[c], f[2 * k2]);
                  f[2 * k2 + 1] = fmaf(x.y, wc[c], f[2 * k2 + 1]);
                }
              }
#pragma unroll
              for (int k2 = 0; k2 < 8; ++k2) f[k2] *= inv;
              const int c8 = cc * 4 + g;  // 16-byte chunk index within the output row
              uint8_t* rowp = s.q[e] + (c8 / 8) * (kTile * 128) + r * 128;
              *reinterpret_cast<uint4*>(rowp + (((c8 & 7) ^ sw) * 16)) = pack16<bf16>(f);
            }
          }
          if ((threadIdx.x & (kEngineThreads - 1)) == 0) *counter = 0;  // ready for the next launch
        }
      } else {
        // stage the bf16 output tile in this engine's Q buffer (its MMAs are complete) in
        // the 128-byte-swizzled layout of the output map
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t w[32];
          tmem_ld32(o_addr + cc * 32, w);
          tmem_wait_ld();
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float f[8];
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) f[k2] = __uint_as_float(w[q4 * 8 + k2]) * linv;
            const int c8 = cc * 4 + q4;
            uint8_t* rowp = s.q[e] + (c8 / 8) * (kTile * 128) + r * 128;
            *reinterpret_cast<uint4*>(rowp + (((c8 & 7) ^ sw) * 16)) = pack16<bf16>(f);
          }
        }
        tc_fence_before();
        mbar_arrive(&s.o_free[e]);  // the next unit's first P.V may overwrite O_e
      }
      if (write_out) {
        // TMA store of the staged tile; rows past seq are clipped by the TMA unit
        fence_proxy_async_smem();
        mbar_arrive(&s.eng_sync[e]);
        if (!warp_wait(&s.eng_sync[e], xc & 1u, &s.abort, 38)) { ok = false; break; }
        ++xc;
        if ((threadIdx.x & (kEngineThreads - 1)) == 0) {
#pragma unroll
          for (int c = 0; c < kSub; ++c) tma_store_3d(&map_o, s.q[e] + c * (kTile * 128), c * 64, qe * kTile, un.head);
          tma_store_commit();
          tma_store_wait_read();
        }
      }
      // the Q buffer may be refilled once the output staging has been read
      if ((threadIdx.x & (kEngineThreads - 1)) == 0) mbar_arrive(&s.q_empty[e]);
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

inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

// Work decomposition and CTA schedule, shared by the workspace-size query and the launch.
struct AttnPlan {
  int q_tiles = 0, pairs = 0, chunk = 0, units = 0, ctas = 0;
  size_t stats_off = 0, o_off = 0, ws_bytes = 0;  // ws_bytes == 0: no split, no workspace
  std::vector<uint16_t> cta_off, unit_list;       // empty: round-robin over CTAs
};

// Cost of a unit in "engine tiles" (tensor-core and exp work scale with the key tiles
// both engines process), plus a fixed charge for the unit's prologue and epilogue
// and, when split, for publishing and combining partials.
inline int unit_cost(const Unit& un, int q_tiles) {
  int c = 3;
  for (int e = 0; e < 2; ++e) {
    const int qe = 2 * un.pm + e;
    if (qe < q_tiles) c += std::max(0, std::min(un.n, qe + 1 - un.j0));
  }
  return c + (un.n_chunks > 1 ? 2 : 0);
}

// Longest-processing-time assignment of units to `ctas` CTAs; returns the makespan and
// (optionally) fills the per-CTA lists.
inline long lpt_schedule(int heads, int pairs, int q_tiles, int C, int units, int ctas, AttnPlan* out) {
  std::vector<std::pair<int, int>> cost(units);  // (cost, unit)
  for (int u = 0; u < units; ++u) cost[u] = {unit_cost(decode_unit(u, heads, pairs, q_tiles, C), q_tiles), u};
  std::stable_sort(cost.begin(), cost.end(), [](const std::pair<int, int>& a, const std::pair<int, int>& b) {
    return a.first > b.first;
  });
  std::vector<long> load(ctas, 0);
  std::vector<std::vector<uint16_t>> lists(out ? ctas : 0);
  for (const auto& cu : cost) {
    int best = 0;
    for (int b = 1; b < ctas; ++b)
      if (load[b] < load[best]) best = b;
    load[best] += cu.first;
    if (out) lists[best].push_back((uint16_t)cu.second);
  }
  if (out) {
    out->cta_off.assign(1, 0);
    out->unit_list.clear();
    for (int b = 0; b < ctas; ++b) {
      out->unit_list.insert(out->unit_list.end(), lists[b].begin(), lists[b].end());
      out->cta_off.push_back((uint16_t)out->unit_list.size());
    }
  }
  return *std::max_element(load.begin(), load.end());
}

inline int count_units(int heads, int pairs, int q_tiles, int C) {
  int per_head = 0;
  for (int pm = 0; pm < pairs; ++pm) per_head += (pair_tiles(pm, q_tiles) + C - 1) / C;
  return heads * per_head;
}

AttnPlan plan_attention(int heads, int seq, int d, bool allow_split, int sms) {
  AttnPlan p;
  p.q_tiles = (seq + kTile - 1) / kTile;
  p.pairs = (p.q_tiles + 1) / 2;
  const int max_nt = pair_tiles(p.pairs - 1, p.q_tiles);
  // Candidate chunk sizes: the whole key range (no split), or any smaller chunk when a
  // workspace is available and the units fit the schedule table.
  long best_span = -1;
  int best_c = max_nt;
  const int min_c = (max_nt + kMaxChunks - 1) / kMaxChunks;
  for (int C = max_nt; C >= min_c; --C) {
    if (C < max_nt && !allow_split) break;
    const int units = count_units(heads, p.pairs, p.q_tiles, C);
    if (units > kMaxSched) {
      if (C == max_nt) { best_c = C; best_span = -1; }
      break;
    }
    const int ctas = std::min(units, sms);
    const long span = lpt_schedule(heads, p.pairs, p.q_tiles, C, units, ctas, nullptr);
    if (best_span < 0 || span < best_span) {
      best_span = span;
      best_c = C;
    }
  }
  p.chunk = best_c;
  p.units = count_units(heads, p.pairs, p.q_tiles, p.chunk);
  p.ctas = std::min(p.units, sms);
  if (p.units <= kMaxSched && p.ctas <= kMaxCtas) lpt_schedule(heads, p.pairs, p.q_tiles, p.chunk, p.units, p.ctas, &p);
  if (p.chunk < max_nt) {
    p.stats_off = round256((size_t)heads * p.q_tiles * sizeof(int));
    p.o_off = p.stats_off + round256((size_t)p.units * 2 * 2 * kTile * sizeof(float));
    p.ws_bytes = p.o_off + (size_t)p.units * 2 * kTile * (size_t)d * sizeof(__half);
  }
  return p;
}

// Plans are cached per (heads, seq, d, split, SMs); the LPT search costs a few ms.
const AttnPlan& cached_plan(int heads, int seq, int d, bool allow_split) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, bool, int>, AttnPlan> cache;
  const int sms = sm_count();
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_tuple(heads, seq, d, allow_split, sms);
  auto it = cache.find(key);
  if (it == cache.end()) it = cache.emplace(key, plan_attention(heads, seq, d, allow_split, sms)).first;
  return it->second;
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
  const AttnPlan& plan = cached_plan(heads, seq, D, ws != nullptr);
  if (plan.ws_bytes > 0 && ws_bytes < plan.ws_bytes)
    return fail(NKL_ERR_ARG, "nkl_attention_ws: workspace %zu B < required %zu B", ws_bytes, plan.ws_bytes);
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
  a.ws = plan.ws_bytes > 0 ? static_cast<unsigned char*>(ws) : nullptr;
  a.heads = heads;
  a.q_tiles = plan.q_tiles;
  a.pairs = plan.pairs;
  a.chunk = plan.chunk;
  a.units = plan.units;
  a.scale_log2 = scale * kLog2e;
  a.ws_stats_off = plan.stats_off;
  a.ws_o_off = plan.o_off;
  a.n_ctas_listed = plan.cta_off.empty() ? 0 : plan.ctas;
  for (size_t i = 0; i < plan.cta_off.size(); ++i) a.cta_off[i] = plan.cta_off[i];
  for (size_t i = 0; i < plan.unit_list.size(); ++i) a.unit_list[i] = plan.unit_list[i];
  attn_fwd_bf16_kernel<D><<<plan.ctas, kAttnThreads, smem, st>>>(mq, mk, mv, mo, a);
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
  return cached_plan((int)heads, (int)seq, (int)head_dim, true).ws_bytes;
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
