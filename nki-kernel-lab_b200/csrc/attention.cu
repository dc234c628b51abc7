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
// As in the reference (attention.py:224-245), P is taken relative to the running max
// m updated on every key tile, and O and l are multiplied by exp(m_old - m_new) whenever
// m grows (the reference multiplies on every tile; where m is unchanged the factor is 1),
// so P is rounded to bf16 at the reference's scale.
//
// bf16 kernel (sm_100a): persistent, one CTA per SM.
//   work unit  (head, query tile, chunk of its causal key range); the host orders units
//              longest first and assigns them to CTAs greedily (LPT). A query tile whose
//              key range is split over several units writes partial (O / sum, max, sum)
//              to a workspace; a second kernel (programmatic dependent launch) merges
//              the partials in chunk order, so the result does not depend on the schedule
//   warps 0-7  softmax engine: two warps per TMEM lane quadrant, each taking 64 of the
//              128 keys of every score row (row maxima and sums exchanged through shared
//              memory). Per key tile: tcgen05.ld of the scores, row max, rescale of
//              O in TMEM, exp2 with the scale folded into one FMA, P (bf16 pairs)
//              written back over the score columns with tcgen05.st
//   warp 8     TMA producer: Q per unit (double buffered), K and V through 2-deep rings
//   warp 9     TMEM allocator + single-thread tcgen05.mma issuer. S is double buffered
//              in TMEM: S(t+2) = Q K(t+2)^T is issued right behind O += P(t) V(t), so the
//              tensor core computes the next tile's scores while the engine exponentiates.
//              Both products take their A operand from TMEM (Q and P), so shared memory
//              only supplies K and V to the tensor core; the engine copies each unit's Q
//              from shared memory into TMEM before the previous unit's epilogue
//   TMEM       S/P buffers [0,128) and [128,256), O [256, 256+d), Q [256+d, 256+2d) (two
//              buffers of d/2 columns of bf16 pairs)
//   epilogue   O from TMEM, * 1/l, bf16, staged in the unit's Q buffer, TMA store
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <vector>

#include <cuda_fp16.h>

#include <atomic>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace nkl {
namespace {

__device__ unsigned int g_attn_dev_error = 0;

using namespace sm100;

constexpr int kTile = 128;  // query / key tile, as the reference's T (attention.py:24)
constexpr int kEngineWarps = 8;  // two warps per TMEM lane quadrant, each taking half of every row
constexpr int kEngineThreads = kEngineWarps * 32;
constexpr int kProducerWarp = kEngineWarps;
constexpr int kMmaWarp = kEngineWarps + 1;
constexpr int kAttnThreads = kEngineThreads + 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxCtas = 192;         // schedule table capacity (>= SMs of any sm_100 part)
constexpr int kMaxSched = 1024;       // units listed explicitly; more units: round-robin
constexpr int kMaxChunks = 8;         // a query tile's key range is split into at most 8 units

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (lo, hi) for fma.rn.f32x2 / add.rn.f32x2: each lane is an ordinary fp32
// FMA / add, so the values equal those of the scalar forms, with half the instructions.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2_pack(float lo, float hi) {
  return ((f32x2)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ f32x2 f2_pack_bits(uint32_t lo, uint32_t hi) { return ((f32x2)hi << 32) | lo; }
__device__ __forceinline__ float f2_lo(f32x2 a) { return __uint_as_float((uint32_t)a); }
__device__ __forceinline__ float f2_hi(f32x2 a) { return __uint_as_float((uint32_t)(a >> 32)); }
__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 f2_add(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// P = 2^(s * scale_log2 - m) for the scores v[0..N), packed as bf16 pairs into v[0..N/2)
// (pair (c, c+1) lands in v[c/2], a score already consumed). The row sum runs in `acc`
// packed accumulators (acc = 1 or 2); accumulator j's lanes take the pairs with
// (c/2) % acc == j, low lane the even scores, high lane the odd ones. Returns the
// accumulators themselves so each caller combines them in its own order.
template <int N, int ACC>
__device__ __forceinline__ void exp_pack(uint32_t* v, float scale_log2, float neg_m, f32x2 (&rs)[ACC]) {
  const f32x2 k2 = f2_pack(scale_log2, scale_log2), m2 = f2_pack(neg_m, neg_m);
#pragma unroll
  for (int j = 0; j < ACC; ++j) rs[j] = 0ull;
#pragma unroll
  for (int c = 0; c < N; c += 2) {
    const f32x2 x2 = f2_fma(f2_pack_bits(v[c], v[c + 1]), k2, m2);
    const float p0 = fast_exp2(f2_lo(x2)), p1 = fast_exp2(f2_hi(x2));
    rs[(c >> 1) % ACC] = f2_add(rs[(c >> 1) % ACC], f2_pack(p0, p1));
    __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
    v[c >> 1] = *reinterpret_cast<uint32_t*>(&h2);
  }
}

// Marks r[0..N) as defined here: placed after tcgen05.wait::ld, it keeps every use of
// registers written by an asynchronous tcgen05.ld behind the wait that completes it.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Named barrier (ids 1..4) for the two engine warps that share a TMEM lane quadrant.
__device__ __forceinline__ void pair_sync(int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

// Max of 64 fp32 scores held as bits.
__device__ __forceinline__ float max64(const uint32_t* v) {
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < 64; c += 8)
#pragma unroll
    for (int a = 0; a < 4; ++a) mx[a] = max3f(mx[a], __uint_as_float(v[c + 2 * a]), __uint_as_float(v[c + 2 * a + 1]));
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// P = 2^(s * scale_log2 - m) for the 64 scores in v[0..64), packed as bf16 pairs into
// v[0..32) (pair (c, c+1) lands in v[c/2], a score already consumed); returns the fp32
// sum of the 64 values.
__device__ __forceinline__ float exp_pack64(uint32_t* v, float scale_log2, float neg_m) {
  f32x2 rs[1];
  exp_pack<64, 1>(v, scale_log2, neg_m, rs);
  return f2_lo(rs[0]) + f2_hi(rs[0]);
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
  uint8_t q[2][kTileBytes];  // Q double buffer: D/64 sub-tiles of [128 rows x 128 B]; output staging
  uint8_t k[2][kTileBytes];  // key ring, K-major (head_dim contiguous)
  uint8_t v[2][kTileBytes];  // value ring, N-major for the P.V product
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];  // S(t) ready in TMEM buffer t & 1 (global tile count t)
  uint64_t p_full[2];  // P(t) ready in buffer t & 1 (all engine threads)
  uint64_t pv_step;    // one phase per P.V tile
  uint64_t pv_done;    // one phase per unit: its last P.V complete
  uint64_t o_free;     // engine has read O (all engine threads)
  uint64_t mma_done;
  float xmax[2][2 * kTile];  // [tile parity][half * 128 + row]: row-max exchange
  float xsum[2 * kTile];     // [half * 128 + row]: row-sum exchange
  uint32_t tmem_base;
  int abort;
};

template <int D>
constexpr size_t attn_smem_bytes() {
  return sizeof(AttnSmem<D>);
}

// ---- split-KV work units
struct AttnArgs {
  unsigned char* ws;  // NULL when no query tile is split
  int heads, q_tiles, chunk, units;
  int kv_group;  // query heads per key/value head (1 = multi-head, heads = multi-query)
  int seq;
  float scale_log2;
  size_t ws_stats_off, ws_o_off;  // byte offsets of the partial (max, sum) and O regions
  int n_ctas_listed;              // > 0: cta_off / unit_desc give each CTA's units
  uint16_t cta_off[kMaxCtas + 1];
  // Units decoded on the host, packed in two words:
  //   a = unit (10 bits) | head << 10 (11 bits) | kv head << 21 (11 bits)
  //   b = query tile (11 bits) | first key tile << 11 (11 bits) | (key tiles - 1) << 22
  // (listed plans have at most kMaxSched = 1024 units, so every field fits). Decoding on
  // the device would cost a chain of integer divisions per unit, and on sm_100 those issue
  // on the MUFU pipe that the softmax warps keep saturated with ex2: the producer and
  // MMA warps stalled ~2 us at every unit boundary behind them.
  uint2 unit_desc[kMaxSched];
};

// Extra output destinations for the head-sharded all-gather (nkl_attention_allgather): the
// other GPUs' output buffers, written through NVLink by the same epilogue that writes this
// GPU's, at head index local head + head_offset (also in this GPU's buffer).
constexpr int kMaxPeers = 7;
struct PeerOut {
  CUtensorMap map[kMaxPeers];  // peers' [heads_total, seq, d] outputs, same layout as map_o
  int n;                       // peer destinations (0: none)
  int head_offset;
};

struct Unit {
  int head, qt, chunk, n_chunks, j0, n, v0;  // v0: per-head index of this query tile's chunk 0
};

// What the kernel needs of a unit: its index (workspace slot), heads, query tile and key
// tile range; split = the unit covers only part of its query tile's causal key range.
struct UnitRun {
  int u, head, kv_head, qt, j0, n;
  bool split;
};

__host__ __device__ __forceinline__ uint2 pack_unit(int u, int head, int kv_head, int qt, int j0, int n) {
  return make_uint2((uint32_t)u | ((uint32_t)head << 10) | ((uint32_t)kv_head << 21),
                    (uint32_t)qt | ((uint32_t)j0 << 11) | ((uint32_t)(n - 1) << 22));
}

// Unit index -> (head, query tile, chunk). Units run head-fastest; query tiles longest
// (latest) first; chunks of C key tiles ascending.
__host__ __device__ __forceinline__ Unit decode_unit(int u, int heads, int q_tiles, int C) {
  Unit r;
  r.head = u % heads;
  const int v = u / heads;
  if (C >= q_tiles) {  // no split: one unit per query tile
    r.qt = q_tiles - 1 - v;
    r.chunk = 0;
    r.n_chunks = 1;
    r.j0 = 0;
    r.n = r.qt + 1;
    r.v0 = v;
    return r;
  }
  int base = 0;
  for (int qt = q_tiles - 1; qt >= 0; --qt) {
    const int c = (qt + C) / C;  // ceil((qt + 1) / C)
    if (v < base + c) {
      r.qt = qt;
      r.chunk = v - base;
      r.n_chunks = c;
      r.j0 = r.chunk * C;
      r.n = (C < qt + 1 - r.j0) ? C : qt + 1 - r.j0;
      r.v0 = base;
      return r;
    }
    base += c;
  }
  r.qt = -1;
  return r;
}

// Wait by lane 0, then broadcast, so the whole warp stays converged for the
// .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, &g_attn_dev_error, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// The i-th unit of this CTA: from the host-decoded list, or (plans too large to list)
// round-robin over CTAs, decoded here once per unit.
__device__ __forceinline__ bool next_unit(const AttnArgs& a, int i, UnitRun& r) {
  if (a.n_ctas_listed > 0) {
    const int k = a.cta_off[blockIdx.x] + i;
    if (k >= a.cta_off[blockIdx.x + 1]) return false;
    const uint2 d = a.unit_desc[k];
    r.u = (int)(d.x & 1023u);
    r.head = (int)((d.x >> 10) & 2047u);
    r.kv_head = (int)(d.x >> 21);
    r.qt = (int)(d.y & 2047u);
    r.j0 = (int)((d.y >> 11) & 2047u);
    r.n = (int)(d.y >> 22) + 1;
  } else {
    r.u = (int)blockIdx.x + i * (int)gridDim.x;
    if (r.u >= a.units) return false;
    const Unit un = decode_unit(r.u, a.heads, a.q_tiles, a.chunk);
    r.head = un.head;
    r.kv_head = un.head / a.kv_group;
    r.qt = un.qt;
    r.j0 = un.j0;
    r.n = un.n;
  }
  r.split = !(r.j0 == 0 && r.n == r.qt + 1);
  return true;
}

// TMA producer (one warp): per unit, in the order the MMA warp consumes them: K(0), Q,
// K(1), then V(t) followed by K(t+2); Q double buffered, K and V through 2-deep rings.
// Shared by the flash kernels whose shared-memory layout names these buffers and barriers.
template <int D, class Smem>
__device__ __forceinline__ void attn_produce(Smem& s, const CUtensorMap* map_q, const CUtensorMap* map_k,
                                             const CUtensorMap* map_v, const AttnArgs& args) {
  constexpr uint32_t kTileBytes = kTile * D * 2;
  constexpr int kSub = D / 64;
  if (elect_one()) {
    uint32_t kc = 0, vc = 0, qc = 0;
    int k_armed[2] = {-1, -1}, v_armed[2] = {-1, -1}, q_armed[2] = {-1, -1};
    bool ok = true;
    UnitRun un;
    // Key / value tile `kt` (absolute key-tile index) of kv head `kvh`.
    auto load_k = [&](int kt, int kvh) -> bool {
      const int ks = kc & 1;
      if (!mbar_wait(&s.k_empty[ks], ((kc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 11)) return false;
      mbar_arrive_expect_tx(&s.k_full[ks], kTileBytes);
      k_armed[ks] = (int)((kc >> 1) & 1u);
      for (int c = 0; c < kSub; ++c)
        tma_load_3d(s.k[ks] + c * (kTile * 128), map_k, &s.k_full[ks], c * 64, kt * kTile, kvh);
      ++kc;
      return true;
    };
    auto load_v = [&](int kt, int kvh) -> bool {
      const int vs = vc & 1;
      if (!mbar_wait(&s.v_empty[vs], ((vc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 12)) return false;
      mbar_arrive_expect_tx(&s.v_full[vs], kTileBytes);
      v_armed[vs] = (int)((vc >> 1) & 1u);
      for (int c = 0; c < kSub; ++c)
        tma_load_3d(s.v[vs] + c * (kTile * 128), map_v, &s.v_full[vs], c * 64, kt * kTile, kvh);
      ++vc;
      return true;
    };
    // Per unit, in the order the MMA warp consumes them: K(0), Q, K(1), then V(t)
    // followed by K(t+2).
    for (int i = 0; ok && next_unit(args, i, un); ++i) {
      const int j0 = un.j0, kvh = un.kv_head;
      ok = load_k(j0, kvh);
      if (ok) {
        const int qb = qc & 1;
        if (!mbar_wait(&s.q_empty[qb], ((qc >> 1) & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 10)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.q_full[qb], kTileBytes);
        q_armed[qb] = (int)((qc >> 1) & 1u);
        for (int c = 0; c < kSub; ++c)
          tma_load_3d(s.q[qb] + c * (kTile * 128), map_q, &s.q_full[qb], c * 64, un.qt * kTile, un.head);
        ++qc;
      }
      if (ok && un.n > 1) ok = load_k(j0 + 1, kvh);
      for (int t = 0; ok && t < un.n; ++t) {
        ok = load_v(j0 + t, kvh);
        if (ok && t + 2 < un.n) ok = load_k(j0 + t + 2, kvh);
      }
    }
    if (!ok) {  // let issued copies land before shared memory is released
      const uint64_t t0 = globaltimer();
      for (int b = 0; b < 2; ++b) {
        if (q_armed[b] >= 0)
          while (!mbar_try_wait(&s.q_full[b], (uint32_t)q_armed[b]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        if (k_armed[b] >= 0)
          while (!mbar_try_wait(&s.k_full[b], (uint32_t)k_armed[b]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        if (v_armed[b] >= 0)
          while (!mbar_try_wait(&s.v_full[b], (uint32_t)v_armed[b]) && globaltimer() - t0 < kWaitTimeoutNs) {}
      }
    }
  }
  __syncwarp();  // the warp reconverges here: the CTA barrier below must see all 32 lanes
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_fwd_bf16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                     const __grid_constant__ AttnArgs args, const __grid_constant__ PeerOut peers) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicCAS(&g_attn_dev_error, 0u, 40u);
    return;
  }
  // The split-KV combine kernel, launched next with programmatic dependent launch, may be
  // scheduled now; it waits in griddepcontrol.wait until this grid has completed.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  auto& s = *reinterpret_cast<AttnSmem<D>*>(smem_raw);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kOCol0 = 2 * kTile;  // S/P buffers at [0,128) and [128,256)
  constexpr uint32_t kQtCol0 = kOCol0 + D;  // Q buffers (bf16 pairs) at kQtCol0 + b * D / 2
  constexpr uint32_t kIdescS = idesc_bf16_f32(kTile, kTile, false, false);
  constexpr uint32_t kIdescPV = idesc_bf16_f32(kTile, D, false, true);
  constexpr int kSub = D / 64;  // 64-column (128-byte) sub-tiles per Q/K/V tile
  static_assert(kQtCol0 + D <= kTmemCols, "TMEM columns");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float scale_log2 = args.scale_log2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 4);  // one arrival per TMEM lane quadrant
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], kEngineThreads);
    }
    mbar_init(&s.pv_step, 1);
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
  // Launched with programmatic dependent launch: the prologue above (barriers, TMEM,
  // descriptor prefetch) overlaps the previous kernel of the stream; nothing in global
  // memory (q, k, v, the output, the workspace a previous combine kernel may still be
  // reading) is read or written before that kernel has completed and its writes are
  // visible. Before waiting, the producer asks L2 to prefetch the first unit's Q, K and
  // V tiles: a prefetch only warms L2, the point of coherence, so a tile the previous
  // kernel is still writing is read correctly by the loads after the wait; it just lets
  // those first loads hit L2 instead of HBM.
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
    // ------------------------------------------------ TMA producer
    attn_produce<D>(s, &map_q, &map_k, &map_v, args);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (elect_one()) {
      uint32_t kc = 0, vc = 0, qc = 0, gt = 0, uc = 0;
      const uint64_t k_desc0 = smem_desc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t k_desc1 = smem_desc_sw128(smem_u32(s.k[1]), 16, 1024);
      const uint64_t v_desc0 = smem_desc_sw128(smem_u32(s.v[0]), kTile * 128, 1024);
      const uint64_t v_desc1 = smem_desc_sw128(smem_u32(s.v[1]), kTile * 128, 1024);
      bool ok = true;
      // S into TMEM buffer b from Q buffer qb and K stage ks
      // S into TMEM buffer b from the unit's Q in TMEM buffer qb (A operand) and K stage ks
      auto issue_s = [&](int qb, int ks, int b) {
        const uint64_t kd = ks ? k_desc1 : k_desc0;
        const uint32_t qt = tmem + kQtCol0 + (uint32_t)(qb * (D / 2));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4);
          mma_bf16_ts(tmem + (uint32_t)(b * kTile), qt + (uint32_t)(kk * 8), kd + off, kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full[b]);
      };
      UnitRun un;
      for (int i = 0; ok && next_unit(args, i, un); ++i) {
        const int n = un.n;
        const int qb = qc & 1;
        // The unit's Q into TMEM buffer qb as the A operand of Q K^T (row r in lane r, bf16
        // pairs (2j, 2j+1) in column j): one 128 x 32-byte copy per 16-column K step, from
        // the same swizzled slices an SS-form MMA would read. The S MMAs below follow the
        // copies in issue order. Buffer qb was last read by the S MMAs of the unit before
        // the previous one, all complete (their scores have been consumed).
        if (!mbar_wait(&s.q_full[qb], (qc >> 1) & 1u, &s.abort, &g_attn_dev_error, 20)) { ok = false; break; }
        tc_fence_after();
        {
          const uint64_t q_desc = smem_desc_sw128(smem_u32(s.q[qb]), 16, 1024);
          const uint32_t qt = tmem + kQtCol0 + (uint32_t)(qb * (D / 2));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            tmem_cp_128x256b(qt + (uint32_t)(kk * 8), q_desc + (uint32_t)(((kk >> 2) * (kTile * 128) + (kk & 3) * 32) >> 4));
        }
        ++qc;
        for (int t = 0; t < n && t < 2; ++t) {  // S for the unit's first two key tiles
          const uint32_t ki = kc + (uint32_t)t;
          if (!mbar_wait(&s.k_full[ki & 1], (ki >> 1) & 1u, &s.abort, &g_attn_dev_error, 21)) { ok = false; break; }
          tc_fence_after();
          issue_s(qb, ki & 1, (gt + t) & 1);
          mma_commit(&s.k_empty[ki & 1]);
        }
        for (int t = 0; ok && t < n; ++t) {
          const uint32_t G = gt + (uint32_t)t;
          const int b = G & 1;
          // V(t) and the free O (first tile of a unit) are normally ready long before P(t):
          // take those waits first, so only the P.V issue itself follows P(t).
          const uint32_t vi = vc + (uint32_t)t;
          if (!mbar_wait(&s.v_full[vi & 1], (vi >> 1) & 1u, &s.abort, &g_attn_dev_error, 24)) { ok = false; break; }
          if (t == 0 && !mbar_wait(&s.o_free, (uc & 1u) ^ 1u, &s.abort, &g_attn_dev_error, 23)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&s.p_full[b], (G >> 1) & 1u, &s.abort, &g_attn_dev_error, 22)) { ok = false; break; }
          tc_fence_after();
          const uint64_t vd = (vi & 1) ? v_desc1 : v_desc0;
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            mma_bf16_ts(tmem + kOCol0, tmem + (uint32_t)(b * kTile + kk * 8), vd + (uint32_t)(kk * 128), kIdescPV,
                        (t > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&s.pv_step);
          mma_commit(&s.v_empty[vi & 1]);
          if (t + 2 < n) {  // next-but-one S into this buffer, behind the P.V that reads its P
            const uint32_t ki = kc + (uint32_t)t + 2;
            if (!mbar_wait(&s.k_full[ki & 1], (ki >> 1) & 1u, &s.abort, &g_attn_dev_error, 25)) { ok = false; break; }
            tc_fence_after();
            issue_s(qb, ki & 1, b);
            mma_commit(&s.k_empty[ki & 1]);
          }
        }
        if (!ok) break;
        mma_commit(&s.pv_done);
        kc += (uint32_t)n;
        vc += (uint32_t)n;
        gt += (uint32_t)n;
        ++uc;
      }
      // Every MMA issued by this thread has completed once mma_done flips.
      mma_commit(&s.mma_done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
    }
    __syncwarp();  // the other lanes wait for the issuing lane before the CTA barrier and dealloc
  } else {
    // ------------------------------------------------ softmax engine (warps 0-7)
    // Warps w and w+4 share TMEM lane quadrant w: warp half hf takes keys hf*64 ..
    // hf*64+63 of every S tile and O columns hf*D/2 .. hf*D/2+D/2-1 in the epilogue.
    // Row maxima (per tile) and row sums (per unit) are exchanged through shared memory
    // under a named barrier of the pair.
    const int qd = warp & 3;
    const int hf = warp >> 2;
    const int r = qd * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + kOCol0 + (uint32_t)(hf * (D / 2));
    const int pair_id = 1 + qd;
    const int sw = r & 7;
    const bool quad_lead = hf == 0 && lane == 0;  // stores its quadrant's output rows, frees the Q buffer
    bool stored_any = false;
    uint32_t gt = 0, uc = 0;
    bool ok = true;
    UnitRun un;
    for (int i = 0; ok && next_unit(args, i, un); ++i) {
      const int u = un.u;
      const int qt = un.qt;
      float m_ref = -INFINITY, l = 0.f;  // l: this half's share of the row sum
      for (int t = 0; t < un.n; ++t) {
        const uint32_t G = gt + (uint32_t)t;
        const int b = G & 1;
        if (!warp_wait(&s.s_full[b], (G >> 1) & 1u, &s.abort, 31)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[64];
        const uint32_t s_addr = tmem + lane_off + (uint32_t)(b * kTile + hf * 64);
        tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        reg_fence<64>(v);
        if (un.j0 + t == qt) {  // diagonal tile: keys above the diagonal are masked
          const int lim = r - hf * 64;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c > lim) v[c] = __float_as_uint(-INFINITY);
        }
        // Row max over both halves. The pair barrier also guarantees that the partner
        // has read its scores before this warp's P overwrites columns 32..63.
        float* xm = s.xmax[b];
        xm[hf * kTile + r] = max64(v);
        pair_sync(pair_id);
        const float mx = fmaxf(xm[r], xm[kTile + r]) * scale_log2;
        // Exponents are taken against the running max m_ref; when it grows, O and l are
        // scaled by exp(m_old - m_new).
        float factor = 1.f;
        if (t == 0) {
          m_ref = mx;  // key 0 of the first tile is never masked: mx is finite
        } else if (mx > m_ref) {
          factor = fast_exp2(m_ref - mx);
          m_ref = mx;
        }
        const float rs = exp_pack64(v, scale_log2, -m_ref);
        tmem_st32(tmem + lane_off + (uint32_t)(b * kTile + hf * 32), v);  // P: bf16 pairs of this half's keys
        if (t > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
          // O *= factor before P.V(G) accumulates into it. O must hold P.V of every tile
          // before this one: wait for P.V(G-1), the one that may still be running
          // (P.V(G-2) completed before S(G) was computed); by now it usually has. Done
          // after the P store so the scores' registers can take this half's D/2 O columns
          // in one TMEM round trip.
          if (!warp_wait(&s.pv_step, (G - 1) & 1u, &s.abort, 32)) { ok = false; break; }
          tc_fence_after();
          tmem_wait_st();  // the P store has read its source registers
#pragma unroll
          for (int c = 0; c < D / 64; ++c) tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
          tmem_wait_ld();
          reg_fence<D / 2>(v);
#pragma unroll
          for (int k2 = 0; k2 < D / 2; k2 += 2) {  // O *= factor, two columns per mul.rn.f32x2
            const f32x2 o2 = f2_mul(f2_pack_bits(v[k2], v[k2 + 1]), f2_pack(factor, factor));
            v[k2] = (uint32_t)o2;
            v[k2 + 1] = (uint32_t)(o2 >> 32);
          }
#pragma unroll
          for (int c = 0; c < D / 64; ++c) tmem_st32(o_addr + c * 32, v + c * 32);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s.p_full[b]);
        l = l * factor + rs;
      }
      if (!ok) break;
      // ---------------- epilogue: O (complete after the unit's last P.V) -> output or partial
      if (!warp_wait(&s.pv_done, uc & 1u, &s.abort, 33)) { ok = false; break; }
      tc_fence_after();
      uint32_t w[D / 2];  // this half's O columns, one TMEM load batch
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&w[c * 32]));
      tmem_wait_ld();
      reg_fence<D / 2>(w);
      tc_fence_before();
      mbar_arrive(&s.o_free);  // the next unit's first P.V may overwrite O
      s.xsum[hf * kTile + r] = l;
      pair_sync(pair_id);
      const float lt = s.xsum[r] + s.xsum[kTile + r];
      const float linv = 1.0f / lt;
      const int qb = uc & 1;  // this unit's Q buffer
      if (un.split) {
        // Split query tile: this chunk's O / sum in fp32 and its (max, sum);
        // attn_combine_bf16_kernel merges the chunks once this kernel has completed.
        float4* op = reinterpret_cast<float4*>(args.ws + args.ws_o_off) + (size_t)u * (kTile * D / 4) + r;
#pragma unroll
        for (int g4 = 0; g4 < D / 8; ++g4)  // layout [col/4][row][4]: a warp stores 512 contiguous bytes
          op[(size_t)(hf * (D / 8) + g4) * kTile] =
              make_float4(__uint_as_float(w[4 * g4]) * linv, __uint_as_float(w[4 * g4 + 1]) * linv,
                          __uint_as_float(w[4 * g4 + 2]) * linv, __uint_as_float(w[4 * g4 + 3]) * linv);
        if (hf == 0) {
          float* st = reinterpret_cast<float*>(args.ws + args.ws_stats_off) + (size_t)u * 2 * kTile;
          st[r] = m_ref;
          st[kTile + r] = lt;
        }
      } else {
        // Stage the bf16 output tile in the unit's Q buffer (its MMAs are complete) in the
        // 128-byte-swizzled layout of the output map; then one TMA store per 64 columns.
#pragma unroll
        for (int g2 = 0; g2 < D / 16; ++g2) {
          const int g = hf * (D / 16) + g2;  // 16-byte chunk of the output row
          float f[8];
#pragma unroll
          for (int k2 = 0; k2 < 8; ++k2) f[k2] = __uint_as_float(w[8 * g2 + k2]) * linv;
          uint8_t* rowp = s.q[qb] + (g / 8) * (kTile * 128) + r * 128;
          *reinterpret_cast<uint4*>(rowp + (((g & 7) ^ sw) * 16)) = pack16<bf16>(f);
        }
        // Each lane quadrant stores its own 32 rows as soon as its two warps have staged
        // them (no CTA-wide barrier); rows past seq are clipped by the TMA unit.
        fence_proxy_async_smem();
        pair_sync(pair_id);
        const int row0 = qt * kTile + qd * 32;
        if (quad_lead && row0 < args.seq) {
          const int oh = un.head + peers.head_offset;
#pragma unroll
          for (int c = 0; c < kSub; ++c)
            tma_store_3d(&map_o, s.q[qb] + c * (kTile * 128) + qd * 32 * 128, c * 64, row0, oh);
          for (int p = 0; p < peers.n; ++p)  // the same staged rows into every peer's buffer
#pragma unroll
            for (int c = 0; c < kSub; ++c)
              tma_store_3d(&peers.map[p], s.q[qb] + c * (kTile * 128) + qd * 32 * 128, c * 64, row0, oh);
          tma_store_commit();
          tma_store_wait_read();
          stored_any = true;
        }
      }
      // the Q buffer may be refilled once every quadrant's output staging has been read
      if (quad_lead) mbar_arrive(&s.q_empty[qb]);
      gt += (uint32_t)un.n;
      ++uc;
    }
    // every output store, local and remote, has completed before the CTA exits
    if (stored_any) tma_store_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ split-KV combine
// A query tile whose key range was split over n_e units has n_e partials: (m_c, l_c) per
// row and O_c / l_c in fp32. The output row is sum_c w_c (O_c / l_c) / sum_c w_c with
// w_c = 2^(m_c - max m) l_c, summed in chunk order so the result does not depend on the
// schedule. One CTA of 64 threads covers 64 rows x 8 * (8 / NC) columns of one (job,
// head), so a thread holds 8 partial vectors whatever the chunk count; every
// partial's loads for a thread are issued together.

constexpr int kMaxCombineJobs = 1024;

struct CombineJob {
  uint16_t qt, v0;  // query tile; per-head index of its chunk-0 unit
  uint16_t n_e, pad;  // chunks covering the tile
};

struct CombineArgs {
  const unsigned char* ws;
  bf16* out;
  bf16* peer_out[kMaxPeers];  // the all-gather's peer destinations (n_peer of them)
  int n_peer, head_offset;    // output head = head + head_offset in every destination
  int heads, seq, n_jobs;
  size_t ws_stats_off, ws_o_off;
  int64_t o_ss, o_hs;  // output strides in elements: between rows (seq) and between heads
  CombineJob job[kMaxCombineJobs];
};

// NC: chunk slots, the smallest of 2, 4, 8 covering the plan (unused slots add exact
// zeros, so every NC gives the same bits).
template <int D, int NC>
__global__ void __launch_bounds__(64) attn_combine_bf16_kernel(const __grid_constant__ CombineArgs args) {
  constexpr int GPT = 8 / NC;  // 8-column groups per thread: every thread keeps 16 partial loads in flight
  pdl_enter();  // the attention grid before this one has completed and its partials are visible
  const CombineJob jb = args.job[blockIdx.x];
  const int head = blockIdx.y;
  const int r = (blockIdx.z & 1) * 64 + threadIdx.x;  // row within the query tile
  const int g0 = (blockIdx.z >> 1) * GPT;              // first 8-column group of the slice
  const int row = jb.qt * kTile + r;
  if (row >= args.seq) return;
  const size_t stride = (size_t)args.heads;  // unit step between consecutive chunks
  const size_t slot0 = (size_t)jb.v0 * args.heads + head;
  const float* stats = reinterpret_cast<const float*>(args.ws + args.ws_stats_off);
  const float4* po = reinterpret_cast<const float4*>(args.ws + args.ws_o_off);
  float4 t[NC][GPT][2];
  float mc[NC], lc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const bool in = c < jb.n_e;
    const size_t sl = slot0 + (size_t)(in ? c : 0) * stride;
    mc[c] = in ? __ldcg(stats + sl * 2 * kTile + r) : -INFINITY;
    lc[c] = in ? __ldcg(stats + sl * 2 * kTile + kTile + r) : 0.f;
#pragma unroll
    for (int g = 0; g < GPT; ++g)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        t[c][g][h] = in ? __ldcg(po + sl * (kTile * D / 4) + (size_t)(2 * (g0 + g) + h) * kTile + r)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mmax = -INFINITY;
#pragma unroll
  for (int c = 0; c < NC; ++c) mmax = fmaxf(mmax, mc[c]);
  float wc[NC], lsum = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    wc[c] = c < jb.n_e ? fast_exp2(mc[c] - mmax) * lc[c] : 0.f;
    lsum += wc[c];
  }
  const float inv = 1.0f / lsum;
  const size_t o_off = (size_t)(head + args.head_offset) * args.o_hs + (size_t)row * args.o_ss + g0 * 8;
  uint4* dst = reinterpret_cast<uint4*>(args.out + o_off);
#pragma unroll
  for (int g = 0; g < GPT; ++g) {
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        f[4 * h + 0] = fmaf(t[c][g][h].x, wc[c], f[4 * h + 0]);
        f[4 * h + 1] = fmaf(t[c][g][h].y, wc[c], f[4 * h + 1]);
        f[4 * h + 2] = fmaf(t[c][g][h].z, wc[c], f[4 * h + 2]);
        f[4 * h + 3] = fmaf(t[c][g][h].w, wc[c], f[4 * h + 3]);
      }
    }
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) f[k2] *= inv;
    const uint4 packed = pack16<bf16>(f);
    dst[g] = packed;
    for (int p = 0; p < args.n_peer; ++p) reinterpret_cast<uint4*>(args.peer_out[p] + o_off)[g] = packed;
  }
}

#include "attention_pair.cuh"
#include "attention_pp.cuh"

// ------------------------------------------------------------------ fp32 exact flash kernel
// CUDA-core flash attention for fp32 inputs (the reference's fp32 tests need 2e-5
// absolute agreement with PyTorch SDPA, beyond TF32 tensor cores). A block of 4 warps
// owns 16 query rows (4 per warp); key/value tiles of 32 rows are staged in shared
// memory; lane k scores key k, lane c accumulates output columns c, c+32, ...

constexpr int kF32Rows = 16;
constexpr int kF32Keys = 32;

__global__ void __launch_bounds__(128)
attn_fwd_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    float* __restrict__ out, int seq, int d, float scale, int kv_group) {
  __shared__ float ks[kF32Keys][129];
  __shared__ float vs[kF32Keys][128];
  __shared__ float qs[kF32Rows][128];
  const int head = blockIdx.y;
  const int r0 = blockIdx.x * kF32Rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qh = q + (int64_t)head * seq * d;
  const float* kh = k + (int64_t)(head / kv_group) * seq * d;
  const float* vh = v + (int64_t)(head / kv_group) * seq * d;
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

// [heads, seq, d] bf16 with the given seq and head strides (elements; d is contiguous),
// moved in boxes of 64 columns x box_rows rows.
int make_qkv_map(CUtensorMap* m, const void* base, int heads, int seq, int d, int64_t seq_stride,
                 int64_t head_stride, const char* what, int box_rows = kTile) {
  const uint64_t dims[3] = {(uint64_t)d, (uint64_t)seq, (uint64_t)heads};
  const uint64_t strides[2] = {(uint64_t)seq_stride * 2, (uint64_t)head_stride * 2};
  const uint32_t box[3] = {64, (uint32_t)box_rows, 1};
  return make_tensor_map_bf16(m, base, 3, dims, strides, box, what);
}

inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

// Element strides of q, k, v and out: between consecutive rows of a head (seq) and
// between heads; the head dimension is contiguous. Contiguous [heads, seq, d] tensors
// have seq stride d and head stride seq * d.
struct AttnLayout {
  int64_t q_ss, q_hs, k_ss, k_hs, v_ss, v_hs, o_ss, o_hs;
};
inline AttnLayout contiguous_layout(int64_t seq, int64_t d) {
  return AttnLayout{d, seq * d, d, seq * d, d, seq * d, d, seq * d};
}

// Work decomposition and CTA schedule, shared by the workspace-size query and the launch.
struct AttnPlan {
  int q_tiles = 0, chunk = 0, units = 0, ctas = 0;
  size_t stats_off = 0, o_off = 0, ws_bytes = 0;  // ws_bytes == 0: no split, no workspace
  std::vector<uint16_t> cta_off;                  // empty: round-robin over CTAs
  std::vector<uint2> unit_desc;                   // per listed unit, in cta_off order
  std::vector<CombineJob> jobs;                   // split query tiles (one job per tile, all heads)
  int max_chunks = 1;                             // most chunks of any split tile
};

// Cost of a unit in key tiles (tensor-core and exp work scale with them), plus a fixed
// charge for the unit's Q load, first scores and epilogue.
inline int unit_cost(const Unit& un) { return 2 + un.n; }

// Charge, in the same units, for the combine kernel that follows a split plan (kernel
// boundary plus one pass over the partials).
constexpr long kCombineCost = 6;

// Longest-processing-time assignment of units to `ctas` CTAs; returns the makespan and
// (optionally) fills the per-CTA lists.
inline long lpt_schedule(int heads, int q_tiles, int C, int units, int ctas, int kv_group, AttnPlan* out) {
  std::vector<std::pair<int, int>> cost(units);  // (cost, unit)
  for (int u = 0; u < units; ++u) cost[u] = {unit_cost(decode_unit(u, heads, q_tiles, C)), u};
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
    out->unit_desc.clear();
    for (int b = 0; b < ctas; ++b) {
      for (const uint16_t u : lists[b]) {
        const Unit un = decode_unit(u, heads, q_tiles, C);
        out->unit_desc.push_back(pack_unit(u, un.head, un.head / kv_group, un.qt, un.j0, un.n));
      }
      out->cta_off.push_back((uint16_t)out->unit_desc.size());
    }
  }
  return *std::max_element(load.begin(), load.end());
}

inline long count_units(int heads, int q_tiles, int C) {
  long per_head = 0;
  for (int qt = 0; qt < q_tiles; ++qt) per_head += (qt + C) / C;
  return (long)heads * per_head;
}

AttnPlan plan_attention(int heads, int kv_group, int seq, int d, bool allow_split, int sms) {
  AttnPlan p;
  p.q_tiles = (seq + kTile - 1) / kTile;
  const int max_nt = p.q_tiles;
  // Candidate chunk sizes: the whole key range (no split), or any smaller chunk when a
  // workspace is available and the units fit the schedule table.
  long best_span = -1;
  int best_c = max_nt;
  const int min_c = (max_nt + kMaxChunks - 1) / kMaxChunks;
  for (int C = max_nt; C >= min_c; --C) {
    if (C < max_nt && (!allow_split || p.q_tiles > kMaxCombineJobs)) break;
    const long units = count_units(heads, p.q_tiles, C);
    if (units > kMaxSched) break;
    const int ctas = (int)std::min<long>(units, sms);
    const long span = lpt_schedule(heads, p.q_tiles, C, (int)units, ctas, kv_group, nullptr) + (C < max_nt ? kCombineCost : 0);
    if (best_span < 0 || span < best_span) {
      best_span = span;
      best_c = C;
    }
  }
  p.chunk = best_c;
  const long units = count_units(heads, p.q_tiles, p.chunk);
  p.units = (int)std::min<long>(units, 1L << 30);
  p.ctas = (int)std::min<long>(units, sms);
  if (units <= kMaxSched && p.ctas <= kMaxCtas) lpt_schedule(heads, p.q_tiles, p.chunk, p.units, p.ctas, kv_group, &p);
  if (p.chunk < max_nt) {
    p.stats_off = 0;
    p.o_off = round256((size_t)p.units * 2 * kTile * sizeof(float));
    p.ws_bytes = p.o_off + (size_t)p.units * kTile * (size_t)d * sizeof(float);
    int base = 0;  // per-head unit index of each query tile's chunk 0, in decode_unit order
    for (int qt = p.q_tiles - 1; qt >= 0; --qt) {
      const int nc = (qt + p.chunk) / p.chunk;
      if (nc > 1) {
        CombineJob j;
        j.qt = (uint16_t)qt;
        j.v0 = (uint16_t)base;
        j.n_e = (uint16_t)nc;
        j.pad = 0;
        p.jobs.push_back(j);
        p.max_chunks = std::max(p.max_chunks, nc);
      }
      base += nc;
    }
  }
  return p;
}

// Plans are cached per (heads, kv group, seq, d, split, SMs); the LPT search costs a few ms.
const AttnPlan& cached_plan(int heads, int kv_group, int seq, int d, bool allow_split) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, bool, int>, AttnPlan> cache;
  const int sms = sm_count();
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_tuple(heads, kv_group, seq, d, allow_split, sms);
  auto it = cache.find(key);
  if (it == cache.end()) it = cache.emplace(key, plan_attention(heads, kv_group, seq, d, allow_split, sms)).first;
  return it->second;
}

// The all-gather's other destinations, for launch_attn_bf16: peer output buffers of
// [heads_total, seq, d] (contiguous) and the head offset of this GPU's heads in them.
struct PeerDest {
  bf16* out[kMaxPeers];
  int n = 0, heads_total = 0, head_offset = 0;
};

// PP: the two-softmax-group kernel (attn_fwd_pp_bf16_kernel), else attn_fwd_bf16_kernel.
template <int D, bool PP>
int launch_attn_bf16(const void* q, const void* k, const void* v, void* out, int heads, int kv_heads, int seq,
                     float scale, void* ws, size_t ws_bytes, const AttnLayout& lay, cudaStream_t st,
                     const PeerDest* pd = nullptr) {
  CUtensorMap mq, mk, mv, mo;
  PeerOut peers;
  peers.n = pd ? pd->n : 0;
  peers.head_offset = pd ? pd->head_offset : 0;
  const int out_heads = pd ? pd->heads_total : heads;
  int rc = make_qkv_map(&mq, q, heads, seq, D, lay.q_ss, lay.q_hs, "nkl_attention(q)");
  if (!rc) rc = make_qkv_map(&mk, k, kv_heads, seq, D, lay.k_ss, lay.k_hs, "nkl_attention(k)");
  if (!rc) rc = make_qkv_map(&mv, v, kv_heads, seq, D, lay.v_ss, lay.v_hs, "nkl_attention(v)");
  if (!rc) rc = make_qkv_map(&mo, out, out_heads, seq, D, lay.o_ss, lay.o_hs, "nkl_attention(out)", 32);
  for (int p = 0; !rc && p < peers.n; ++p)
    rc = make_qkv_map(&peers.map[p], pd->out[p], out_heads, seq, D, lay.o_ss, lay.o_hs, "nkl_attention(peer out)", 32);
  if (rc) return rc;
  const AttnPlan& plan = cached_plan(heads, heads / kv_heads, seq, D, ws != nullptr);
  if (plan.ws_bytes > 0 && ws_bytes < plan.ws_bytes)
    return fail(NKL_ERR_ARG, "nkl_attention_ws: workspace %zu B < required %zu B", ws_bytes, plan.ws_bytes);
  constexpr size_t smem = PP ? sizeof(PPSmem<D>) : attn_smem_bytes<D>();
  static_assert(smem <= 232448, "attention kernel shared memory above the 227 KB per-block limit");
  constexpr auto kernel = PP ? attn_fwd_pp_bf16_kernel<D> : attn_fwd_bf16_kernel<D>;
  static std::atomic<bool> attr_set[64] = {};  // per device: the smem attribute is set (idempotent)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "nkl_attention: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  AttnArgs a;
  a.ws = plan.ws_bytes > 0 ? static_cast<unsigned char*>(ws) : nullptr;
  a.heads = heads;
  a.kv_group = heads / kv_heads;
  a.seq = seq;
  a.q_tiles = plan.q_tiles;
  a.chunk = plan.chunk;
  a.units = plan.units;
  a.scale_log2 = scale * kLog2e;
  a.ws_stats_off = plan.stats_off;
  a.ws_o_off = plan.o_off;
  a.n_ctas_listed = plan.cta_off.empty() ? 0 : plan.ctas;
  for (size_t i = 0; i < plan.cta_off.size(); ++i) a.cta_off[i] = plan.cta_off[i];
  for (size_t i = 0; i < plan.unit_desc.size(); ++i) a.unit_desc[i] = plan.unit_desc[i];
  rc = launch_pdl(kernel, dim3(plan.ctas), dim3(PP ? kPPThreads : kAttnThreads), smem, st, "nkl_attention", mq, mk, mv,
                  mo, a, peers);
  if (rc || plan.jobs.empty()) return rc;
  // split query tiles: merge the partials (programmatic dependent launch: the combine
  // grid is scheduled early and waits on the device for the attention grid)
  static CombineArgs ca;  // large kernel-parameter block, filled under the lock below
  static std::mutex ca_mu;
  std::lock_guard<std::mutex> lock(ca_mu);
  ca.ws = static_cast<const unsigned char*>(ws);
  ca.out = static_cast<bf16*>(out);
  ca.n_peer = peers.n;
  ca.head_offset = peers.head_offset;
  for (int p = 0; p < peers.n; ++p) ca.peer_out[p] = pd->out[p];
  ca.heads = heads;
  ca.seq = seq;
  ca.n_jobs = (int)plan.jobs.size();
  ca.ws_stats_off = plan.stats_off;
  ca.ws_o_off = plan.o_off;
  ca.o_ss = lay.o_ss;
  ca.o_hs = lay.o_hs;
  std::copy(plan.jobs.begin(), plan.jobs.end(), ca.job);
  // grid z: (2 row halves) x (8-column groups / groups per thread)
  auto grid = [&](int nc) { return dim3((unsigned)plan.jobs.size(), (unsigned)heads, (unsigned)(2 * (D / 8) / (8 / nc))); };
  if (plan.max_chunks <= 2)
    return launch_pdl(attn_combine_bf16_kernel<D, 2>, grid(2), dim3(64), 0, st, "nkl_attention(combine)", ca);
  if (plan.max_chunks <= 4)
    return launch_pdl(attn_combine_bf16_kernel<D, 4>, grid(4), dim3(64), 0, st, "nkl_attention(combine)", ca);
  return launch_pdl(attn_combine_bf16_kernel<D, 8>, grid(8), dim3(64), 0, st, "nkl_attention(combine)", ca);
}

// ---- two-query-tile kernel: plan and launch

struct PairPlan {
  int pairs = 0, chunk = 0, ctas = 0, units = 0;
  size_t stats_off = 0, o_off = 0, ws_bytes = 0;  // ws_bytes == 0: no split, no workspace
  std::vector<uint16_t> cta_off;                  // empty: round-robin over CTAs
  std::vector<uint4> unit;                        // per listed unit, in cta_off order
  std::vector<CombineJob> jobs;                   // split query tiles (one job per tile, all heads)
  int max_chunks = 1;
};

// Key-tile chunks [j0, j0 + n) of pair p's causal range [0, 2p + 2) for chunk size C,
// from key tile 0 up; a last chunk of a single key tile (2p + 1, which only tile B uses)
// is merged into the one before, so every chunk holds key tiles of both query tiles.
inline int pair_chunks(int p, int C, int* j0 = nullptr, int* n = nullptr) {
  const int K = 2 * p + 2;
  int nc = (K + C - 1) / C;
  if (nc > 1 && K - (nc - 1) * C == 1) --nc;
  if (j0)
    for (int c = 0; c < nc; ++c) {
      j0[c] = c * C;
      n[c] = c == nc - 1 ? K - c * C : C;
    }
  return nc;
}

// Unit cost in query-tile key steps (tile A's plus tile B's), plus a fixed charge for the
// unit's Q load, first scores and epilogue; a split plan adds one charge for the
// combine kernel that follows.
constexpr long kPairUnitFixed = 4;
constexpr long kPairCombineCost = 10;

inline long pair_unit_cost(int p, int j0, int n) {
  const int nA = std::min(n, 2 * p + 1 - j0);
  return kPairUnitFixed + nA + n;
}

PairPlan plan_pairs(int heads, int kv_group, int seq, int d, bool allow_split, int sms) {
  PairPlan plan;
  const int q_tiles = seq / kTile;
  plan.pairs = q_tiles / 2;
  const int P = plan.pairs;
  const int kmax = 2 * P;
  struct U { long cost; int head, p, c, j0, n, nc; };
  auto units_for = [&](int C, std::vector<U>* out) -> long {
    long count = 0;
    int j0[kMaxChunks + 2], n[kMaxChunks + 2];
    for (int p = P - 1; p >= 0; --p) {
      const int nc = pair_chunks(p, C, j0, n);
      count += (long)nc * heads;
      if (out)
        for (int h = 0; h < heads; ++h)
          for (int c = 0; c < nc; ++c) out->push_back(U{pair_unit_cost(p, j0[c], n[c]), h, p, c, j0[c], n[c], nc});
    }
    return count;
  };
  auto lpt = [&](std::vector<U>& us, int ctas, std::vector<std::vector<int>>* lists) -> long {
    std::stable_sort(us.begin(), us.end(), [](const U& a, const U& b) { return a.cost > b.cost; });
    std::vector<long> load(ctas, 0);
    for (int i = 0; i < (int)us.size(); ++i) {
      int best = 0;
      for (int b = 1; b < ctas; ++b)
        if (load[b] < load[best]) best = b;
      load[best] += us[i].cost;
      if (lists) (*lists)[best].push_back(i);
    }
    return *std::max_element(load.begin(), load.end());
  };
  long best_span = -1;
  int best_c = kmax;
  const int min_c = std::max(2, (kmax + kMaxChunks - 1) / kMaxChunks);
  for (int C = kmax; C >= min_c; --C) {
    if (C < kmax && (!allow_split || 2 * P > kMaxCombineJobs)) break;
    const long count = units_for(C, nullptr);
    if (count > kMaxPairSched) break;
    std::vector<U> us;
    units_for(C, &us);
    const int ctas = (int)std::min<long>(count, sms);
    const long span = lpt(us, ctas, nullptr) + (C < kmax ? kPairCombineCost : 0);
    if (best_span < 0 || span < best_span) {
      best_span = span;
      best_c = C;
    }
  }
  plan.chunk = best_c;
  const long count = units_for(plan.chunk, nullptr);
  plan.units = (int)std::min<long>(count, 1L << 30);
  plan.ctas = (int)std::min<long>(count, sms);
  if (count > kMaxPairSched || plan.ctas > kMaxCtas) return plan;  // round-robin, no split
  std::vector<U> us;
  units_for(plan.chunk, &us);
  // workspace slots of split pairs: tile A chunk c -> (base + c) * heads + head, tile B
  // chunk c -> (base + n_e + c) * heads + head, bases in decreasing pair order
  std::vector<int> base(P, -1);
  int next = 0;
  for (int p = P - 1; p >= 0; --p) {
    const int nc = pair_chunks(p, plan.chunk);
    if (nc > 1) {
      base[p] = next;
      for (int T = 0; T < 2; ++T) {
        CombineJob j;
        j.qt = (uint16_t)(2 * p + T);
        j.v0 = (uint16_t)(next + T * nc);
        j.n_e = (uint16_t)nc;
        j.pad = 0;
        plan.jobs.push_back(j);
      }
      plan.max_chunks = std::max(plan.max_chunks, nc);
      next += 2 * nc;
    }
  }
  std::vector<std::vector<int>> lists(plan.ctas);
  lpt(us, plan.ctas, &lists);
  plan.cta_off.assign(1, 0);
  for (int b = 0; b < plan.ctas; ++b) {
    for (const int i : lists[b]) {
      const U& u = us[i];
      const uint32_t slot = base[u.p] < 0 ? 0xffffffffu : (uint32_t)((base[u.p] + u.c) * heads + u.head);
      plan.unit.push_back(make_uint4((uint32_t)u.head | ((uint32_t)(u.head / kv_group) << 16),
                                     (uint32_t)u.p | ((uint32_t)u.j0 << 16), (uint32_t)u.n | ((uint32_t)u.nc << 16),
                                     slot));
    }
    plan.cta_off.push_back((uint16_t)plan.unit.size());
  }
  if (next > 0) {
    const size_t slots = (size_t)next * heads;
    plan.stats_off = 0;
    plan.o_off = round256(slots * 2 * kTile * sizeof(float));
    plan.ws_bytes = plan.o_off + slots * kTile * (size_t)d * sizeof(float);
  }
  return plan;
}

const PairPlan& cached_pair_plan(int heads, int kv_group, int seq, int d, bool allow_split) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, bool, int>, PairPlan> cache;
  const int sms = sm_count();
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_tuple(heads, kv_group, seq, d, allow_split, sms);
  auto it = cache.find(key);
  if (it == cache.end()) it = cache.emplace(key, plan_pairs(heads, kv_group, seq, d, allow_split, sms)).first;
  return it->second;
}

// The two-query-tile kernel takes bf16, head_dim 128 and whole 256-row query-tile pairs.
inline bool pair_kernel_fits(int64_t seq, int64_t d) { return d == 128 && seq % (2 * kTile) == 0; }

template <int D>
int launch_attn_pair_bf16(const void* q, const void* k, const void* v, void* out, int heads, int kv_heads, int seq,
                          float scale, void* ws, size_t ws_bytes, const AttnLayout& lay, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo;
  int rc = make_qkv_map(&mq, q, heads, seq, D, lay.q_ss, lay.q_hs, "nkl_attention(q)");
  if (!rc) rc = make_qkv_map(&mk, k, kv_heads, seq, D, lay.k_ss, lay.k_hs, "nkl_attention(k)");
  if (!rc) rc = make_qkv_map(&mv, v, kv_heads, seq, D, lay.v_ss, lay.v_hs, "nkl_attention(v)");
  if (!rc) rc = make_qkv_map(&mo, out, heads, seq, D, lay.o_ss, lay.o_hs, "nkl_attention(out)", 32);
  if (rc) return rc;
  const PairPlan& plan = cached_pair_plan(heads, heads / kv_heads, seq, D, ws != nullptr);
  if (plan.ws_bytes > 0 && ws_bytes < plan.ws_bytes)
    return fail(NKL_ERR_ARG, "nkl_attention_ws: workspace %zu B < required %zu B", ws_bytes, plan.ws_bytes);
  constexpr size_t smem = pair_smem_bytes<D>();
  static std::atomic<bool> attr_set[64] = {};  // per device: the smem attribute is set (idempotent)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_fwd_pair_bf16_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "nkl_attention: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  static PairArgs a;  // large kernel-parameter block, filled under the lock below
  static std::mutex a_mu;
  std::lock_guard<std::mutex> lock(a_mu);
  a.ws = plan.ws_bytes > 0 ? static_cast<unsigned char*>(ws) : nullptr;
  a.heads = heads;
  a.pairs = plan.pairs;
  a.kv_group = heads / kv_heads;
  a.seq = seq;
  a.scale_log2 = scale * kLog2e;
  a.ws_stats_off = plan.stats_off;
  a.ws_o_off = plan.o_off;
  a.n_ctas_listed = plan.cta_off.empty() ? 0 : plan.ctas;
  a.units = plan.units;
  std::copy(plan.cta_off.begin(), plan.cta_off.end(), a.cta_off);
  std::copy(plan.unit.begin(), plan.unit.end(), a.unit);
  rc = launch_pdl(attn_fwd_pair_bf16_kernel<D>, dim3(plan.ctas), dim3(kPairThreads), smem, st, "nkl_attention", mq,
                  mk, mv, mo, a);
  if (rc || plan.jobs.empty()) return rc;
  static CombineArgs ca;
  ca.ws = static_cast<const unsigned char*>(ws);
  ca.out = static_cast<bf16*>(out);
  ca.n_peer = 0;
  ca.head_offset = 0;
  ca.heads = heads;
  ca.seq = seq;
  ca.n_jobs = (int)plan.jobs.size();
  ca.ws_stats_off = plan.stats_off;
  ca.ws_o_off = plan.o_off;
  ca.o_ss = lay.o_ss;
  ca.o_hs = lay.o_hs;
  std::copy(plan.jobs.begin(), plan.jobs.end(), ca.job);
  auto grid = [&](int nc) { return dim3((unsigned)plan.jobs.size(), (unsigned)heads, (unsigned)(2 * (D / 8) / (8 / nc))); };
  if (plan.max_chunks <= 2)
    return launch_pdl(attn_combine_bf16_kernel<D, 2>, grid(2), dim3(64), 0, st, "nkl_attention(combine)", ca);
  if (plan.max_chunks <= 4)
    return launch_pdl(attn_combine_bf16_kernel<D, 4>, grid(4), dim3(64), 0, st, "nkl_attention(combine)", ca);
  return launch_pdl(attn_combine_bf16_kernel<D, 8>, grid(8), dim3(64), 0, st, "nkl_attention(combine)", ca);
}

// ---- the all-gather's completion barrier over NVLink
// Every rank's flag array holds world + 1 words in device memory that all ranks map (CUDA
// IPC): word j is written by rank j when it has finished writing its heads into every
// buffer, word `world` is the owner's call count. One warp: rank r stores its new count
// into word r of every peer's array (release, system scope, after a system-scope fence),
// then waits until every peer's word in its own array has reached the count (acquire,
// bounded: after kWaitTimeoutNs it records code 90 in the device flag and returns). The
// counts only grow, so a peer that is already one call ahead satisfies the wait too.
struct PeerFlags {
  unsigned int* ptr[kMaxPeers + 1];  // indexed by rank
  int world, rank;
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const __grid_constant__ PeerFlags f) {
  // Launched with programmatic dependent launch behind the attention (or merge) kernel:
  // scheduled early, it waits here until that grid has completed and its writes, the
  // stores into the other GPUs' buffers included, are performed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int t = threadIdx.x;
  unsigned int* mine = f.ptr[f.rank];
  unsigned int epoch = 0;
  if (t == 0) epoch = mine[f.world] + 1u;
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  asm volatile("fence.sc.sys;" ::: "memory");  // this GPU's output writes (earlier kernels) before the flags
  const bool peer = t < f.world && t != f.rank;
  if (peer) st_release_sys(f.ptr[t] + f.rank, epoch);
  if (peer) {
    const uint64_t t0 = globaltimer();
    while ((int)(ld_acquire_sys(mine + t) - epoch) < 0) {
      if (globaltimer() - t0 > kWaitTimeoutNs) {
        atomicCAS(&g_attn_dev_error, 0u, 90u);
        break;
      }
    }
  }
  __syncwarp();
  if (t == 0) mine[f.world] = epoch;
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

namespace {

// Shared body of the fused attention entry points: heads query heads read K and V
// head h / (heads / kv_heads); a NULL workspace (or fp32) keeps every query tile in
// one unit.
int attention_impl(const char* op, const void* q, const void* k, const void* v, void* out, void* workspace,
                   size_t workspace_bytes, int64_t heads, int64_t kv_heads, int64_t seq, int64_t head_dim,
                   float scale, int dtype, void* stream, const AttnLayout* layout = nullptr,
                   int mode = NKL_ATTN_AUTO, const PeerDest* peers = nullptr) {
  int rc = check_attn(op, heads, seq, head_dim, dtype);
  if (rc) return rc;
  if (heads == 0 || seq == 0) return NKL_OK;
  if (kv_heads < 1 || kv_heads > heads || heads % kv_heads != 0)
    return fail(NKL_ERR_SHAPE, "%s: kv_heads must divide heads (got heads=%lld kv_heads=%lld)", op, (long long)heads,
                (long long)kv_heads);
  if (!q || !k || !v || !out) return fail(NKL_ERR_ARG, "%s: NULL pointer", op);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (layout && dtype != NKL_BFLOAT16)
    return fail(NKL_ERR_DTYPE, "%s: strided q/k/v/out are supported for bf16 only", op);
  const AttnLayout lay = layout ? *layout : contiguous_layout(seq, head_dim);
  if (dtype == NKL_FLOAT32) {
    dim3 grid((unsigned)((seq + kF32Rows - 1) / kF32Rows), (unsigned)heads);
    attn_fwd_f32_kernel<<<grid, 128, 0, st>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                              static_cast<const float*>(v), static_cast<float*>(out), (int)seq,
                                              (int)head_dim, scale, (int)(heads / kv_heads));
    return check_launch(op);
  }
  if (head_dim != 64 && head_dim != 128)
    return fail(NKL_ERR_SHAPE, "%s: bf16 head_dim must be 64 or 128 (got %lld); pad on the host", op,
                (long long)head_dim);
  if (!is_aligned(q, 16) || !is_aligned(k, 16) || !is_aligned(v, 16) || !is_aligned(out, 16))
    return fail(NKL_ERR_ALIGN, "%s: bf16 tensors must be 16-byte aligned", op);
  if (workspace && !is_aligned(workspace, 256)) return fail(NKL_ERR_ALIGN, "%s: workspace not 256-byte aligned", op);
  if (mode == NKL_ATTN_TWO_TILE) {
    if (!pair_kernel_fits(seq, head_dim))
      return fail(NKL_ERR_SHAPE, "%s: the two-query-tile kernel needs head_dim 128 and seq %% 256 == 0 (got %lld, %lld)",
                  op, (long long)head_dim, (long long)seq);
    return launch_attn_pair_bf16<128>(q, k, v, out, (int)heads, (int)kv_heads, (int)seq, scale, workspace,
                                      workspace ? workspace_bytes : 0, lay, st);
  }
  if (mode == NKL_ATTN_ONE_TILE_UNSPLIT) workspace = nullptr;
  const size_t wsb = workspace ? workspace_bytes : 0;
  const int h = (int)heads, kvh = (int)kv_heads, n = (int)seq;
  if (mode == NKL_ATTN_TWO_GROUPS)
    return head_dim == 64 ? launch_attn_bf16<64, true>(q, k, v, out, h, kvh, n, scale, workspace, wsb, lay, st, peers)
                          : launch_attn_bf16<128, true>(q, k, v, out, h, kvh, n, scale, workspace, wsb, lay, st, peers);
  return head_dim == 64 ? launch_attn_bf16<64, false>(q, k, v, out, h, kvh, n, scale, workspace, wsb, lay, st, peers)
                        : launch_attn_bf16<128, false>(q, k, v, out, h, kvh, n, scale, workspace, wsb, lay, st, peers);
}

}  // namespace

extern "C" int nkl_attention(const void* q, const void* k, const void* v, void* out, int64_t heads, int64_t seq,
                             int64_t head_dim, float scale, int dtype, void* stream) {
  return attention_impl("nkl_attention", q, k, v, out, nullptr, 0, heads, heads, seq, head_dim, scale, dtype, stream);
}

extern "C" size_t nkl_attention_workspace_size(int64_t heads, int64_t seq, int64_t head_dim, int dtype) {
  if (dtype != NKL_BFLOAT16 || heads <= 0 || seq <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  if (heads > 65535 || seq > (1 << 24)) return 0;
  return cached_plan((int)heads, 1, (int)seq, (int)head_dim, true).ws_bytes;  // independent of the kv group
}

extern "C" int nkl_attention_ws(const void* q, const void* k, const void* v, void* out, void* workspace,
                                size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim, float scale,
                                int dtype, void* stream) {
  return attention_impl("nkl_attention_ws", q, k, v, out, dtype == NKL_BFLOAT16 ? workspace : nullptr,
                        workspace_bytes, heads, heads, seq, head_dim, scale, dtype, stream);
}

extern "C" int nkl_attention_gqa(const void* q, const void* k, const void* v, void* out, void* workspace,
                                 size_t workspace_bytes, int64_t heads, int64_t kv_heads, int64_t seq,
                                 int64_t head_dim, float scale, int dtype, void* stream) {
  return attention_impl("nkl_attention_gqa", q, k, v, out, dtype == NKL_BFLOAT16 ? workspace : nullptr,
                        workspace_bytes, heads, kv_heads, seq, head_dim, scale, dtype, stream);
}

extern "C" int nkl_attention_strided(const void* q, const void* k, const void* v, void* out, void* workspace,
                                     size_t workspace_bytes, int64_t heads, int64_t kv_heads, int64_t seq,
                                     int64_t head_dim, int64_t q_seq_stride, int64_t q_head_stride,
                                     int64_t kv_seq_stride, int64_t kv_head_stride, int64_t out_seq_stride,
                                     int64_t out_head_stride, float scale, int dtype, void* stream) {
  const char* op = "nkl_attention_strided";
  const int64_t st[6] = {q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride, out_seq_stride, out_head_stride};
  for (int i = 0; i < 6; ++i)
    if (st[i] < 1 || st[i] % 8 != 0 || st[i] > (int64_t(1) << 38))
      return fail(NKL_ERR_ALIGN, "%s: strides must be positive multiples of 8 elements (16 bytes), got %lld", op,
                  (long long)st[i]);
  if (q_seq_stride < head_dim || kv_seq_stride < head_dim || out_seq_stride < head_dim)
    return fail(NKL_ERR_SHAPE, "%s: a row stride is smaller than head_dim", op);
  const AttnLayout lay{q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride,
                       kv_seq_stride, kv_head_stride, out_seq_stride, out_head_stride};
  return attention_impl(op, q, k, v, out, dtype == NKL_BFLOAT16 ? workspace : nullptr, workspace_bytes, heads,
                        kv_heads, seq, head_dim, scale, dtype, stream, &lay);
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

extern "C" size_t nkl_attention_mode_workspace_size(int64_t heads, int64_t seq, int64_t head_dim, int dtype, int mode) {
  if (mode == NKL_ATTN_ONE_TILE_UNSPLIT) return 0;
  if (mode != NKL_ATTN_TWO_TILE) return nkl_attention_workspace_size(heads, seq, head_dim, dtype);
  if (dtype != NKL_BFLOAT16 || heads <= 0 || heads > 65535 || seq <= 0 || seq > (1 << 24) ||
      !pair_kernel_fits(seq, head_dim))
    return 0;
  return cached_pair_plan((int)heads, 1, (int)seq, (int)head_dim, true).ws_bytes;
}

extern "C" int nkl_attention_mode(const void* q, const void* k, const void* v, void* out, void* workspace,
                                  size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim, float scale,
                                  int dtype, int mode, void* stream) {
  if (mode != NKL_ATTN_AUTO && mode != NKL_ATTN_ONE_TILE_UNSPLIT && mode != NKL_ATTN_TWO_TILE &&
      mode != NKL_ATTN_TWO_GROUPS)
    return fail(NKL_ERR_ARG, "nkl_attention_mode: unknown mode %d", mode);
  if (mode == NKL_ATTN_TWO_TILE && dtype != NKL_BFLOAT16)
    return fail(NKL_ERR_DTYPE, "nkl_attention_mode: the two-query-tile kernel is bf16 only");
  return attention_impl("nkl_attention_mode", q, k, v, out, dtype == NKL_BFLOAT16 ? workspace : nullptr,
                        workspace_bytes, heads, heads, seq, head_dim, scale, dtype, stream, nullptr, mode);
}

extern "C" int nkl_attention_allgather(const void* q, const void* k, const void* v, void* const* outs,
                                       unsigned int* const* flags, int world, int rank, int64_t heads_total,
                                       int64_t head_offset, void* workspace, size_t workspace_bytes, int64_t heads,
                                       int64_t seq, int64_t head_dim, float scale, int dtype, void* stream) {
  const char* op = "nkl_attention_allgather";
  if (dtype != NKL_BFLOAT16) return fail(NKL_ERR_DTYPE, "%s: bf16 only", op);
  if (world < 1 || world > kMaxPeers + 1 || rank < 0 || rank >= world)
    return fail(NKL_ERR_ARG, "%s: need 1 <= world <= %d and 0 <= rank < world (got %d, %d)", op, kMaxPeers + 1, world,
                rank);
  if (heads < 1 || head_offset < 0 || heads_total < heads || head_offset > heads_total - heads || heads_total > 65535)
    return fail(NKL_ERR_SHAPE, "%s: heads [%lld, %lld) outside the %lld output heads", op, (long long)head_offset,
                (long long)(head_offset + heads), (long long)heads_total);
  if (!outs || !flags) return fail(NKL_ERR_ARG, "%s: NULL pointer array", op);
  PeerDest pd;
  pd.heads_total = (int)heads_total;
  pd.head_offset = (int)head_offset;
  PeerFlags pf;
  pf.world = world;
  pf.rank = rank;
  for (int r = 0; r < world; ++r) {
    if (!outs[r] || !flags[r]) return fail(NKL_ERR_ARG, "%s: NULL buffer of rank %d", op, r);
    if (!is_aligned(outs[r], 16) || !is_aligned(flags[r], 16))
      return fail(NKL_ERR_ALIGN, "%s: buffers must be 16-byte aligned (rank %d)", op, r);
    pf.ptr[r] = flags[r];
    if (r != rank) pd.out[pd.n++] = static_cast<bf16*>(outs[r]);
  }
  int rc = attention_impl(op, q, k, v, outs[rank], workspace, workspace_bytes, heads, heads, seq, head_dim, scale,
                          dtype, stream, nullptr, NKL_ATTN_AUTO, &pd);
  if (rc || world == 1) return rc;
  return launch_pdl(peer_barrier_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), op, pf);
}
