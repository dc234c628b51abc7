// gemm.cu - C[M,N] = A[M,K] @ B[K,N] with fp32 accumulation and one rounding.
//
// Reference: nkilab/kernels/matmul.py:46-82 (matmul_blocked: BM x BN fp32 PSUM
// accumulators per output block, K streamed in 128-row stripes, one cast on the way
// out) and :24-43 (matmul_naive: both operand tiles reloaded for every (m, n, k)).
// nkilab/ops.py:38-52 pads to tile multiples and transposes A on the host; here TMA
// reads row-major A and B directly (out-of-range boxes are zero-filled) and the
// epilogue masks partial tiles, so no host padding or transpose is needed.
//
// bf16 path (the hot path): persistent, warp-specialised tcgen05 kernel.
//   warp 0      TMA producer: A tile [128 x 64] (K-major) and B tile [64 x BN]
//               (N-major) per stage, 128-byte swizzle, STAGES-deep ring
//   warp 1      TMEM allocator + single-thread MMA issuer: 4 x tcgen05.mma
//               (M=128, N=BN, K=16) per stage into a TMEM accumulator
//   warps 2-5   epilogue: tcgen05.ld the fp32 accumulator (thread = output row),
//               round to bf16, store; two TMEM accumulators so the epilogue of tile
//               i overlaps the main loop of tile i+1
// fp32 path: exact fp32 FMA tiled kernel on CUDA cores (tcgen05 has no full-precision
// fp32 MMA; kind::tf32 would miss the reference's 1e-5 fp32 tolerance).
#include <atomic>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace nkl {
namespace {

__device__ unsigned int g_gemm_dev_error = 0;

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle row of bf16
constexpr int kGemmThreads = 192;
constexpr int kGroupM = 8;  // tile rasterisation: 8 M-tiles share each B column panel in L2

template <int BN, int STAGES>
struct GemmSmem {
  uint8_t a[STAGES][kBM * kBK * 2];  // each 16 KB, 1024-aligned (offsets are multiples of 1024)
  uint8_t b[STAGES][kBK * BN * 2];   // BN/64 boxes of [64 K rows x 128 B]
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

template <int BN, int STAGES>
constexpr size_t gemm_smem_bytes() {
  return sizeof(GemmSmem<BN, STAGES>) + 1024;  // + alignment slack
}

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_group = kGroupM * n_tiles;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(m_tiles - first_m, kGroupM);
  const int r = t - g * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

// EPI: kEpiStore writes C = A.B in bf16. kEpiSwiglu takes B as [gate | up] column blocks
// of 128 (see nkl_matmul_swiglu) and writes silu(gate) * up, each rounded to bf16 first
// exactly as the unfused matmul -> swiglu path rounds them, into C[M, N/2]. kEpiResidual
// writes C = R + A.B with A.B rounded to bf16 first and the sum rounded once more, as a
// bf16 matmul followed by a bf16 add rounds it. kEpiF32 writes the fp32 accumulator
// unrounded into a float C (the partial products of a tensor-parallel layer, summed
// across GPUs before their one rounding).
constexpr int kEpiStore = 0, kEpiSwiglu = 1, kEpiResidual = 2, kEpiF32 = 3;

template <int BN, int STAGES, int EPI = kEpiStore>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    void* __restrict__ c_out, const bf16* __restrict__ res, int M, int N, int K, int m_tiles,
                    int n_tiles) {
  extern __shared__ uint8_t smem_raw[];
  pdl_launch_dependents();
  auto& s = *reinterpret_cast<GemmSmem<BN, STAGES>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                      ~uintptr_t(1023));
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, BN, false, true);
  constexpr uint32_t kStageBytes = (kBM * kBK + kBK * BN) * 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (K + kBK - 1) / kBK;
  bf16* const c = static_cast<bf16*>(c_out);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 128);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // Launched with programmatic dependent launch: the prologue above overlaps the previous
  // kernel of the stream, and A, B and C are touched only after its writes are visible.
  // Before waiting, the producer asks L2 for the first tile's first k-blocks (a prefetch
  // only warms L2, the point of coherence: an operand the previous kernel is still
  // writing is read correctly by the loads after the wait).
  if (warp == 0 && elect_one() && (int)blockIdx.x < num_tiles) {
    int mt, nt;
    tile_coords(blockIdx.x, m_tiles, n_tiles, mt, nt);
    const int pre = k_blocks < STAGES ? k_blocks : STAGES;
    for (int kb = 0; kb < pre; ++kb) {
      tma_prefetch_2d(&map_a, kb * kBK, mt * kBM);
#pragma unroll
      for (int j = 0; j < BN / 64; ++j) tma_prefetch_2d(&map_b, nt * BN + j * 64, kb * kBK);
    }
  }
  __syncwarp();
  pdl_wait();

  if (warp == 0) {
    // ---------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int armed_phase[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) armed_phase[i] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, m_tiles, n_tiles, mt, nt);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, &s.abort, &g_gemm_dev_error, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.full[stage], kStageBytes);
          armed_phase[stage] = (int)phase;
          tma_load_2d(s.a[stage], &map_a, &s.full[stage], kb * kBK, mt * kBM);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(s.b[stage] + j * (kBK * 128), &map_b, &s.full[stage], nt * BN + j * 64, kb * kBK);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // Let copies already issued land before the CTA's shared memory is released.
        for (int i = 0; i < STAGES; ++i) {
          if (armed_phase[i] < 0) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&s.full[i], (uint32_t)armed_phase[i]) && globaltimer() - t0 < kWaitTimeoutNs) {}
        }
      }
    }
    __syncwarp();  // the warp reconverges here: the CTA barrier below must see all 32 lanes
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, &s.abort, &g_gemm_dev_error, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, &s.abort, &g_gemm_dev_error, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.a[stage]);
          const uint32_t b_base = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b_base + kk * 2048, kBK * 128, 1024);
            mma_bf16_ss(d_tmem, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&s.empty[stage]);  // frees the smem stage once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(&s.acc_full[acc]);
      }
      // Every MMA issued by this thread has completed once mma_done flips.
      mma_commit(&s.mma_done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&s.mma_done, 0) && globaltimer() - t0 < kWaitTimeoutNs) {}
    }
    __syncwarp();  // the other lanes wait for the issuing lane before the CTA barrier and dealloc
  } else {
    // ---------------- epilogue (warps 2..5 = TMEM lane quadrants 2,3,0,1)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      int mt, nt;
      tile_coords(t, m_tiles, n_tiles, mt, nt);
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&s.acc_full[acc], acc_phase, &s.abort, &g_gemm_dev_error, 4) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);  // whole warp follows lane 0 (keeps .sync.aligned ops converged)
      if (!ok) break;
      tc_fence_after();
      const int gm = mt * kBM + row;
      if constexpr (EPI == kEpiSwiglu) {
        static_assert(BN == 256, "the fused SwiGLU epilogue pairs 128 gate with 128 up columns");
        const int F = N / 2;
        bf16* orow = c + (int64_t)gm * F;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t rg[32], ru[32];
          const uint32_t base = tmem + (uint32_t)(acc * BN + cc * 32) + ((uint32_t)(q * 32) << 16);
          tmem_ld32(base, rg);
          tmem_ld32(base + 128, ru);
          tmem_wait_ld();
          const int gn = nt * 128 + cc * 32;
          if (gm < M) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              if (gn + v * 8 < F) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float g = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rg[v * 8 + e])));
                  const float u = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[v * 8 + e])));
                  f[e] = silu_f32<bf16>(g) * u;
                }
                *reinterpret_cast<uint4*>(orow + gn + v * 8) = pack16<bf16>(f);
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&s.acc_empty[acc]);
        continue;
      }
      if constexpr (EPI == kEpiF32) {
        float* frow = static_cast<float*>(c_out) + (int64_t)gm * N;
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tmem + (uint32_t)(acc * BN + cc * 32) + ((uint32_t)(q * 32) << 16), r);
          tmem_wait_ld();
          const int gn = nt * BN + cc * 32;
          if (gm < M) {
#pragma unroll
            for (int v = 0; v < 8; ++v)  // N % 8 == 0: a 4-column group is all in range or all out
              if (gn + v * 4 < N)
                *reinterpret_cast<uint4*>(frow + gn + v * 4) =
                    make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&s.acc_empty[acc]);
        continue;
      }
      bf16* crow = c + (int64_t)gm * N;
      const bf16* rrow = EPI == kEpiResidual ? res + (int64_t)gm * N : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t)(acc * BN + cc * 32) + ((uint32_t)(q * 32) << 16), r);
        tmem_wait_ld();
        const int gn = nt * BN + cc * 32;
        if (gm < M) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (gn + v * 8 < N) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[v * 8 + e]);
              if constexpr (EPI == kEpiResidual) {
                Vec16<bf16> rv;
                rv.raw = *reinterpret_cast<const uint4*>(rrow + gn + v * 8);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = __bfloat162float(__float2bfloat16_rn(f[e])) + rv.get(e);
              }
              *reinterpret_cast<uint4*>(crow + gn + v * 8) = pack16<bf16>(f);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&s.acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ fp32 exact path

constexpr int kF32Tile = 64;
constexpr int kF32K = 16;

__global__ void __launch_bounds__(256)
gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M, int N, int K) {
  __shared__ float As[kF32K][kF32Tile + 4];
  __shared__ float Bs[kF32K][kF32Tile + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kF32Tile, n0 = blockIdx.x * kF32Tile;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kF32K) {
    for (int i = threadIdx.x; i < kF32Tile * kF32K; i += 256) {
      const int r = i / kF32K, kk = i % kF32K;  // A tile: 64 rows x 16 k
      const int gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? A[(int64_t)gm * K + gk] : 0.f;
      const int kr = i / kF32Tile, cn = i % kF32Tile;  // B tile: 16 k x 64 cols
      const int gk2 = k0 + kr, gn = n0 + cn;
      Bs[kr][cn] = (gk2 < K && gn < N) ? B[(int64_t)gk2 * N + gn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kF32K; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
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
      if (gn < N) C[(int64_t)gm * N + gn] = acc[i][j];
    }
  }
}

// ------------------------------------------------------------------ naive (no reuse)

// One thread per output element, both operands streamed from global memory for every
// k: the reference's naive kernel reloads both tiles for every (m, n, k) step.
template <typename T>
__global__ void __launch_bounds__(256)
gemm_naive_kernel(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, int M, int N, int K) {
  const int n = blockIdx.x * 32 + (threadIdx.x & 31);
  const int m = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (m >= M || n >= N) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc = fmaf(to_f32(A[(int64_t)m * K + k]), to_f32(B[(int64_t)k * N + n]), acc);
  C[(int64_t)m * N + n] = from_f32<T>(acc);
}

// ------------------------------------------------------------------ host

template <int BN, int STAGES, int EPI = kEpiStore>
int launch_tc(const void* a, const void* b, void* c, int M, int N, int K, cudaStream_t st,
              const void* res = nullptr) {
  CUtensorMap ma, mb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {kBK, kBM};
    int rc = make_tensor_map_bf16(&ma, a, 2, dims, strides, box, "nkl_matmul(A)");
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {64, kBK};
    int rc = make_tensor_map_bf16(&mb, b, 2, dims, strides, box, "nkl_matmul(B)");
    if (rc) return rc;
  }
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  constexpr size_t smem = gemm_smem_bytes<BN, STAGES>();
  // The attribute is per device; setting the same value twice from racing threads is harmless.
  static std::atomic<bool> attr_set[64] = {};  // per device: the smem attribute is set (idempotent)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN, STAGES, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "nkl_matmul: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  return launch_pdl(gemm_bf16_tc_kernel<BN, STAGES, EPI>, dim3(grid), dim3(kGemmThreads), smem, st, "nkl_matmul", ma,
                    mb, c, static_cast<const bf16*>(res), M, N, K, m_tiles, n_tiles);
}

// Tile width by how many tiles the SMs get. 256-column tiles read 96 B/clk of MMA
// operands from shared memory per SM and keep the tensor pipe fed; 128-column tiles need
// 128 B/clk, at the limit, so they are used only when 256-column tiles would leave more
// than half of the SMs idle, and 64-column tiles (more CTAs, smaller operands) when
// 128-column tiles would.
template <int EPI>
int dispatch_tc(const void* a, const void* b, void* c, const void* res, int64_t M, int64_t N, int64_t K,
                cudaStream_t st) {
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  const int64_t tiles256 = m_tiles * ((N + 255) / 256);
  const int64_t tiles128 = m_tiles * ((N + 127) / 128);
  if (2 * tiles256 >= sm_count()) return launch_tc<256, 4, EPI>(a, b, c, (int)M, (int)N, (int)K, st, res);
  if (2 * tiles128 <= sm_count()) return launch_tc<64, 8, EPI>(a, b, c, (int)M, (int)N, (int)K, st, res);
  return launch_tc<128, 6, EPI>(a, b, c, (int)M, (int)N, (int)K, st, res);
}

int check_gemm(const char* op, int64_t M, int64_t N, int64_t K, int dtype) {
  if (!valid_dtype(dtype)) return fail(NKL_ERR_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (M < 0 || N < 0 || K < 0) return fail(NKL_ERR_SHAPE, "%s: negative size", op);
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(NKL_ERR_SHAPE, "%s: size exceeds 2^31-1", op);
  return NKL_OK;
}

}  // namespace

int gemm_read_and_clear_device_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_dev_error, sizeof(v)) != cudaSuccess) return -1;
  if (v && cudaMemcpyToSymbol(g_gemm_dev_error, &zero, sizeof(zero)) != cudaSuccess) return -1;
  return (int)v;
}

}  // namespace nkl

using namespace nkl;

extern "C" int nkl_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int dtype,
                          void* stream) {
  int rc = check_gemm("nkl_matmul", M, N, K, dtype);
  if (rc) return rc;
  if (M == 0 || N == 0) return NKL_OK;
  if (!a || !b || !c) return fail(NKL_ERR_ARG, "nkl_matmul: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(c, 0, (size_t)M * (size_t)N * dtype_size(dtype), st);
    return e == cudaSuccess ? NKL_OK : fail(NKL_ERR_CUDA, "nkl_matmul: %s", cudaGetErrorString(e));
  }
  if (dtype == NKL_FLOAT32) {
    dim3 grid((unsigned)((N + kF32Tile - 1) / kF32Tile), (unsigned)((M + kF32Tile - 1) / kF32Tile));
    gemm_f32_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(a), static_cast<const float*>(b),
                                          static_cast<float*>(c), (int)M, (int)N, (int)K);
    return check_launch("nkl_matmul");
  }
  if (K % 8 != 0 || N % 8 != 0)
    return fail(NKL_ERR_SHAPE, "nkl_matmul: bf16 needs K and N multiples of 8 (got K=%lld N=%lld)", (long long)K,
                (long long)N);
  if (!is_aligned(a, 16) || !is_aligned(b, 16) || !is_aligned(c, 16))
    return fail(NKL_ERR_ALIGN, "nkl_matmul: bf16 operands must be 16-byte aligned");
  return dispatch_tc<kEpiStore>(a, b, c, nullptr, M, N, K, st);
}

extern "C" int nkl_matmul_residual(const void* a, const void* b, const void* residual, void* out, int64_t M,
                                   int64_t N, int64_t K, int dtype, void* stream) {
  int rc = check_gemm("nkl_matmul_residual", M, N, K, dtype);
  if (rc) return rc;
  if (dtype != NKL_BFLOAT16) return fail(NKL_ERR_DTYPE, "nkl_matmul_residual: bf16 only");
  if (M == 0 || N == 0) return NKL_OK;
  if (!a || !b || !residual || !out) return fail(NKL_ERR_ARG, "nkl_matmul_residual: NULL pointer");
  if (K == 0 || K % 8 != 0 || N % 8 != 0)
    return fail(NKL_ERR_SHAPE, "nkl_matmul_residual: needs K > 0 and K, N multiples of 8 (got K=%lld N=%lld)",
                (long long)K, (long long)N);
  if (!is_aligned(a, 16) || !is_aligned(b, 16) || !is_aligned(residual, 16) || !is_aligned(out, 16))
    return fail(NKL_ERR_ALIGN, "nkl_matmul_residual: operands must be 16-byte aligned");
  return dispatch_tc<kEpiResidual>(a, b, out, residual, M, N, K, static_cast<cudaStream_t>(stream));
}

extern "C" int nkl_matmul_f32out(const void* a, const void* b, float* c, int64_t M, int64_t N, int64_t K,
                                 int dtype, void* stream) {
  int rc = check_gemm("nkl_matmul_f32out", M, N, K, dtype);
  if (rc) return rc;
  if (dtype != NKL_BFLOAT16) return fail(NKL_ERR_DTYPE, "nkl_matmul_f32out: bf16 inputs only");
  if (M == 0 || N == 0) return NKL_OK;
  if (!a || !b || !c) return fail(NKL_ERR_ARG, "nkl_matmul_f32out: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(c, 0, (size_t)M * (size_t)N * sizeof(float), st);
    return e == cudaSuccess ? NKL_OK : fail(NKL_ERR_CUDA, "nkl_matmul_f32out: %s", cudaGetErrorString(e));
  }
  if (K % 8 != 0 || N % 8 != 0)
    return fail(NKL_ERR_SHAPE, "nkl_matmul_f32out: needs K and N multiples of 8 (got K=%lld N=%lld)", (long long)K,
                (long long)N);
  if (!is_aligned(a, 16) || !is_aligned(b, 16) || !is_aligned(c, 16))
    return fail(NKL_ERR_ALIGN, "nkl_matmul_f32out: operands must be 16-byte aligned");
  return dispatch_tc<kEpiF32>(a, b, c, nullptr, M, N, K, st);
}

extern "C" int nkl_matmul_swiglu(const void* a, const void* b_gate_up, void* out, int64_t M, int64_t F, int64_t K,
                                 int dtype, void* stream) {
  int rc = check_gemm("nkl_matmul_swiglu", M, 2 * F, K, dtype);
  if (rc) return rc;
  if (dtype != NKL_BFLOAT16) return fail(NKL_ERR_DTYPE, "nkl_matmul_swiglu: bf16 only");
  if (M == 0 || F == 0) return NKL_OK;
  if (!a || !b_gate_up || !out) return fail(NKL_ERR_ARG, "nkl_matmul_swiglu: NULL pointer");
  if (K == 0 || K % 8 != 0 || F % 128 != 0)
    return fail(NKL_ERR_SHAPE, "nkl_matmul_swiglu: needs K > 0, K %% 8 == 0 and F %% 128 == 0 (got K=%lld F=%lld)",
                (long long)K, (long long)F);
  if (!is_aligned(a, 16) || !is_aligned(b_gate_up, 16) || !is_aligned(out, 16))
    return fail(NKL_ERR_ALIGN, "nkl_matmul_swiglu: operands must be 16-byte aligned");
  return launch_tc<256, 4, kEpiSwiglu>(a, b_gate_up, out, (int)M, (int)(2 * F), (int)K,
                                        static_cast<cudaStream_t>(stream));
}

extern "C" int nkl_matmul_naive(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int dtype,
                                void* stream) {
  int rc = check_gemm("nkl_matmul_naive", M, N, K, dtype);
  if (rc) return rc;
  if (M == 0 || N == 0) return NKL_OK;
  if (!a || !b || !c) return fail(NKL_ERR_ARG, "nkl_matmul_naive: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)((M + 7) / 8));
  if (dtype == NKL_FLOAT32)
    gemm_naive_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(a), static_cast<const float*>(b),
                                                   static_cast<float*>(c), (int)M, (int)N, (int)K);
  else
    gemm_naive_kernel<bf16><<<grid, 256, 0, st>>>(static_cast<const bf16*>(a), static_cast<const bf16*>(b),
                                                  static_cast<bf16*>(c), (int)M, (int)N, (int)K);
  return check_launch("nkl_matmul_naive");
}
