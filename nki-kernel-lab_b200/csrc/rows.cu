// rows.cu - memory-bound row kernels: RMSNorm, softmax (fused and unfused), SwiGLU.
//
// Reference algorithms (Nags-gk/nki-kernel-lab):
//   rmsnorm_fused    nkilab/kernels/norm.py:92-118
//   softmax_fused    nkilab/kernels/norm.py:65-89
//   softmax_unfused  nkilab/kernels/norm.py:22-62
//   swiglu_fused     nkilab/kernels/norm.py:121-136
// The reference tiles 128 rows onto SBUF partitions; on B200 a row maps to one warp
// (rows up to 512 16-byte vectors) held entirely in registers, so every byte of the
// input is read from HBM once and every output byte written once, with 16-byte
// coalesced accesses. A warp issues every load of its row before the first reduction,
// and the launch shapes keep enough warps resident that (at the benchmark shape) every
// row is in flight at once; kernels are launched with programmatic dependent launch
// (launch_pdl). Rows that are too long
// or not 16-byte aligned fall back to a block-per-row kernel that streams the row more
// than once (still exact).
//
// Rounding points follow the reference: statistics in fp32, one rounding to the
// output dtype at the end (rmsnorm rounds x*rstd to fp32 before the weight multiply,
// norm.py:114-116; fused softmax multiplies by a reciprocal, norm.py:84-87; unfused
// softmax divides, norm.py:142).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace nkl {
namespace {

// Launch shapes, chosen by measurement on B200 at [4096, 2048] bf16 (4096 rows, one
// warp each). A warp holds its row in registers from the first load to the last store,
// so the number of rows in flight is the number of resident warps: RMSNorm is capped at
// 72 registers (7 four-warp blocks, 28 warps per SM), which puts all 4096 rows on the
// GPU in one wave; softmax keeps its 64 exponentials in registers (about 80 registers,
// 24 warps per SM) and runs two-warp blocks, which fill the last partial wave at the
// finest grain.
constexpr int kRmsWarpsPerBlock = 4;
// Resident four-warp blocks per SM that the register cap allows: 7 (72 registers) for rows
// of up to 8 vectors per lane, 4 (128 registers) for the 16-vector rows.
constexpr int rms_min_blocks(int nv) { return nv <= 8 ? 7 : 4; }
// The fused residual add holds two rows (x and the residual) while its loads are in flight;
// two-warp blocks without a register cap measured fastest for it.
constexpr int kAddRmsWarpsPerBlock = 2;
constexpr int kSoftmaxWarpsPerBlock = 2;
constexpr int kMaxVecPerLane = 16;  // 512 vectors per row: 4096 bf16 / 2048 fp32 columns

// Element e of a 16-byte vector as fp32, with `z` (zero at run time) folded into the bit
// pattern. The fold costs nothing (the bf16 unpack is an integer op either way) but makes
// the value depend on whatever produced z: a pass that unpacks a row a second time after
// a reduction ties its unpacks to the reduction's result, so the compiler keeps only the
// packed row (4 registers per vector) live across the reduction instead of hoisting the
// unpacked fp32 values (8 per vector) above it.
template <typename T> __device__ __forceinline__ float vec_get_tied(const Vec16<T>& v, int e, uint32_t z) {
  if constexpr (sizeof(T) == 4) {
    return reinterpret_cast<const float*>(&v.raw)[e];
  } else {
    const uint32_t w = reinterpret_cast<const uint32_t*>(&v.raw)[e >> 1];
    return __uint_as_float((e & 1) ? ((w & 0xffff0000u) | z) : (w * 65536u + z));
  }
}

// ------------------------------------------------------------------ RMSNorm

// FULL: the row fills every lane's NV vectors (cols == 32 * NV * V), so no column guards.
template <typename T, int NV, bool FULL>
__global__ void __launch_bounds__(kRmsWarpsPerBlock * 32, rms_min_blocks(NV))
rmsnorm_warp_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, int64_t rows, int cols,
                    float inv_cols, float eps) {
  constexpr int V = Vec16<T>::N;
  pdl_launch_dependents();
  // The weight row, staged once per block: every warp reads it right after its reduction,
  // from shared memory instead of an L2 round trip on its critical path.
  __shared__ uint4 wsm[NV * 32];
  const int64_t row = (int64_t)blockIdx.x * kRmsWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < rows && lane == 0) l2_prefetch(x + row * cols, (uint32_t)(cols * sizeof(T)));
  pdl_wait();
  const int nvec = cols / V;
  const T* xr = x + row * cols;
  Vec16<T> xv[NV];
  if (row < rows) {  // the row's loads go out first; the weight loads overlap their latency
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = i * 32 + lane;
      xv[i].raw = (FULL || j < nvec) ? ld_stream(xr + j * V) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  constexpr int kPerThread = (NV * 32 + kRmsWarpsPerBlock * 32 - 1) / (kRmsWarpsPerBlock * 32);
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int j = k * kRmsWarpsPerBlock * 32 + (int)threadIdx.x;
    if (j < nvec) wsm[j] = *reinterpret_cast<const uint4*>(w + j * V);
  }
  __syncthreads();
  if (row >= rows) return;
  // Four partial sums break the dependent chain of NV * V fused multiply-adds.
  float ssq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int e = 0; e < V; ++e) { const float f = xv[i].get(e); ssq[e & 3] = fmaf(f, f, ssq[e & 3]); }
  }
  const float rstd = rsqrtf(warp_sum((ssq[0] + ssq[1]) + (ssq[2] + ssq[3])) * inv_cols + eps);
  const uint32_t z = __float_as_uint(rstd) >> 31;  // rstd > 0: zero, and tied to the reduction
  T* yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * 32 + lane;
    if (FULL || j < nvec) {
      Vec16<T> wv;
      wv.raw = wsm[j + z];
      float o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = (vec_get_tied(xv[i], e, z) * rstd) * wv.get(e);  // fp32 x * rstd, then * weight
      st_stream(yr + j * V, pack16<T>(o));
    }
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < nw) ? red[l] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < nw) ? red[l] : -INFINITY;
  return warp_max(t);
}

template <typename T>
__global__ void __launch_bounds__(256)
rmsnorm_block_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                     int64_t rows, int64_t cols, float inv_cols, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  float ssq = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) { const float f = to_f32(xr[c]); ssq += f * f; }
  ssq = block_sum(ssq, red);
  const float rstd = rsqrtf(ssq * inv_cols + eps);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float xn = to_f32(xr[c]) * rstd;
    yr[c] = from_f32<T>(xn * to_f32(w[c]));
  }
}

// ------------------------------------------------------------------ fused softmax

// exp(x - max) for the fused softmax. fp32 outputs use the accurate library expf (the
// reference's fp32 tolerance is 1e-5). bf16 outputs use exp(t) = 2^(t * log2(e)) with the
// argument formed by one fused multiply-add, x * log2(e) + (-max * log2(e)), and the
// hardware base-2 exponential (ex2.approx.ftz: relative error about 2^-22, far below one
// bf16 ulp; results under 2^-126 flush to zero, where the rounded bf16 output is zero or
// subnormal anyway).
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx_ftz(float t) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}
template <typename T> __device__ __forceinline__ float softmax_exp(float x, float mx, float neg_mx_log2e) {
  if constexpr (sizeof(T) == 4) return expf(x - mx);
  else return ex2_approx_ftz(fmaf(x, kLog2e, neg_mx_log2e));
}

template <typename T, int NV, bool FULL>
__global__ void __launch_bounds__(kSoftmaxWarpsPerBlock * 32)
softmax_warp_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int cols) {
  constexpr int V = Vec16<T>::N;
  pdl_launch_dependents();
  const int64_t row = (int64_t)blockIdx.x * kSoftmaxWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < rows && lane == 0) l2_prefetch(x + row * cols, (uint32_t)(cols * sizeof(T)));
  pdl_wait();
  if (row >= rows) return;
  const int nvec = cols / V;
  const T* xr = x + row * cols;
  Vec16<T> xv[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * 32 + lane;
    if (FULL || j < nvec) xv[i].raw = ld_stream(xr + j * V);
  }
  // Four partial maxima / sums break the dependent chains of NV * V operations.
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (FULL || i * 32 + lane < nvec) {
#pragma unroll
      for (int e = 0; e < V; ++e) m[e & 3] = fmaxf(m[e & 3], xv[i].get(e));
    }
  }
  const float mx = warp_max(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])));
  const float neg_mx_log2e = -mx * kLog2e;
  // Rows of up to 64 values per lane keep exp(x - max) in registers, so each element
  // costs one exp; longer rows recompute it in the output pass to bound registers.
  constexpr bool kKeep = NV * V <= 64;
  float ex[kKeep ? NV * V : 1];
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (FULL || i * 32 + lane < nvec) {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const float t = softmax_exp<T>(xv[i].get(e), mx, neg_mx_log2e);
        if constexpr (kKeep) ex[i * V + e] = t;
        s[e & 3] += t;
      }
    }
  }
  const float rinv = 1.0f / warp_sum((s[0] + s[1]) + (s[2] + s[3]));
  T* yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * 32 + lane;
    if (FULL || j < nvec) {
      float o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) {
        if constexpr (kKeep) o[e] = ex[i * V + e] * rinv;
        else o[e] = softmax_exp<T>(xv[i].get(e), mx, neg_mx_log2e) * rinv;
      }
      st_stream(yr + j * V, pack16<T>(o));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
softmax_block_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int64_t cols) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, to_f32(xr[c]));
  const float neg_max = -block_max(m, red);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s += row_exp<T>(to_f32(xr[c]) + neg_max);
  const float rinv = 1.0f / block_sum(s, red);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    yr[c] = from_f32<T>(row_exp<T>(to_f32(xr[c]) + neg_max) * rinv);
}

// ------------------------------------------------------------------ unfused softmax
// Three launches, each a full HBM round trip, as in norm.py:22-62:
//   pass 1  m[r] = max_c x[r,c]                        -> workspace
//   pass 2  e[r,c] = exp(x[r,c] - m[r]) (fp32), s[r] = sum_c e[r,c]  -> workspace
//   pass 3  y[r,c] = e[r,c] / s[r]

template <typename T>
__global__ void __launch_bounds__(256)
softmax_pass_max(const T* __restrict__ x, float* __restrict__ m_out, int64_t cols) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, to_f32(xr[c]));
  m = block_max(m, red);
  if (threadIdx.x == 0) m_out[row] = m;
}

template <typename T>
__global__ void __launch_bounds__(256)
softmax_pass_exp(const T* __restrict__ x, const float* __restrict__ m_in, float* __restrict__ e_out,
                 float* __restrict__ s_out, int64_t cols) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  float* er = e_out + row * cols;
  const float m = m_in[row];
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float sh = to_f32(xr[c]) - m;
    const float e = row_exp<float>(sh);
    er[c] = e;
    s += e;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) s_out[row] = s;
}

template <typename T>
__global__ void __launch_bounds__(256)
softmax_pass_div(const float* __restrict__ e_in, const float* __restrict__ s_in, T* __restrict__ y,
                 int64_t cols) {
  const int64_t row = blockIdx.x;
  const float* er = e_in + row * cols;
  T* yr = y + row * cols;
  const float s = s_in[row];
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = from_f32<T>(er[c] / s);
}

// ------------------------------------------------------------------ SwiGLU

constexpr int kSwigluThreads = 256;
constexpr int kSwigluUnroll = 4;

// Every thread handles kSwigluUnroll 16-byte vectors of gate and up, all loads
// issued before any math so 8 x 16 B are in flight per thread.
template <typename T>
__global__ void __launch_bounds__(kSwigluThreads)
swiglu_vec_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y, int64_t nvec) {
  constexpr int V = Vec16<T>::N;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {  // this block's contiguous span of gate and up
    const int64_t v0 = (int64_t)blockIdx.x * kSwigluThreads * kSwigluUnroll;
    const int64_t nv = nvec - v0 < (int64_t)kSwigluThreads * kSwigluUnroll ? nvec - v0 : (int64_t)kSwigluThreads * kSwigluUnroll;
    l2_prefetch(g + v0 * V, (uint32_t)(nv * 16));
    l2_prefetch(u + v0 * V, (uint32_t)(nv * 16));
  }
  pdl_wait();
  const int64_t base = (int64_t)blockIdx.x * kSwigluThreads * kSwigluUnroll + threadIdx.x;
  Vec16<T> gv[kSwigluUnroll], uv[kSwigluUnroll];
#pragma unroll
  for (int i = 0; i < kSwigluUnroll; ++i) {
    const int64_t j = base + (int64_t)i * kSwigluThreads;
    if (j < nvec) {
      gv[i].raw = ld_stream(g + j * V);
      uv[i].raw = ld_stream(u + j * V);
    }
  }
#pragma unroll
  for (int i = 0; i < kSwigluUnroll; ++i) {
    const int64_t j = base + (int64_t)i * kSwigluThreads;
    if (j < nvec) {
      float o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = silu_f32<T>(gv[i].get(e)) * uv[i].get(e);
      st_stream(y + j * V, pack16<T>(o));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
swiglu_scalar_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f32<T>(silu_f32<T>(to_f32(g[i])) * to_f32(u[i]));
}

// ------------------------------------------------------------------ residual add + RMSNorm

// s = x + r rounded to the dtype (the reference adds the residual on the host in x.dtype,
// nkilab/model.py:86,89), written out, then y = rmsnorm(s) with the same rounding points
// as rmsnorm_warp_kernel: one pass over x and r instead of an add kernel and a norm kernel.
template <typename T, int NV>
__global__ void __launch_bounds__(kAddRmsWarpsPerBlock * 32)
add_rmsnorm_warp_kernel(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ w,
                        T* __restrict__ s_out, T* __restrict__ y, int64_t rows, int cols, float inv_cols, float eps) {
  constexpr int V = Vec16<T>::N;
  pdl_launch_dependents();
  const int64_t row = (int64_t)blockIdx.x * kAddRmsWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < rows && lane == 0 && (cols * sizeof(T)) % 16 == 0) {
    l2_prefetch(x + row * cols, (uint32_t)(cols * sizeof(T)));
    l2_prefetch(res + row * cols, (uint32_t)(cols * sizeof(T)));
  }
  pdl_wait();
  if (row >= rows) return;
  const int nvec = cols / V;
  Vec16<T> sv[NV];
  {
    Vec16<T> rv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = i * 32 + lane;
      if (j < nvec) {
        sv[i].raw = ld_stream(x + row * cols + (int64_t)j * V);
        rv[i].raw = ld_stream(res + row * cols + (int64_t)j * V);
      } else {
        sv[i].raw = rv[i].raw = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float f[V];
#pragma unroll
      for (int e = 0; e < V; ++e) f[e] = sv[i].get(e) + rv[i].get(e);
      sv[i].raw = pack16<T>(f);  // the sum, rounded to the dtype
      const int j = i * 32 + lane;
      if (j < nvec) st_stream(s_out + row * cols + (int64_t)j * V, sv[i].raw);
    }
  }
  // The same partial sums in the same order as rmsnorm_warp_kernel, so the result equals
  // rmsnorm(x + residual) bit for bit.
  float ssq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int e = 0; e < V; ++e) { const float f = sv[i].get(e); ssq[e & 3] = fmaf(f, f, ssq[e & 3]); }
  }
  const float rstd = rsqrtf(warp_sum((ssq[0] + ssq[1]) + (ssq[2] + ssq[3])) * inv_cols + eps);
  T* yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * 32 + lane;
    if (j < nvec) {
      Vec16<T> wv;
      wv.raw = __ldg(reinterpret_cast<const uint4*>(w + (int64_t)j * V));
      float o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = (sv[i].get(e) * rstd) * wv.get(e);  // fp32 s * rstd, then * weight
      st_stream(yr + (int64_t)j * V, pack16<T>(o));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
add_scalar_kernel(const T* __restrict__ x, const T* __restrict__ r, T* __restrict__ s, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s[i] = from_f32<T>(to_f32(x[i]) + to_f32(r[i]));
}

// ------------------------------------------------------------------ rotary embedding

// Rotary position embedding, rotate-half convention: for i < d/2, with
// theta_i = base^(-2i/d) (computed in fp32 as 1 / powf(base, 2i/d)) and angle = pos * theta_i,
//   out[i]       = x[i] * cos(angle) - x[i + d/2] * sin(angle)
//   out[i + d/2] = x[i + d/2] * cos(angle) + x[i] * sin(angle)
// in fp32 with one rounding to the output dtype; pos = row index within the sequence +
// pos_offset. A thread handles one 16-byte vector of each half. No reference counterpart
// (rotary embeddings are the reference's listed next step, README.md:89).
template <typename T>
__global__ void __launch_bounds__(256)
rope_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int seq, int d, float base, int pos_offset) {
  constexpr int V = Vec16<T>::N;
  pdl_enter();
  const int half_vecs = d / 2 / V;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * half_vecs) return;
  const int64_t row = i / half_vecs;
  const int c0 = (int)(i - row * half_vecs) * V;  // first column of this thread's vector in the first half
  const float pos = (float)((int)(row % seq) + pos_offset);
  const T* xr = x + row * d;
  T* yr = y + row * d;
  Vec16<T> a, b;
  a.raw = ld_stream(xr + c0);
  b.raw = ld_stream(xr + c0 + d / 2);
  float oa[V], ob[V];
#pragma unroll
  for (int e = 0; e < V; ++e) {
    const float inv_freq = 1.0f / powf(base, (float)(2 * (c0 + e)) / (float)d);
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    const float xa = a.get(e), xb = b.get(e);
    oa[e] = xa * cs - xb * sn;
    ob[e] = xb * cs + xa * sn;
  }
  st_stream(yr + c0, pack16<T>(oa));
  st_stream(yr + c0 + d / 2, pack16<T>(ob));
}

// ------------------------------------------------------------------ dispatch

template <typename T>
bool row_vectorizable(int64_t cols, const void* a, const void* b, const void* c) {
  constexpr int V = 16 / sizeof(T);
  return cols % V == 0 && cols / V <= 32 * kMaxVecPerLane && is_aligned(a, 16) && is_aligned(b, 16) &&
         (c == nullptr || is_aligned(c, 16));
}

// Vectors per lane rounded up to a power of two (1..16).
inline int nv_bucket(int64_t nvec) {
  const int64_t per_lane = (nvec + 31) / 32;
  int nv = 1;
  while (nv < per_lane) nv <<= 1;
  return nv;
}

template <typename T>
int rmsnorm_launch(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                   cudaStream_t st) {
  const float inv_cols = (float)(1.0 / (double)cols);
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  T* yp = static_cast<T*>(y);
  if (row_vectorizable<T>(cols, x, y, w)) {
    const int64_t nvec = cols / (16 / (int64_t)sizeof(T));
    const int nv = nv_bucket(nvec);
    const bool full = nvec == 32 * (int64_t)nv;
    const int c = (int)cols;
    const dim3 grid((unsigned)((rows + kRmsWarpsPerBlock - 1) / kRmsWarpsPerBlock)), blk(kRmsWarpsPerBlock * 32);
    auto go = [&](auto kernel) { return launch_pdl(kernel, grid, blk, 0, st, "nkl_rmsnorm", xp, wp, yp, rows, c, inv_cols, eps); };
    switch (nv) {
      case 1: return full ? go(rmsnorm_warp_kernel<T, 1, true>) : go(rmsnorm_warp_kernel<T, 1, false>);
      case 2: return full ? go(rmsnorm_warp_kernel<T, 2, true>) : go(rmsnorm_warp_kernel<T, 2, false>);
      case 4: return full ? go(rmsnorm_warp_kernel<T, 4, true>) : go(rmsnorm_warp_kernel<T, 4, false>);
      case 8: return full ? go(rmsnorm_warp_kernel<T, 8, true>) : go(rmsnorm_warp_kernel<T, 8, false>);
      default: return full ? go(rmsnorm_warp_kernel<T, 16, true>) : go(rmsnorm_warp_kernel<T, 16, false>);
    }
  } else {
    rmsnorm_block_kernel<T><<<(unsigned)rows, 256, 0, st>>>(xp, wp, yp, rows, cols, inv_cols, eps);
  }
  return check_launch("nkl_rmsnorm");
}

template <typename T>
int softmax_launch(const void* x, void* y, int64_t rows, int64_t cols, cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (row_vectorizable<T>(cols, x, y, nullptr)) {
    const int64_t nvec = cols / (16 / (int64_t)sizeof(T));
    const int nv = nv_bucket(nvec);
    const bool full = nvec == 32 * (int64_t)nv;
    const int c = (int)cols;
    const dim3 grid((unsigned)((rows + kSoftmaxWarpsPerBlock - 1) / kSoftmaxWarpsPerBlock)), blk(kSoftmaxWarpsPerBlock * 32);
    auto go = [&](auto kernel) { return launch_pdl(kernel, grid, blk, 0, st, "nkl_softmax", xp, yp, rows, c); };
    switch (nv) {
      case 1: return full ? go(softmax_warp_kernel<T, 1, true>) : go(softmax_warp_kernel<T, 1, false>);
      case 2: return full ? go(softmax_warp_kernel<T, 2, true>) : go(softmax_warp_kernel<T, 2, false>);
      case 4: return full ? go(softmax_warp_kernel<T, 4, true>) : go(softmax_warp_kernel<T, 4, false>);
      case 8: return full ? go(softmax_warp_kernel<T, 8, true>) : go(softmax_warp_kernel<T, 8, false>);
      default: return full ? go(softmax_warp_kernel<T, 16, true>) : go(softmax_warp_kernel<T, 16, false>);
    }
  } else {
    softmax_block_kernel<T><<<(unsigned)rows, 256, 0, st>>>(xp, yp, rows, cols);
  }
  return check_launch("nkl_softmax");
}

// Workspace layout of the unfused softmax: m [rows] | s [rows] | e [rows, cols], each
// fp32 and each region starting on a 256-byte boundary.
inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

template <typename T>
int softmax_unfused_launch(const void* x, void* y, void* ws, int64_t rows, int64_t cols, cudaStream_t st) {
  float* m = static_cast<float*>(ws);
  float* s = reinterpret_cast<float*>(static_cast<char*>(ws) + round256(rows * sizeof(float)));
  float* e = reinterpret_cast<float*>(static_cast<char*>(ws) + 2 * round256(rows * sizeof(float)));
  const T* xp = static_cast<const T*>(x);
  softmax_pass_max<T><<<(unsigned)rows, 256, 0, st>>>(xp, m, cols);
  softmax_pass_exp<T><<<(unsigned)rows, 256, 0, st>>>(xp, m, e, s, cols);
  softmax_pass_div<T><<<(unsigned)rows, 256, 0, st>>>(e, s, static_cast<T*>(y), cols);
  return check_launch("nkl_softmax_unfused");
}

template <typename T>
int swiglu_launch(const void* g, const void* u, void* y, int64_t n, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const T* gp = static_cast<const T*>(g);
  const T* up = static_cast<const T*>(u);
  T* yp = static_cast<T*>(y);
  if (n % V == 0 && is_aligned(g, 16) && is_aligned(u, 16) && is_aligned(y, 16)) {
    const int64_t nvec = n / V;
    const int64_t per_block = (int64_t)kSwigluThreads * kSwigluUnroll;
    const unsigned grid = (unsigned)((nvec + per_block - 1) / per_block);
    return launch_pdl(swiglu_vec_kernel<T>, dim3(grid), dim3(kSwigluThreads), 0, st, "nkl_swiglu", gp, up, yp, nvec);
  } else {
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    swiglu_scalar_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(gp, up, yp, n);
  }
  return check_launch("nkl_swiglu");
}

int check_rows(const char* op, int64_t rows, int64_t cols, int dtype) {
  if (!valid_dtype(dtype)) return fail(NKL_ERR_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (rows < 0 || cols < 1) return fail(NKL_ERR_SHAPE, "%s: bad shape [%lld, %lld]", op, (long long)rows, (long long)cols);
  if (rows > 0x7fffffffLL) return fail(NKL_ERR_SHAPE, "%s: rows %lld exceed 2^31-1", op, (long long)rows);
  return NKL_OK;
}

}  // namespace
}  // namespace nkl

using namespace nkl;

extern "C" int nkl_rmsnorm(const void* x, const void* weight, void* out, int64_t rows, int64_t cols,
                           float eps, int dtype, void* stream) {
  int rc = check_rows("nkl_rmsnorm", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!x || !weight || !out) return fail(NKL_ERR_ARG, "nkl_rmsnorm: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NKL_FLOAT32 ? rmsnorm_launch<float>(x, weight, out, rows, cols, eps, st)
                              : rmsnorm_launch<bf16>(x, weight, out, rows, cols, eps, st);
}

extern "C" int nkl_add_rmsnorm(const void* x, const void* residual, const void* weight, void* sum_out, void* out,
                               int64_t rows, int64_t cols, float eps, int dtype, void* stream) {
  int rc = check_rows("nkl_add_rmsnorm", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!x || !residual || !weight || !sum_out || !out) return fail(NKL_ERR_ARG, "nkl_add_rmsnorm: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float inv_cols = (float)(1.0 / (double)cols);
  auto fused = [&](auto tag) -> int {
    using T = decltype(tag);
    const int nv = nv_bucket(cols / (16 / (int64_t)sizeof(T)));
    const dim3 grid((unsigned)((rows + kAddRmsWarpsPerBlock - 1) / kAddRmsWarpsPerBlock)), blk(kAddRmsWarpsPerBlock * 32);
    const T* xp = static_cast<const T*>(x);
    const T* rp = static_cast<const T*>(residual);
    const T* wp = static_cast<const T*>(weight);
    T* sp = static_cast<T*>(sum_out);
    T* yp = static_cast<T*>(out);
    const int c = (int)cols;
    switch (nv) {
      case 1: return launch_pdl(add_rmsnorm_warp_kernel<T, 1>, grid, blk, 0, st, "nkl_add_rmsnorm", xp, rp, wp, sp, yp, rows, c, inv_cols, eps);
      case 2: return launch_pdl(add_rmsnorm_warp_kernel<T, 2>, grid, blk, 0, st, "nkl_add_rmsnorm", xp, rp, wp, sp, yp, rows, c, inv_cols, eps);
      case 4: return launch_pdl(add_rmsnorm_warp_kernel<T, 4>, grid, blk, 0, st, "nkl_add_rmsnorm", xp, rp, wp, sp, yp, rows, c, inv_cols, eps);
      case 8: return launch_pdl(add_rmsnorm_warp_kernel<T, 8>, grid, blk, 0, st, "nkl_add_rmsnorm", xp, rp, wp, sp, yp, rows, c, inv_cols, eps);
      default: return launch_pdl(add_rmsnorm_warp_kernel<T, 16>, grid, blk, 0, st, "nkl_add_rmsnorm", xp, rp, wp, sp, yp, rows, c, inv_cols, eps);
    }
  };
  const bool vec = dtype == NKL_FLOAT32 ? row_vectorizable<float>(cols, x, out, weight) &&
                                              is_aligned(residual, 16) && is_aligned(sum_out, 16)
                                        : row_vectorizable<bf16>(cols, x, out, weight) &&
                                              is_aligned(residual, 16) && is_aligned(sum_out, 16);
  if (vec) return dtype == NKL_FLOAT32 ? fused(float{}) : fused(bf16{});
  // other shapes: the add, then the norm of the rounded sum (same results, two passes)
  const int64_t n = rows * cols;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148LL * 16);
  if (dtype == NKL_FLOAT32)
    add_scalar_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), static_cast<const float*>(residual),
                                                     static_cast<float*>(sum_out), n);
  else
    add_scalar_kernel<bf16><<<blocks, 256, 0, st>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(residual),
                                                    static_cast<bf16*>(sum_out), n);
  rc = check_launch("nkl_add_rmsnorm");
  if (rc) return rc;
  return dtype == NKL_FLOAT32 ? rmsnorm_launch<float>(sum_out, weight, out, rows, cols, eps, st)
                              : rmsnorm_launch<bf16>(sum_out, weight, out, rows, cols, eps, st);
}

extern "C" int nkl_softmax(const void* x, void* out, int64_t rows, int64_t cols, int dtype, void* stream) {
  int rc = check_rows("nkl_softmax", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!x || !out) return fail(NKL_ERR_ARG, "nkl_softmax: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NKL_FLOAT32 ? softmax_launch<float>(x, out, rows, cols, st)
                              : softmax_launch<bf16>(x, out, rows, cols, st);
}

extern "C" size_t nkl_softmax_unfused_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  // rows * cols fp32 values plus two fp32 per row; sizes whose byte count does not fit
  // in size_t report SIZE_MAX, which no workspace can satisfy
  const size_t limit = (SIZE_MAX - 4096) / sizeof(float);
  if ((uint64_t)cols > limit || (uint64_t)rows > limit / (uint64_t)cols) return SIZE_MAX;
  return 2 * round256((size_t)rows * sizeof(float)) + round256((size_t)rows * (size_t)cols * sizeof(float));
}

extern "C" int nkl_softmax_unfused(const void* x, void* out, void* workspace, size_t workspace_bytes,
                                   int64_t rows, int64_t cols, int dtype, void* stream) {
  int rc = check_rows("nkl_softmax_unfused", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!x || !out || !workspace) return fail(NKL_ERR_ARG, "nkl_softmax_unfused: NULL pointer");
  if (nkl_softmax_unfused_workspace_size(rows, cols) == SIZE_MAX)
    return fail(NKL_ERR_SHAPE, "nkl_softmax_unfused: [%lld, %lld] is too large for any workspace", (long long)rows,
                (long long)cols);
  if (workspace_bytes < nkl_softmax_unfused_workspace_size(rows, cols))
    return fail(NKL_ERR_ARG, "nkl_softmax_unfused: workspace %zu B < required %zu B", workspace_bytes,
                nkl_softmax_unfused_workspace_size(rows, cols));
  if (!is_aligned(workspace, 256)) return fail(NKL_ERR_ALIGN, "nkl_softmax_unfused: workspace not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NKL_FLOAT32 ? softmax_unfused_launch<float>(x, out, workspace, rows, cols, st)
                              : softmax_unfused_launch<bf16>(x, out, workspace, rows, cols, st);
}

extern "C" int nkl_swiglu(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
                          int dtype, void* stream) {
  int rc = check_rows("nkl_swiglu", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!gate || !up || !out) return fail(NKL_ERR_ARG, "nkl_swiglu: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NKL_FLOAT32 ? swiglu_launch<float>(gate, up, out, rows * cols, st)
                              : swiglu_launch<bf16>(gate, up, out, rows * cols, st);
}

// ------------------------------------------------------------------ allocation-free variant
// nkl_softmax_unfused_static: the three-pass softmax above with its scratch (row maxima,
// row sums, fp32 exponentials) in a fixed array that lives in this library's device
// image instead of a caller-supplied workspace. It exists for callers that cannot call
// cudaMalloc: hosts that bind only this C ABI from a language runtime with no CUDA
// allocator binding, or that run inside a device-memory budget owned by another
// allocator and may not take memory outside it.
//
// The array is NKL_SOFTMAX_UNFUSED_STATIC_BYTES (16 MiB). Every GPU that loads the
// library holds it until the process exits. Its host-side name is only a stand-in for
// the device symbol, so the device address is looked up with cudaGetSymbolAddress, once
// per device, with that device current, on the first call made on that device.
namespace nkl {
namespace {

static __device__ __align__(256) unsigned char g_softmax_static_scratch[NKL_SOFTMAX_UNFUSED_STATIC_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_static_scratch_mu;
void* g_static_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_softmax_static_scratch on the current device (looked up once).
int static_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "nkl_softmax_unfused_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(NKL_ERR_ARG, "nkl_softmax_unfused_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_softmax_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(NKL_ERR_CUDA, "nkl_softmax_unfused_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_static_scratch_addr[dev] = p;
  }
  *out = g_static_scratch_addr[dev];
  return NKL_OK;
}

}  // namespace
}  // namespace nkl

extern "C" int nkl_softmax_unfused_static(const void* x, void* out, int64_t rows, int64_t cols, int dtype,
                                          void* stream) {
  int rc = check_rows("nkl_softmax_unfused_static", rows, cols, dtype);
  if (rc) return rc;
  if (rows == 0) return NKL_OK;
  if (!x || !out) return fail(NKL_ERR_ARG, "nkl_softmax_unfused_static: NULL pointer");
  // rows * cols is bounded before any product is formed, so no size can wrap around
  constexpr uint64_t kStaticFloats = NKL_SOFTMAX_UNFUSED_STATIC_BYTES / sizeof(float);
  const bool fits = (uint64_t)cols <= kStaticFloats && (uint64_t)rows <= kStaticFloats / (uint64_t)cols;
  const size_t need = fits ? nkl_softmax_unfused_workspace_size(rows, cols) : SIZE_MAX;
  if (!fits || need > (size_t)NKL_SOFTMAX_UNFUSED_STATIC_BYTES)
    return fail(NKL_ERR_SHAPE,
                "nkl_softmax_unfused_static: [%lld, %lld] needs %zu B of scratch, above the fixed %zu B "
                "(use nkl_softmax_unfused with a caller-owned workspace)",
                (long long)rows, (long long)cols, need, (size_t)NKL_SOFTMAX_UNFUSED_STATIC_BYTES);
  void* scratch = nullptr;
  rc = static_scratch_address(&scratch);
  if (rc) return rc;
  // Every scratch byte a pass reads was written by an earlier pass of the same call,
  // so the array needs no clearing between calls.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NKL_FLOAT32 ? softmax_unfused_launch<float>(x, out, scratch, rows, cols, st)
                              : softmax_unfused_launch<bf16>(x, out, scratch, rows, cols, st);
}

extern "C" int nkl_rope(const void* x, void* out, int64_t heads, int64_t seq, int64_t head_dim, float base,
                        int64_t pos_offset, int dtype, void* stream) {
  using namespace nkl;
  if (!valid_dtype(dtype)) return fail(NKL_ERR_DTYPE, "nkl_rope: unsupported dtype %d", dtype);
  const int64_t V = 16 / (int64_t)dtype_size(dtype);
  if (heads < 0 || seq < 0 || head_dim <= 0 || head_dim % (2 * V) != 0 || head_dim > 65536)
    return fail(NKL_ERR_SHAPE, "nkl_rope: head_dim must be a positive multiple of %lld (got %lld)", (long long)(2 * V),
                (long long)head_dim);
  if (!(base > 1.0f) || pos_offset < 0 || seq + pos_offset > (1LL << 24))
    return fail(NKL_ERR_ARG, "nkl_rope: need base > 1 and 0 <= positions < 2^24");
  if (heads == 0 || seq == 0) return NKL_OK;
  if (!x || !out) return fail(NKL_ERR_ARG, "nkl_rope: NULL pointer");
  if (!is_aligned(x, 16) || !is_aligned(out, 16)) return fail(NKL_ERR_ALIGN, "nkl_rope: tensors must be 16-byte aligned");
  const int64_t rows = heads * seq;
  const int64_t threads = rows * (head_dim / 2 / V);
  const dim3 grid((unsigned)((threads + 255) / 256));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NKL_BFLOAT16)
    return launch_pdl(rope_kernel<bf16>, grid, dim3(256), 0, st, "nkl_rope", static_cast<const bf16*>(x),
                      static_cast<bf16*>(out), rows, (int)seq, (int)head_dim, base, (int)pos_offset);
  return launch_pdl(rope_kernel<float>, grid, dim3(256), 0, st, "nkl_rope", static_cast<const float*>(x),
                    static_cast<float*>(out), rows, (int)seq, (int)head_dim, base, (int)pos_offset);
}
