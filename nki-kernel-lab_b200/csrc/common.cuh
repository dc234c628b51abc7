// common.cuh - shared host/device helpers for the nkilab B200 kernels.
//
// Host side: argument checks that turn into nkl_status codes plus a per-thread
// error message (the reference raises Python AssertionError from kernel asserts,
// e.g. nkilab/kernels/matmul.py:29,57-58 and nkilab/kernels/attention.py:38; a C
// ABI cannot raise, so it returns a code and keeps the message).
// Device side: bf16/fp32 element access, 16-byte vector types and warp reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/nkilab.h"

namespace nkl {

// ---------------------------------------------------------------- host errors

// Message buffer of the last failing call on this thread (see nkl_last_error).
char* last_error_buffer();

inline int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(last_error_buffer(), 512, fmt, ap);
  va_end(ap);
  return status;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NKL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NKL_OK;
}

inline bool is_aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline bool valid_dtype(int dt) { return dt == NKL_FLOAT32 || dt == NKL_BFLOAT16; }
inline size_t dtype_size(int dt) { return dt == NKL_FLOAT32 ? 4 : 2; }

// Number of SMs of the current device (148 on B200), cached per device.
int sm_count();

// Device-failure flag readers, one per translation unit that waits on barriers.
int gemm_read_and_clear_device_error();
int attention_read_and_clear_device_error();

// ---------------------------------------------------------------- device helpers

typedef __nv_bfloat16 bf16;

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(bf16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float v) { return __float2bfloat16_rn(v); }

// A 16-byte vector of T: 8 bf16 or 4 fp32 lanes.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    if constexpr (sizeof(T) == 4) {
      return reinterpret_cast<const float*>(&raw)[i];
    } else {
      return __bfloat162float(reinterpret_cast<const bf16*>(&raw)[i]);
    }
  }
};

// Pack N floats into a 16-byte vector of T with round-to-nearest-even.
template <typename T> __device__ __forceinline__ uint4 pack16(const float* f) {
  uint4 r;
  if constexpr (sizeof(T) == 4) {
    r.x = __float_as_uint(f[0]); r.y = __float_as_uint(f[1]);
    r.z = __float_as_uint(f[2]); r.w = __float_as_uint(f[3]);
  } else {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(f[0], f[1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(f[2], f[3]);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(f[4], f[5]);
    __nv_bfloat162 h3 = __floats2bfloat162_rn(f[6], f[7]);
    r.x = *reinterpret_cast<uint32_t*>(&h0); r.y = *reinterpret_cast<uint32_t*>(&h1);
    r.z = *reinterpret_cast<uint32_t*>(&h2); r.w = *reinterpret_cast<uint32_t*>(&h3);
  }
  return r;
}

// Streaming 16-byte global load that does not allocate in L1 (data is touched once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch. A kernel launched with launch_pdl() lets the next
// kernel of the stream start launching as soon as every CTA of this one has begun
// (launch_dependents), and waits for the previous kernel of the stream to complete and
// publish its memory (wait) before it reads anything. Stream order is unchanged; what
// overlaps is one kernel's launch latency and ramp with the previous kernel's drain.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// The two halves of pdl_enter, for kernels that prefetch between them.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Ask L2 to fetch [p, p + bytes) (p 16-byte aligned, bytes a multiple of 16). Issued
// before pdl_wait it overlaps a kernel's first HBM reads with the previous kernel's
// tail; a prefetch only warms L2, the point of coherence, so it is correct even while
// the previous kernel is still writing that memory (the loads after the wait read the
// final data).
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char* what,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // a refused launch must not be reported again by the next call
    return fail(NKL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return NKL_OK;
}

// exp(x) for the row kernels: the accurate library expf for fp32 outputs (the
// reference's fp32 tolerances are 1e-5), the fast hardware-approximate __expf when
// the result is rounded to bf16 (its error is far below one bf16 ulp).
template <typename T> __device__ __forceinline__ float row_exp(float x) {
  if constexpr (sizeof(T) == 4) return expf(x);
  else return __expf(x);
}

// silu(g) = g / (1 + exp(-g)) in fp32 (nkilab/kernels/norm.py:131-132): the accurate
// expf and a true division for fp32 outputs, the fast forms when the product is rounded
// to bf16. Shared by the SwiGLU row kernel and the GEMM's fused SwiGLU epilogue so the
// two paths round identically.
template <typename T> __device__ __forceinline__ float silu_f32(float g) {
  if constexpr (sizeof(T) == 4) return g / (1.0f + expf(-g));
  else return __fdividef(g, 1.0f + __expf(-g));
}

}  // namespace nkl
