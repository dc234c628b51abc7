// capi.cu - library-level C entry points: version, status strings, the per-thread
// error message and the device-failure check. The op entry points live beside their
// kernels (rows.cu, gemm.cu, attention.cu).
#include <atomic>

#include <cstring>

#include "common.cuh"

namespace nkl {

char* last_error_buffer() {
  static thread_local char buf[512] = {0};
  return buf;
}

// SMs the persistent kernels of the calling host thread may fill (0: all); see
// nkl_set_sm_budget.
thread_local int g_sm_budget = 0;

int sm_count() {
  static std::atomic<int> cached[64] = {};  // per device, filled once (idempotent)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return (g_sm_budget > 0 && g_sm_budget < n) ? g_sm_budget : n;
}

}  // namespace nkl

extern "C" int nkl_abi_version(void) { return NKL_ABI_VERSION; }

extern "C" const char* nkl_status_string(int status) {
  switch (status) {
    case NKL_OK: return "ok";
    case NKL_ERR_SHAPE: return "unsupported shape";
    case NKL_ERR_DTYPE: return "unsupported dtype";
    case NKL_ERR_ALIGN: return "misaligned pointer";
    case NKL_ERR_CUDA: return "CUDA error";
    case NKL_ERR_ARG: return "invalid argument";
    case NKL_ERR_DEVICE: return "device-side failure (bounded wait expired)";
    default: return "unknown status";
  }
}

extern "C" const char* nkl_last_error(void) { return nkl::last_error_buffer(); }

extern "C" int nkl_check_device(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return nkl::fail(NKL_ERR_CUDA, "nkl_check_device: %s", cudaGetErrorString(e));
  const int g = nkl::gemm_read_and_clear_device_error();
  const int a = nkl::attention_read_and_clear_device_error();
  if (g < 0 || a < 0) return nkl::fail(NKL_ERR_CUDA, "nkl_check_device: could not read the device flag");
  if (g || a)
    return nkl::fail(NKL_ERR_DEVICE, "nkl_check_device: kernel gave up waiting (gemm code %d, attention code %d)", g, a);
  return NKL_OK;
}

// ---- device memory shared between the processes of one node (CUDA IPC), for the
// all-gather's output buffers and flag arrays

extern "C" size_t nkl_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int nkl_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return nkl::fail(NKL_ERR_ARG, "nkl_ipc_alloc: bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return nkl::fail(NKL_ERR_CUDA, "nkl_ipc_alloc: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return NKL_OK;
}

extern "C" int nkl_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return nkl::fail(NKL_ERR_ARG, "nkl_ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? NKL_OK : nkl::fail(NKL_ERR_CUDA, "nkl_ipc_open: %s", cudaGetErrorString(e));
}

extern "C" int nkl_ipc_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? NKL_OK : nkl::fail(NKL_ERR_CUDA, "nkl_ipc_close: %s", cudaGetErrorString(e));
}

extern "C" int nkl_ipc_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? NKL_OK : nkl::fail(NKL_ERR_CUDA, "nkl_ipc_free: %s", cudaGetErrorString(e));
}

extern "C" int nkl_set_sm_budget(int sms, int* previous) {
  if (sms < 0) return nkl::fail(NKL_ERR_ARG, "nkl_set_sm_budget: negative SM count %d", sms);
  if (previous) *previous = nkl::g_sm_budget;
  nkl::g_sm_budget = sms;
  return NKL_OK;
}
