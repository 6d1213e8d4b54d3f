// b2g_timing.cu — device side of the candidate timer: a stream gate the host releases.
//
// To time kernels of a few microseconds with CUDA events, the GPU must find every timed launch already queued when
// it reaches the first one; otherwise the events measure the host's launch rate. The timer therefore queues a
// one-thread kernel that spins on a flag in mapped, pinned host memory, enqueues the whole chunk of samples behind
// it, and then sets the flag. The spin is bounded: after `timeout_ns` the kernel records a status code and returns,
// so a host that never releases the gate (it died, or forgot) costs at most that long and leaves the stream usable.

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "b2g.h"

namespace b2g {

constexpr int kStatusHoldTimeout = 0x201;  // b2g_status_string names it

__device__ __forceinline__ uint64_t timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int32_t load_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void hold_kernel(const int32_t* flag, int32_t expect, uint64_t timeout_ns, int32_t* status) {
  const uint64_t t0 = timer_ns();
  while (load_sys(flag) != expect) {
    if (timer_ns() - t0 > timeout_ns) {
      if (status) atomicCAS(status, 0, kStatusHoldTimeout);
      return;
    }
    __nanosleep(256);
  }
}

}  // namespace b2g

namespace b2g {
int32_t record_error(int32_t code, const std::string& msg);  // b2g_gemm.cu: sets b2g_last_error()
}

namespace {
int32_t tfail(int32_t code, const char* what, cudaError_t e) {
  return b2g::record_error(code, std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

extern "C" {

int32_t b2g_host_flag_create(int32_t** host_ptr, int32_t** device_ptr) {
  if (!host_ptr || !device_ptr) return B2G_ERR_INVALID_ARG;
  *host_ptr = nullptr;
  *device_ptr = nullptr;
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) return tfail(B2G_ERR_CUDA, "cudaHostAlloc", e);
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaFreeHost(h);
    return tfail(B2G_ERR_CUDA, "cudaHostGetDevicePointer", e);
  }
  __atomic_store_n(static_cast<int32_t*>(h), 0, __ATOMIC_SEQ_CST);
  *host_ptr = static_cast<int32_t*>(h);
  *device_ptr = static_cast<int32_t*>(d);
  return B2G_OK;
}

int32_t b2g_host_flag_set(int32_t* host_ptr, int32_t value) {
  if (!host_ptr) return B2G_ERR_INVALID_ARG;
  __atomic_store_n(host_ptr, value, __ATOMIC_SEQ_CST);
  return B2G_OK;
}

int32_t b2g_host_flag_destroy(int32_t* host_ptr) {
  if (!host_ptr) return B2G_OK;
  cudaError_t e = cudaFreeHost(host_ptr);
  return e == cudaSuccess ? B2G_OK : tfail(B2G_ERR_CUDA, "cudaFreeHost", e);
}

int32_t b2g_hold(const int32_t* device_flag, int32_t expect, uint64_t timeout_ns, int32_t* status, void* stream) {
  if (!device_flag) return B2G_ERR_INVALID_ARG;
  b2g::hold_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(device_flag, expect, timeout_ns, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B2G_OK : tfail(B2G_ERR_CUDA, "hold launch", e);
}

}  // extern "C"
