// b2g_gemm_mxf4_noalloc: the a4w4 GEMM on scratch memory that the library
// itself holds, for callers that must not allocate device memory per call.
//
// Who cannot allocate, and why:
//  - a process that reserves (nearly) all of HBM up front for its own pool,
//    e.g. a serving engine holding weights and KV pages; a cudaMalloc issued
//    later may fail outright or split the reserved space;
//  - a host reached through an FFI (C, Go, Java, ...) that has no caching
//    device allocator and would otherwise pay cudaMalloc and cudaFree around
//    every call; cudaFree waits for the whole device, which a latency-bound
//    loop cannot afford.
//
// The scratch is one file-scope __device__ array; every device the library's
// module is loaded on has its own copy. Its address is looked up once per
// device, by the first call made while that device is current, and is then
// handed to the kernels like any workspace pointer. Nothing in this file, nor
// in the path it calls, allocates device memory.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "b2g.h"
#include "capi_internal.h"

static __device__ __align__(256) uint8_t g_noalloc_scratch[B2G_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_addr[kMaxDevices];
std::mutex g_setup_mutex;

// This device's copy of the scratch. The first call per device resolves it
// (which may load this module onto the device); later calls read the cache.
int scratch_for_device(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) return B2G_ENODEVICE;
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();  // do not leave the failure in the caller's error state
        return e != cudaSuccess ? static_cast<int>(e) : B2G_ENODEVICE;
      }
      g_scratch_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return B2G_OK;
}

}  // namespace

extern "C" int b2g_gemm_mxf4_noalloc(const uint8_t* A, int64_t lda, const uint8_t* B,
                                     int64_t ldb, const uint8_t* sfa, int64_t sfa_s0,
                                     int64_t sfa_s1, const uint8_t* sfb, int64_t sfb_s0,
                                     int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K,
                                     int out_dtype, int* status, void* stream) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return B2G_ENODEVICE;
  }
  void* scratch = nullptr;
  const int rc = scratch_for_device(dev, &scratch);
  if (rc != B2G_OK) return rc;
  return b2g::gemm_mxf4_fixed_scratch(A, lda, B, ldb, sfa, sfa_s0, sfa_s1, sfb, sfb_s0, sfb_s1,
                                      C, ldc, M, N, K, out_dtype, scratch,
                                      B2G_NOALLOC_SCRATCH_BYTES, status,
                                      static_cast<cudaStream_t>(stream));
}
