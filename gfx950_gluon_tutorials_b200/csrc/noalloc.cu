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
// The scratch is one file-scope __device__ array; every CUDA context the
// library's module is loaded in has its own copy. Its address belongs to that
// context, so it is cached per device together with the unique ID of the
// context it was looked up in (cuCtxGetId): a call made in another context on
// the same device (after cudaDeviceReset, or a context a driver-API host made
// current) looks the address up again in that context instead of using a
// stale one. Nothing in this file, nor in the path it calls, allocates device
// memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "b2g.h"
#include "capi_internal.h"

static __device__ __align__(256) uint8_t g_noalloc_scratch[B2G_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

struct ScratchCache {
  unsigned long long ctx_id;  // cuCtxGetId of the context `addr` belongs to
  void* addr;                 // null: not looked up yet
};
ScratchCache g_cache[kMaxDevices];
std::mutex g_cache_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique ID of the context current on this thread (0 when none is current).
int current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    cudaGetLastError();
  });
  if (get_current == nullptr || get_id == nullptr) return B2G_ENODEVICE;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return B2G_ENODEVICE;
  *id = 0;
  if (ctx != nullptr && get_id(ctx, id) != CUDA_SUCCESS) return B2G_ENODEVICE;
  return B2G_OK;
}

// The scratch of the context current on device `dev`. The first call in a
// context resolves it with cudaGetSymbolAddress (which may load this module
// into the context, and makes the device's primary context current if none
// is); later calls in the same context read the cache.
int scratch_for_device(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) return B2G_ENODEVICE;
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  unsigned long long id = 0;
  int rc = current_context_id(&id);
  if (rc != B2G_OK) return rc;
  ScratchCache& c = g_cache[dev];
  if (c.addr != nullptr && id != 0 && c.ctx_id == id) {
    *out = c.addr;
    return B2G_OK;
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    cudaGetLastError();  // do not leave the failure in the caller's error state
    return e != cudaSuccess ? static_cast<int>(e) : B2G_ENODEVICE;
  }
  // the lookup made a context current if none was: key the cache on it
  rc = current_context_id(&id);
  if (rc != B2G_OK || id == 0) return rc != B2G_OK ? rc : B2G_ENODEVICE;
  c.ctx_id = id;
  c.addr = p;
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
