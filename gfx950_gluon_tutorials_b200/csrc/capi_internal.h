// Library-internal entry shared between capi.cu and noalloc.cu (hidden
// visibility: not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdint>

namespace b2g {

// b2g_gemm_mxf4 with `scratch` (256-byte aligned, `capacity` bytes) in place
// of a caller workspace. Returns B2G_ECAPACITY, launching nothing, when the
// problem needs more than `capacity`; otherwise clears the stream-K flag words
// of the scratch on `stream` and launches exactly what b2g_gemm_mxf4 would.
int gemm_mxf4_fixed_scratch(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                            const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1,
                            const uint8_t* sfb, int64_t sfb_s0, int64_t sfb_s1, void* C,
                            int64_t ldc, int M, int N, int K, int out_dtype, void* scratch,
                            size_t capacity, int* status, cudaStream_t stream);

// SM count of the current device, or -1 when it is not an sm_100 part.
int current_device_sms();

// cuTensorMapEncodeTiled from the driver, or null.
PFN_cuTensorMapEncodeTiled_v12000 tma_encoder();

// The bounded-wait limit (B2G_OPT_TIMEOUT_MS) in nanoseconds.
uint64_t wait_timeout_ns();

}  // namespace b2g
