// Host launchers of the pack / relayout kernels (pack.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b2g {

cudaError_t launch_quant_mxfp4(const float* src, int64_t ld, int rows, int K, uint8_t* q,
                               int64_t ldq, uint8_t* sc, int64_t s0, int64_t s1,
                               cudaStream_t stream);
cudaError_t launch_quant_mxe5m2(const float* src, int64_t ld, int rows, int K,
                                const uint8_t* sc, int64_t s0, int64_t s1, uint8_t* q,
                                int64_t ldq, cudaStream_t stream);
cudaError_t launch_cast_e5m2(const void* src, int dtype, int64_t n, uint8_t* dst,
                             cudaStream_t stream);
// Converts up to two (rows, K/32) scale tensors (either may be null) into the
// blocked layout in one launch.
cudaError_t launch_sf_relayout(const uint8_t* sa, int64_t sa0, int64_t sa1, int rows_a,
                               uint8_t* dst_a, const uint8_t* sb, int64_t sb0, int64_t sb1,
                               int rows_b, uint8_t* dst_b, int kscales, cudaStream_t stream);

}  // namespace b2g
