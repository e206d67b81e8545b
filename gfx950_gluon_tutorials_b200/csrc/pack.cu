// Quantise-and-pack kernels for the low-precision operands, and the relayout
// of E8M0 scales into the blocked layout the GEMM's TMA loads.
//
// The reference has no quantiser: its bench draws random packed nibbles and
// random scale bytes (kernels/gemm/intra_wave/a4w4/bench.py:115-146) and casts
// to BF8 with torch (kernels/gemm/intra_wave/a8w8/bench.py:133-134). What it
// does fix is the storage format these kernels produce:
//   - e2m1 codes, two per byte, even k in the low nibble, value table
//     {0, .5, 1, 1.5, 2, 3, 4, 6} with bit 3 the sign (a4w4/bench.py:80-105);
//   - E8M0 scale bytes, value 2^(e-127), 255 = NaN (a4w4/bench.py:108-112),
//     stored as a (rows, K/32) tensor of any strides; the reference's own are
//     M-contiguous, (1, rows_pad) (a4w4/bench.py:138-144);
//   - e5m2 bytes with the rounding of torch's float -> float8_e5m2 cast.
// All kernels are HBM-bound streaming passes: coalesced 16-byte loads, one
// thread per 8 source elements.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pack.cuh"

namespace b2g {

// fp32 -> e5m2, round to nearest even, no saturation (overflow -> inf,
// NaN -> 0x7F with the sign kept). e5m2: bias 15, normals from 2^-14,
// subnormals m * 2^-16 (m = 1..3), largest finite 57344.
__device__ __forceinline__ uint32_t e5m2_from_f32(float y) {
  const uint32_t u = __float_as_uint(y);
  const uint32_t sign = (u >> 24) & 0x80u;
  uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return sign | 0x7Fu;   // NaN
  if (a >= 0x47700000u) return sign | 0x7Cu;  // >= 61440 (the tie above 57344) and inf
  if (a >= 0x38800000u) {                     // >= 2^-14: normal
    a += 0x000FFFFFu + ((a >> 21) & 1u);      // round the 21 dropped bits, ties to even
    return sign | (((a >> 23) - 112u) << 2) | ((a >> 21) & 3u);
  }
  // below 2^-14: integer multiple of 2^-16, the value 4 being 2^-14 itself
  const float v = __uint_as_float(a) * 65536.0f;
  return sign | static_cast<uint32_t>(rintf(v));
}

// |y| -> e2m1 magnitude code (0..7), round to nearest even, saturating at 6.
__device__ __forceinline__ uint32_t e2m1_mag_code(float a) {
  if (a <= 0.25f) return 0u;
  if (a < 0.75f) return 1u;
  if (a <= 1.25f) return 2u;
  if (a < 1.75f) return 3u;
  if (a <= 2.5f) return 4u;
  if (a < 3.5f) return 5u;
  if (a <= 5.0f) return 6u;
  return 7u;
}

__device__ __forceinline__ uint32_t e2m1_from_f32(float y) {
  return ((__float_as_uint(y) >> 28) & 0x8u) | e2m1_mag_code(fabsf(y));
}

// floor(log2(a)) for a finite a > 0 (exact, from the bits).
__device__ __forceinline__ int32_t floor_log2_f32(float a) {
  const uint32_t u = __float_as_uint(a);
  const int32_t e = static_cast<int32_t>(u >> 23);
  if (e != 0) return e - 127;
  return (31 - __clz(static_cast<int32_t>(u & 0x7FFFFFu))) - 149;  // subnormal
}

// 2^n as fp32 for n in [-127, 127].
__device__ __forceinline__ float exp2i(int32_t n) {
  if (n >= -126) return __uint_as_float(static_cast<uint32_t>(n + 127) << 23);
  return __uint_as_float(0x00400000u);  // 2^-127
}

// ------------------------------------------------------------------ MXFP4 --
// Four lanes per 32-element block, eight elements per lane.
__global__ void quant_mxfp4_kernel(const float* __restrict__ src, int64_t ld, int32_t rows,
                                   int32_t K, uint8_t* __restrict__ q, int64_t ldq,
                                   uint8_t* __restrict__ sc, int64_t s0, int64_t s1) {
  const int64_t blocks_per_row = K / 32;
  const int64_t total = static_cast<int64_t>(rows) * blocks_per_row * 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t warp_base = (static_cast<int64_t>(blockIdx.x) * blockDim.x) + (threadIdx.x & ~31u);
  const uint32_t lane = threadIdx.x & 31u;
  for (int64_t wb = warp_base; wb < total; wb += stride) {  // uniform per warp
    const int64_t i = wb + lane;
    const bool active = i < total;
    const int64_t blk = i >> 2;
    const int32_t part = static_cast<int32_t>(i & 3);
    const int64_t row = active ? blk / blocks_per_row : 0;
    const int64_t jb = active ? blk - row * blocks_per_row : 0;
    const int64_t k0 = jb * 32 + part * 8;
    float x[8];
    if (active) {
      const float4* p = reinterpret_cast<const float4*>(src + row * ld + k0);
      const float4 lo = __ldcs(p), hi = __ldcs(p + 1);
      x[0] = lo.x; x[1] = lo.y; x[2] = lo.z; x[3] = lo.w;
      x[4] = hi.x; x[5] = hi.y; x[6] = hi.z; x[7] = hi.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) x[t] = 0.0f;
    }
    float amax = 0.0f;
    uint32_t nonfinite = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float a = fabsf(x[t]);
      nonfinite |= (__float_as_uint(a) >= 0x7F800000u) ? 1u : 0u;
      amax = fmaxf(amax, a);
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
    }
    uint32_t sbyte, packed = 0;
    if (nonfinite) {
      sbyte = 255u;
    } else if (amax == 0.0f) {
      sbyte = 0u;
      // scale 2^-127: every element rounds to a (signed) zero code
#pragma unroll
      for (int t = 0; t < 8; ++t) packed |= ((__float_as_uint(x[t]) >> 28) & 0x8u) << (4 * t);
    } else {
      int32_t s = floor_log2_f32(amax) - 2;
      if (s < -127) s = -127;
      sbyte = static_cast<uint32_t>(s + 127);
      const float mul = exp2i(-s);
#pragma unroll
      for (int t = 0; t < 8; ++t) packed |= e2m1_from_f32(x[t] * mul) << (4 * t);
    }
    if (active) {
      *reinterpret_cast<uint32_t*>(q + row * ldq + (k0 >> 1)) = packed;
      if (part == 0) sc[row * s0 + jb * s1] = static_cast<uint8_t>(sbyte);
    }
  }
}

// ------------------------------------------------------------ scaled e5m2 --
__global__ void quant_mxe5m2_kernel(const float* __restrict__ src, int64_t ld, int32_t rows,
                                    int32_t K, const uint8_t* __restrict__ sc, int64_t s0,
                                    int64_t s1, uint8_t* __restrict__ q, int64_t ldq) {
  const int64_t per_row = K / 8;
  const int64_t total = static_cast<int64_t>(rows) * per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t row = i / per_row;
    const int64_t k0 = (i - row * per_row) * 8;
    const uint32_t e = sc[row * s0 + (k0 >> 5) * s1];
    const float4* p = reinterpret_cast<const float4*>(src + row * ld + k0);
    const float4 lo = __ldcs(p), hi = __ldcs(p + 1);
    const float x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint32_t w0 = 0, w1 = 0;
    if (e != 255u) {
      const float mul = exp2i(127 - static_cast<int32_t>(e));
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        w0 |= e5m2_from_f32(x[t] * mul) << (8 * t);
        w1 |= e5m2_from_f32(x[t + 4] * mul) << (8 * t);
      }
    }
    *reinterpret_cast<uint2*>(q + row * ldq + k0) = make_uint2(w0, w1);
  }
}

// ------------------------------------------------------------ plain e5m2 --
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__global__ void cast_e5m2_kernel(const T* __restrict__ src, int64_t n, uint8_t* __restrict__ dst) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = static_cast<uint8_t>(e5m2_from_f32(to_f32<T>(src[i])));
}


// ------------------------------------------------------- scale relayout --
// (rows, K/32) E8M0 bytes of any strides -> blocked layout: for 128-row block
// rb and 4-scale group g, 512 bytes at (rb * groups + g) * 512 where byte
// r0 * 16 + r1 * 4 + j holds the scale of row rb*128 + r1*32 + r0, k-block
// 4g + j. That is the 32 lanes x 16 bytes source of a 32x128b (warpx4)
// tcgen05.cp, which spreads it into the TMEM scale-factor layout of a
// 128-row operand. Positions past the matrix hold 127 (scale 1.0). One launch
// converts both operands: threads [0, n_a) do A, the rest B.
struct RelayoutArgs {
  const uint8_t* src;
  int64_t s0, s1;
  int32_t rows, row_blocks;
  uint8_t* dst;
};

__global__ void sf_relayout_kernel(RelayoutArgs a, RelayoutArgs b, int32_t kscales,
                                   int32_t groups) {
  const int64_t n_a = static_cast<int64_t>(a.row_blocks) * groups * 32;
  const int64_t total = n_a + static_cast<int64_t>(b.row_blocks) * groups * 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const bool is_a = i < n_a;
    const RelayoutArgs& t = is_a ? a : b;
    const int64_t li = is_a ? i : i - n_a;
    const int32_t r0 = static_cast<int32_t>(li & 31);
    const int64_t q = li >> 5;
    const int32_t g = static_cast<int32_t>(q % groups);
    const int64_t rb = q / groups;
    uint32_t w[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int64_t row = rb * 128 + r1 * 32 + r0;
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int32_t k = g * 4 + j;
        const uint32_t v =
            (row < t.rows && k < kscales) ? __ldg(t.src + row * t.s0 + k * t.s1) : 127u;
        word |= v << (8 * j);
      }
      w[r1] = word;
    }
    *reinterpret_cast<uint4*>(t.dst + (rb * groups + g) * 512 + r0 * 16) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

static int grid_for(int64_t work, int threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

cudaError_t launch_quant_mxfp4(const float* src, int64_t ld, int rows, int K, uint8_t* q,
                               int64_t ldq, uint8_t* sc, int64_t s0, int64_t s1,
                               cudaStream_t stream) {
  const int64_t work = static_cast<int64_t>(rows) * (K / 32) * 4;
  quant_mxfp4_kernel<<<grid_for(work, 256), 256, 0, stream>>>(src, ld, rows, K, q, ldq, sc, s0,
                                                              s1);
  return cudaGetLastError();
}

cudaError_t launch_quant_mxe5m2(const float* src, int64_t ld, int rows, int K,
                                const uint8_t* sc, int64_t s0, int64_t s1, uint8_t* q,
                                int64_t ldq, cudaStream_t stream) {
  const int64_t work = static_cast<int64_t>(rows) * (K / 8);
  quant_mxe5m2_kernel<<<grid_for(work, 256), 256, 0, stream>>>(src, ld, rows, K, sc, s0, s1, q,
                                                               ldq);
  return cudaGetLastError();
}

cudaError_t launch_cast_e5m2(const void* src, int dtype, int64_t n, uint8_t* dst,
                             cudaStream_t stream) {
  const int g = grid_for(n, 256);
  if (dtype == 2)
    cast_e5m2_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(src), n, dst);
  else if (dtype == 0)
    cast_e5m2_kernel<__half><<<g, 256, 0, stream>>>(static_cast<const __half*>(src), n, dst);
  else
    cast_e5m2_kernel<__nv_bfloat16>
        <<<g, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), n, dst);
  return cudaGetLastError();
}

cudaError_t launch_sf_relayout(const uint8_t* sa, int64_t sa0, int64_t sa1, int rows_a,
                               uint8_t* dst_a, const uint8_t* sb, int64_t sb0, int64_t sb1,
                               int rows_b, uint8_t* dst_b, int kscales, cudaStream_t stream) {
  const int32_t groups = (kscales + 3) / 4;
  RelayoutArgs a{sa, sa0, sa1, rows_a, (rows_a + 127) / 128, dst_a};
  RelayoutArgs b{sb, sb0, sb1, rows_b, (rows_b + 127) / 128, dst_b};
  if (sa == nullptr) a.row_blocks = 0;
  if (sb == nullptr) b.row_blocks = 0;
  const int64_t work = (static_cast<int64_t>(a.row_blocks) + b.row_blocks) * groups * 32;
  if (work == 0) return cudaSuccess;
  sf_relayout_kernel<<<grid_for(work, 256), 256, 0, stream>>>(a, b, kscales, groups);
  return cudaGetLastError();
}

}  // namespace b2g
