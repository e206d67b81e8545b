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
// All kernels are HBM-bound streaming passes (several 16-byte loads in flight
// per lane); the element conversions use the hardware cvt instructions.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "pack.cuh"
#include "ptx.cuh"

namespace b2g {

// Load flavour of the streaming passes (build macro B2G_PACK_LOAD: 0 plain,
// 1 read-only path, 2 evict-first streaming).
#ifndef B2G_PACK_LOAD
#define B2G_PACK_LOAD 0
#endif
template <typename T>
__device__ __forceinline__ T stream_load(const T* p) {
#if B2G_PACK_LOAD == 1
  return __ldg(p);
#elif B2G_PACK_LOAD == 2
  return __ldcs(p);
#else
  return *p;
#endif
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

// Hardware conversions (sm_100a). cvt.rn.satfinite rounds to nearest even
// and saturates finite overflow to the largest finite code; `hi` lands in the
// upper half of the result.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ uint32_t cvt_e5m2x2_satfinite(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %2, %1;" : "=h"(r) : "f"(lo), "f"(hi));
  return r;
}

// torch's float -> float8_e5m2 cast does not saturate: magnitudes from 61440
// (the rounding midpoint above 57344) up, infinities included, become
// infinity, and a NaN keeps its sign (0x7F | sign).
__device__ __forceinline__ uint32_t e5m2_fix(uint32_t code, float y) {
  const uint32_t u = __float_as_uint(y);
  const uint32_t sign = (u >> 24) & 0x80u;
  const uint32_t a = u & 0x7FFFFFFFu;
  code = a >= 0x47700000u ? (sign | 0x7Cu) : code;
  return a > 0x7F800000u ? (sign | 0x7Fu) : code;
}

__device__ __forceinline__ uint32_t e5m2x4(float a, float b, float c, float d) {
  const uint32_t lo = cvt_e5m2x2_satfinite(a, b), hi = cvt_e5m2x2_satfinite(c, d);
  return e5m2_fix(lo & 0xFFu, a) | (e5m2_fix(lo >> 8, b) << 8) | (e5m2_fix(hi & 0xFFu, c) << 16) |
         (e5m2_fix(hi >> 8, d) << 24);
}

// ------------------------------------------------------------------ MXFP4 --
// A warp takes segments of 256 elements (8 blocks of 32) of one row; four
// lanes share a block, eight elements (32 bytes) each. kSegs segments per
// warp iteration keep 32 * kSegs bytes per lane in flight. IDX is the index
// type (32-bit unless the segment count needs 64).
template <typename IDX, int kSegs>
__global__ void __launch_bounds__(256) quant_mxfp4_kernel(const float* __restrict__ src,
                                                          int64_t ld, int32_t rows, int32_t K,
                                                          uint8_t* __restrict__ q, int64_t ldq,
                                                          uint8_t* __restrict__ sc, int64_t s0,
                                                          int64_t s1) {
  const IDX blocks_per_row = static_cast<IDX>(K / 32);
  const IDX segs_per_row = (blocks_per_row + 7) / 8;
  const IDX total = static_cast<IDX>(rows) * segs_per_row;
  const IDX nwarps = static_cast<IDX>(gridDim.x) * (blockDim.x / 32);
  const uint32_t lane = threadIdx.x & 31u;
  const IDX jl = static_cast<IDX>(lane >> 2);  // block within the segment
  const int32_t part = static_cast<int32_t>(lane & 3u);
  for (IDX seg0 = static_cast<IDX>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
       seg0 < total; seg0 += nwarps * kSegs) {  // uniform per warp
    float x[kSegs][8];
    IDX row[kSegs], jb[kSegs];
    bool on[kSegs];
#pragma unroll
    for (int u = 0; u < kSegs; ++u) {
      const IDX seg = seg0 + static_cast<IDX>(u) * nwarps;
      row[u] = seg / segs_per_row;
      jb[u] = (seg - row[u] * segs_per_row) * 8 + jl;
      on[u] = seg < total && jb[u] < blocks_per_row;
      if (on[u]) {
        const float4* p = reinterpret_cast<const float4*>(
            src + static_cast<int64_t>(row[u]) * ld + static_cast<int64_t>(jb[u]) * 32 + part * 8);
        const float4 lo = stream_load(p), hi = stream_load(p + 1);
        x[u][0] = lo.x; x[u][1] = lo.y; x[u][2] = lo.z; x[u][3] = lo.w;
        x[u][4] = hi.x; x[u][5] = hi.y; x[u][6] = hi.z; x[u][7] = hi.w;
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) x[u][t] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kSegs; ++u) {
      float amax = 0.0f;
#pragma unroll
      for (int t = 0; t < 8; ++t) amax = fmaxf(amax, fabsf(x[u][t]));
      // fmaxf drops NaN: flag non-finite elements separately
      uint32_t nonfinite = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) nonfinite |= (__float_as_uint(x[u][t]) & 0x7F800000u) == 0x7F800000u;
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
      }
      uint32_t sbyte, packed = 0;
      if (nonfinite) {
        sbyte = 255u;
      } else if (amax == 0.0f) {
        sbyte = 0u;  // scale 2^-127: every element rounds to a (signed) zero code
#pragma unroll
        for (int t = 0; t < 8; ++t) packed |= ((__float_as_uint(x[u][t]) >> 28) & 0x8u) << (4 * t);
      } else {
        int32_t sx = floor_log2_f32(amax) - 2;
        if (sx < -127) sx = -127;
        sbyte = static_cast<uint32_t>(sx + 127);
        const float mul = exp2i(-sx);
#pragma unroll
        for (int t = 0; t < 8; t += 2)
          packed |= cvt_e2m1x2(x[u][t] * mul, x[u][t + 1] * mul) << (4 * t);
      }
      if (on[u]) {
        const int64_t r = static_cast<int64_t>(row[u]), j = static_cast<int64_t>(jb[u]);
        *reinterpret_cast<uint32_t*>(q + r * ldq + j * 16 + part * 4) = packed;
        if (part == 0) sc[r * s0 + j * s1] = static_cast<uint8_t>(sbyte);
      }
    }
  }
}

// ------------------------------------------------------------ scaled e5m2 --
// One thread per 8 elements (32 bytes loaded), kUnroll groups per iteration.
template <typename IDX, int kUnroll>
__global__ void __launch_bounds__(256) quant_mxe5m2_kernel(const float* __restrict__ src,
                                                           int64_t ld, int32_t rows, int32_t K,
                                                           const uint8_t* __restrict__ sc,
                                                           int64_t s0, int64_t s1,
                                                           uint8_t* __restrict__ q, int64_t ldq) {
  const IDX per_row = static_cast<IDX>(K / 8);
  const IDX total = static_cast<IDX>(rows) * per_row;
  const IDX stride = static_cast<IDX>(gridDim.x) * blockDim.x;
  for (IDX i0 = static_cast<IDX>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < total;
       i0 += stride * kUnroll) {
    float x[kUnroll][8];
    uint32_t e[kUnroll];
    int64_t row[kUnroll], k0[kUnroll];
    bool on[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const IDX i = i0 + static_cast<IDX>(u) * stride;
      on[u] = i < total;
      const IDX r = on[u] ? i / per_row : 0;
      row[u] = static_cast<int64_t>(r);
      k0[u] = static_cast<int64_t>(i - r * per_row) * 8;
      if (on[u]) {
        e[u] = sc[row[u] * s0 + (k0[u] >> 5) * s1];
        const float4* p = reinterpret_cast<const float4*>(src + row[u] * ld + k0[u]);
        const float4 lo = stream_load(p), hi = stream_load(p + 1);
        x[u][0] = lo.x; x[u][1] = lo.y; x[u][2] = lo.z; x[u][3] = lo.w;
        x[u][4] = hi.x; x[u][5] = hi.y; x[u][6] = hi.z; x[u][7] = hi.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (!on[u]) continue;
      uint32_t w0 = 0, w1 = 0;
      if (e[u] != 255u) {
        const float mul = exp2i(127 - static_cast<int32_t>(e[u]));
        w0 = e5m2x4(x[u][0] * mul, x[u][1] * mul, x[u][2] * mul, x[u][3] * mul);
        w1 = e5m2x4(x[u][4] * mul, x[u][5] * mul, x[u][6] * mul, x[u][7] * mul);
      }
      *reinterpret_cast<uint2*>(q + row[u] * ldq + k0[u]) = make_uint2(w0, w1);
    }
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
  {
    const float y = to_f32<T>(src[i]);
    dst[i] = static_cast<uint8_t>(e5m2_fix(cvt_e5m2x2_satfinite(y, 0.0f) & 0xFFu, y));
  }
}

// Four elements per thread and group: one 16-byte (fp32) or 8-byte (fp16 /
// bf16) load and one 4-byte store; kUnroll groups in flight per thread. Needs
// n % 4 == 0 and aligned pointers.
template <typename T, int kUnroll>
__global__ void __launch_bounds__(256) cast_e5m2_x4_kernel(const T* __restrict__ src, int64_t n4,
                                                           uint32_t* __restrict__ dst) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n4;
       i0 += stride * kUnroll) {
    float v[kUnroll][4];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n4) continue;
      if constexpr (sizeof(T) == 4) {
        const float4 f = stream_load(reinterpret_cast<const float4*>(src) + i);
        v[u][0] = f.x; v[u][1] = f.y; v[u][2] = f.z; v[u][3] = f.w;
      } else {
        const uint2 h = stream_load(reinterpret_cast<const uint2*>(src) + i);
        T t[4];
        memcpy(t, &h, sizeof(h));
#pragma unroll
        for (int j = 0; j < 4; ++j) v[u][j] = to_f32<T>(t[j]);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n4) dst[i] = e5m2x4(v[u][0], v[u][1], v[u][2], v[u][3]);
    }
  }
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

template <typename IDX>
__global__ void __launch_bounds__(256) sf_relayout_kernel(RelayoutArgs a, RelayoutArgs b,
                                                          int32_t kscales, int32_t groups) {
  // Launched with programmatic stream serialization: first wait for every
  // earlier kernel (one may still be reading this workspace, or writing the
  // scales or the GEMM's operands), then let the GEMM that reads this output
  // start its prologue and its A/B loads.
  grid_dependency_wait();
  grid_launch_dependents();
  const IDX n_a = static_cast<IDX>(a.row_blocks) * groups * 32;
  const IDX total = n_a + static_cast<IDX>(b.row_blocks) * groups * 32;
  const IDX stride = static_cast<IDX>(gridDim.x) * blockDim.x;
  for (IDX i = static_cast<IDX>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const bool is_a = i < n_a;
    const RelayoutArgs& t = is_a ? a : b;
    const IDX li = is_a ? i : i - n_a;
    const int32_t r0 = static_cast<int32_t>(li & 31);
    const IDX qa = li >> 5;
    const IDX rb = qa / static_cast<IDX>(groups);
    const int32_t g = static_cast<int32_t>(qa - rb * static_cast<IDX>(groups));
    const int64_t row0 = static_cast<int64_t>(rb) * 128 + r0;
    uint32_t w[4];
    // K-contiguous scales with 4-byte aligned rows: one 32-bit load per row
    // (the four scales of a group are adjacent); otherwise byte loads
    const bool words = t.s1 == 1 && (t.s0 & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(t.src) & 3u) == 0 && g * 4 + 3 < kscales;
    if (words) {
#pragma unroll
      for (int r1 = 0; r1 < 4; ++r1) {
        const int64_t row = row0 + r1 * 32;
        w[r1] = row < t.rows ? __ldg(reinterpret_cast<const uint32_t*>(t.src + row * t.s0 + g * 4))
                             : 0x7F7F7F7Fu;
      }
    } else {
      uint32_t v[4][4];
#pragma unroll
      for (int r1 = 0; r1 < 4; ++r1) {
        const int64_t row = row0 + r1 * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t k = g * 4 + j;
          v[r1][j] = (row < t.rows && k < kscales) ? __ldg(t.src + row * t.s0 + k * t.s1) : 127u;
        }
      }
#pragma unroll
      for (int r1 = 0; r1 < 4; ++r1)
        w[r1] = v[r1][0] | (v[r1][1] << 8) | (v[r1][2] << 16) | (v[r1][3] << 24);
    }
    *reinterpret_cast<uint4*>(t.dst + (static_cast<int64_t>(rb) * groups + g) * 512 + r0 * 16) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Scales with 16-byte aligned rows in either common storage: K-contiguous
// (s1 = 1) or M-contiguous (s0 = 1, the reference's storage). One CTA per
// (128-row block, 16 groups): the source tile (128 rows x 64 k-blocks) is read
// with coalesced 16-byte loads into shared memory, then each warp writes one
// 512-byte block. (A thread per output word loading straight from global
// memory touches a separate 32-byte sector for every 1 or 4 useful bytes.)
// K-contiguous: shared rows 17 words apart, so the 32 rows one output word
// gathers sit in 32 different banks. M-contiguous: 64 k-rows of 128 bytes,
// 144 bytes apart; an output word gathers one byte from each of 4 k-rows.
// Rows and k-blocks past the matrix read as 127 (scale 1.0).
constexpr int kRlGroups = 16;  // 4-scale groups per CTA (64 k-blocks)

__device__ __forceinline__ bool rl_kmajor(const RelayoutArgs& t) {
  return t.s1 == 1 && t.s0 % 16 == 0;
}

__global__ void __launch_bounds__(256) sf_relayout_tile_kernel(RelayoutArgs a, RelayoutArgs b,
                                                               int32_t kscales, int32_t groups) {
  grid_dependency_wait();
  grid_launch_dependents();
  __shared__ __align__(16) uint8_t sm[64 * 144];  // >= 128 rows x 17 words
  const int32_t gchunks = (groups + kRlGroups - 1) / kRlGroups;
  const int64_t blk = blockIdx.x;
  const int32_t rbi = static_cast<int32_t>(blk / gchunks);
  const int32_t gc = static_cast<int32_t>(blk - int64_t{rbi} * gchunks);
  const bool is_a = rbi < a.row_blocks;
  const RelayoutArgs& t = is_a ? a : b;
  const int32_t rb = is_a ? rbi : rbi - a.row_blocks;
  const int32_t k0 = gc * kRlGroups * 4;
  const int64_t row0 = int64_t{rb} * 128;
  auto byte_at = [&](int64_t row, int32_t k) -> uint32_t {
    return (row < t.rows && k < kscales) ? __ldg(t.src + row * t.s0 + int64_t{k} * t.s1) : 127u;
  };
  if (rl_kmajor(t)) {
    uint32_t* tile = reinterpret_cast<uint32_t*>(sm);
    for (int32_t pc = threadIdx.x; pc < 128 * 4; pc += blockDim.x) {
      const int32_t r = pc >> 2, k = k0 + 16 * (pc & 3);
      const int64_t row = row0 + r;
      uint32_t w[4];
      if (row < t.rows && k + 16 <= kscales) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(t.src + row * t.s0 + k));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = byte_at(row, k + 4 * i) | (byte_at(row, k + 4 * i + 1) << 8) |
                 (byte_at(row, k + 4 * i + 2) << 16) | (byte_at(row, k + 4 * i + 3) << 24);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) tile[r * 17 + 4 * (pc & 3) + i] = w[i];
    }
    __syncthreads();
    for (int32_t o = threadIdx.x; o < kRlGroups * 32; o += blockDim.x) {
      const int32_t gl = o >> 5, r0 = o & 31;  // one group per warp
      const int32_t g = gc * kRlGroups + gl;
      if (g >= groups) break;
      const uint4 v = make_uint4(tile[r0 * 17 + gl], tile[(32 + r0) * 17 + gl],
                                 tile[(64 + r0) * 17 + gl], tile[(96 + r0) * 17 + gl]);
      *reinterpret_cast<uint4*>(t.dst + (int64_t{rb} * groups + g) * 512 + r0 * 16) = v;
    }
  } else {
    for (int32_t pc = threadIdx.x; pc < 64 * 8; pc += blockDim.x) {
      const int32_t kr = pc >> 3, k = k0 + kr;
      const int64_t row = row0 + 16 * (pc & 7);
      uint4 v;
      if (k < kscales && row + 16 <= t.rows) {
        v = __ldg(reinterpret_cast<const uint4*>(t.src + row + int64_t{k} * t.s1));
      } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = byte_at(row + 4 * i, k) | (byte_at(row + 4 * i + 1, k) << 8) |
                 (byte_at(row + 4 * i + 2, k) << 16) | (byte_at(row + 4 * i + 3, k) << 24);
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
      *reinterpret_cast<uint4*>(sm + kr * 144 + 16 * (pc & 7)) = v;
    }
    __syncthreads();
    for (int32_t o = threadIdx.x; o < kRlGroups * 32; o += blockDim.x) {
      const int32_t gl = o >> 5, r0 = o & 31;
      const int32_t g = gc * kRlGroups + gl;
      if (g >= groups) break;
      const uint8_t* col = sm + 4 * gl * 144 + r0;
      uint32_t w[4];
#pragma unroll
      for (int r1 = 0; r1 < 4; ++r1)
        w[r1] = uint32_t{col[32 * r1]} | (uint32_t{col[144 + 32 * r1]} << 8) |
                (uint32_t{col[288 + 32 * r1]} << 16) | (uint32_t{col[432 + 32 * r1]} << 24);
      *reinterpret_cast<uint4*>(t.dst + (int64_t{rb} * groups + g) * 512 + r0 * 16) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Operands the tiled kernel takes: absent, or K- / M-contiguous with
// 16-byte aligned base and rows.
static bool tile_layout(const RelayoutArgs& t) {
  if (t.row_blocks == 0) return true;
  if ((reinterpret_cast<uintptr_t>(t.src) & 15u) != 0) return false;
  return (t.s1 == 1 && t.s0 % 16 == 0) || (t.s0 == 1 && t.s1 % 16 == 0);
}

// Enough CTAs to cover `work` items once (the block scheduler balances the
// waves); the kernels' grid-stride loops only matter past the grid limit.
static int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  if (blocks > (int64_t{1} << 30)) blocks = int64_t{1} << 30;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

cudaError_t launch_quant_mxfp4(const float* src, int64_t ld, int rows, int K, uint8_t* q,
                               int64_t ldq, uint8_t* sc, int64_t s0, int64_t s1,
                               cudaStream_t stream) {
  constexpr int kSegs = 2;
  const int64_t segs = static_cast<int64_t>(rows) * ((K / 32 + 7) / 8);
  const int grid = grid_for((segs + kSegs - 1) / kSegs * 32, 256);
  if (segs + int64_t{kSegs} * grid * 8 < (int64_t{1} << 31))
    quant_mxfp4_kernel<uint32_t, kSegs><<<grid, 256, 0, stream>>>(src, ld, rows, K, q, ldq, sc,
                                                                  s0, s1);
  else
    quant_mxfp4_kernel<int64_t, kSegs><<<grid, 256, 0, stream>>>(src, ld, rows, K, q, ldq, sc,
                                                                 s0, s1);
  return cudaGetLastError();
}

cudaError_t launch_quant_mxe5m2(const float* src, int64_t ld, int rows, int K,
                                const uint8_t* sc, int64_t s0, int64_t s1, uint8_t* q,
                                int64_t ldq, cudaStream_t stream) {
  constexpr int kUnroll = 2;
  const int64_t work = static_cast<int64_t>(rows) * (K / 8);
  const int grid = grid_for((work + kUnroll - 1) / kUnroll, 256);
  if (work + int64_t{kUnroll} * grid * 256 < (int64_t{1} << 31))
    quant_mxe5m2_kernel<uint32_t, kUnroll><<<grid, 256, 0, stream>>>(src, ld, rows, K, sc, s0,
                                                                     s1, q, ldq);
  else
    quant_mxe5m2_kernel<int64_t, kUnroll><<<grid, 256, 0, stream>>>(src, ld, rows, K, sc, s0,
                                                                    s1, q, ldq);
  return cudaGetLastError();
}

cudaError_t launch_cast_e5m2(const void* src, int dtype, int64_t n, uint8_t* dst,
                             cudaStream_t stream) {
  const size_t esz = dtype == 2 ? 4 : 2;
  if (n % 4 == 0 && reinterpret_cast<uintptr_t>(src) % (4 * esz) == 0 &&
      reinterpret_cast<uintptr_t>(dst) % 4 == 0) {
    constexpr int kUnroll = 4;
    const int64_t n4 = n / 4;
    const int g4 = grid_for((n4 + kUnroll - 1) / kUnroll, 256);
    uint32_t* d4 = reinterpret_cast<uint32_t*>(dst);
    if (dtype == 2)
      cast_e5m2_x4_kernel<float, kUnroll>
          <<<g4, 256, 0, stream>>>(static_cast<const float*>(src), n4, d4);
    else if (dtype == 0)
      cast_e5m2_x4_kernel<__half, kUnroll>
          <<<g4, 256, 0, stream>>>(static_cast<const __half*>(src), n4, d4);
    else
      cast_e5m2_x4_kernel<__nv_bfloat16, kUnroll>
          <<<g4, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), n4, d4);
    return cudaGetLastError();
  }
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
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = static_cast<int>(std::min<int64_t>(grid_for(work, 256), int64_t{sms} * 4));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (tile_layout(a) && tile_layout(b)) {
    const int64_t blocks = (static_cast<int64_t>(a.row_blocks) + b.row_blocks) *
                           ((groups + kRlGroups - 1) / kRlGroups);
    if (blocks < (int64_t{1} << 31)) {
      cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
      return cudaLaunchKernelEx(&cfg, sf_relayout_tile_kernel, a, b, kscales, groups);
    }
  }
  const cudaError_t e = work < (int64_t{1} << 31)
                            ? cudaLaunchKernelEx(&cfg, sf_relayout_kernel<uint32_t>, a, b, kscales, groups)
                            : cudaLaunchKernelEx(&cfg, sf_relayout_kernel<int64_t>, a, b, kscales, groups);
  return e;
}

}  // namespace b2g
