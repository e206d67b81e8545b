// Memory-bound C = A * B^T for a few rows of A (M <= 128), the shape of a
// decode step against a weight matrix B; the reference lists this
// "memory-bound GEMM" as the next item after its compute-bound kernels
// (README.md:84). The time floor is reading B (N x K) once from HBM.
//
// Swap-AB: tcgen05.mma's 128-row M side takes 128 rows of B (128 columns of
// C) and its N side the BN rows of A (BN = 16, 32, 64 or 128, the smallest
// that holds M), so the tensor core computes C^T tiles of 128 x BN with no
// padding of M up to a full tile. Per 128-byte K chunk the MMA work is a
// few dozen cycles against ~16 KB of B to stream, so the kernel is bound by
// HBM as long as enough CTAs stream B at once.
//
// Each CTA takes one (128-column tile of C, K split) item; the grid is about
// one wave of such items (more when C has more tiles than the GPU has SMs).
// Several K splits of a tile add their fp32 partial tiles through the
// workspace: every split stores its partial, counts itself in the tile's
// arrival counter, and the split that arrives last sums the partials in
// split order (so the result does not depend on arrival order) and writes C.
// No CTA ever waits for another one.
//
// CTA layout (192 threads): warp 0 one-thread TMA producer over a ring of
// two-chunk stages, warp 1 one-thread MMA issuer (TMEM accumulator of BN
// columns), warps 2-5 epilogue (TMEM lanes 32*(w%4).. hold C columns, the BN
// accumulator columns hold C rows; each warp stores 32 consecutive C
// elements per row, 16 or 32 accumulator columns at a time).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "b2g.h"
#include "ptx.cuh"

namespace b2g {

struct alignas(64) SkinnyParams {
  CUtensorMap tmB;     // wide operand N x K (K-contiguous bytes), 128 x 128-byte boxes, 128B swizzle
  CUtensorMap tmA;     // the few rows M x K, BN x 128-byte boxes, 128B swizzle
  void* C;             // M x N row-major (fp16 or bf16), row stride ldc elements
  int64_t ldc;
  float* partials;     // [tiles][splits][128][BN] fp32 when splits > 1
  uint32_t* counters;  // [tiles] split arrivals; zero between calls
  int* status;
  int32_t M, N, k_chunks, splits, chunks_per_split;
  uint64_t timeout_ns;
};

template <int BN>
struct SkinnyPlan {
  static constexpr uint32_t kThreads = 192;
  static constexpr uint32_t kChunks = 2;         // 128-byte K chunks per stage
  static constexpr uint32_t kChunkB = 128 * 128; // 128 rows of B x 128 bytes of K
  static constexpr uint32_t kChunkA = BN * 128;  // BN rows of A (a multiple of 1024 bytes)
  static constexpr uint32_t kStage = kChunks * (kChunkB + kChunkA);
  static constexpr uint32_t kStages = (196608u / kStage) < 6u ? (196608u / kStage) : 6u;
  static constexpr uint32_t kBOff = 0;
  static constexpr uint32_t kAOff = kStages * kChunks * kChunkB;
  static constexpr uint32_t kBarOff = kAOff + kStages * kChunks * kChunkA;
  // full[S], empty[S], acc_full
  static constexpr uint32_t kMiscOff = kBarOff + (2 * kStages + 1) * 8;  // tmem slot, abort, last
  static constexpr uint32_t kBytes = kMiscOff + 16;
  static constexpr uint32_t kDynBytes = kBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "BN");
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(kDynBytes <= 232448, "shared memory");
};

template <int KIND, int BN>
__host__ __device__ constexpr uint32_t skinny_idesc() {
  // D fp32 | A fmt | B fmt | K-major both | N = BN | M = 128
  constexpr uint32_t f = KIND == 0 ? 0u : 1u;  // f16 0, bf16 1; f8f6f4: e5m2 1
  return (1u << 4) | (f << 7) | (f << 10) | ((static_cast<uint32_t>(BN) >> 3) << 17) |
         ((128u >> 4) << 24);
}

__device__ __forceinline__ void skinny_report(const SkinnyParams& p, int code) {
  if (p.status != nullptr) atomicCAS(p.status, 0, code);
}

// Bounded mbarrier wait (CTA scope): the deadline and the CTA's abort flag
// are checked between sleeping probes.
__device__ __noinline__ bool skinny_wait_slow(uint32_t bar, uint32_t parity,
                                              volatile uint32_t* abort_flag,
                                              const SkinnyParams& p, int site) {
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
    if (*abort_flag != 0u) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      skinny_report(p, B2G_STATUS_TIMEOUT | site);
      *abort_flag = 1u;
      return false;
    }
  }
}

__device__ __forceinline__ bool skinny_wait(uint32_t bar, uint32_t parity,
                                            volatile uint32_t* abort_flag, const SkinnyParams& p,
                                            int site) {
  if (mbar_try_wait(bar, parity)) return true;
  return skinny_wait_slow(bar, parity, abort_flag, p, site);
}

template <bool kBF16>
__device__ __forceinline__ uint16_t skinny_cvt(float v) {
  if constexpr (kBF16) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<const uint16_t*>(&h);
  } else {
    const __half h = __float2half_rn(v);
    return *reinterpret_cast<const uint16_t*>(&h);
  }
}

__device__ __forceinline__ void epilogue_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");  // warps 2-5 only
}

template <int KIND, int BN, bool OUT_BF16>
__global__ void __launch_bounds__(192, 1) skinny_kernel(const __grid_constant__ SkinnyParams p) {
  using SP = SkinnyPlan<BN>;
  constexpr uint32_t S = SP::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t tile = static_cast<int32_t>(blockIdx.x) / p.splits;
  const int32_t split = static_cast<int32_t>(blockIdx.x) - tile * p.splits;
  const int32_t c0 = split * p.chunks_per_split;
  const int32_t c1 = min(p.k_chunks, c0 + p.chunks_per_split);
  const int32_t n_stages = (c1 - c0 + 1) / 2;  // the last stage may hold one chunk

  const uint32_t bar0 = sbase + SP::kBarOff;
  auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
  auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (S + s); };
  const uint32_t accf_bar = bar0 + 8u * (2 * S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SP::kMiscOff);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + SP::kMiscOff + 4);
  volatile uint32_t* last_flag = reinterpret_cast<volatile uint32_t*>(smem + SP::kMiscOff + 8);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accf_bar, 1);
    *abort_flag = 0u;
    *last_flag = 0u;
    fence_mbarrier_init();
    prefetch_tensormap(&p.tmA);
    prefetch_tensormap(&p.tmB);
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(tmem_slot), SP::kTmemCols);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int32_t st = 0;
      for (; st < n_stages; ++st) {
        const uint32_t s = static_cast<uint32_t>(st) % S, ph = (static_cast<uint32_t>(st) / S) & 1u;
        if (!skinny_wait(empty_bar(s), ph ^ 1u, abort_flag, p, B2G_SITE_EMPTY)) break;
        const int32_t kc0 = c0 + 2 * st;
        const int32_t nc = min(2, c1 - kc0);
        mbar_arrive_expect_tx(full_bar(s), static_cast<uint32_t>(nc) * (SP::kChunkB + SP::kChunkA));
        for (int32_t c = 0; c < nc; ++c) {
          const uint32_t slot = s * 2 + static_cast<uint32_t>(c);
          tma_load_2d(sbase + SP::kBOff + slot * SP::kChunkB, &p.tmB, full_bar(s),
                      (kc0 + c) * 128, tile * 128);
          tma_load_2d(sbase + SP::kAOff + slot * SP::kChunkA, &p.tmA, full_bar(s),
                      (kc0 + c) * 128, 0);
        }
      }
      // every load issued lands before the CTA can exit
      for (int32_t i = st > static_cast<int32_t>(S) ? st - static_cast<int32_t>(S) : 0; i < st; ++i) {
        uint32_t spins = 0;
        while (!mbar_try_wait(full_bar(static_cast<uint32_t>(i) % S), (static_cast<uint32_t>(i) / S) & 1u) &&
               spins < (1u << 20))
          ++spins;
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    if (lane == 0) {
      constexpr uint32_t idesc = skinny_idesc<KIND, BN>();
      for (int32_t st = 0; st < n_stages; ++st) {
        const uint32_t s = static_cast<uint32_t>(st) % S, ph = (static_cast<uint32_t>(st) / S) & 1u;
        if (!skinny_wait(full_bar(s), ph, abort_flag, p, B2G_SITE_FULL)) break;
        tc_fence_after();
        const int32_t nc = min(2, c1 - (c0 + 2 * st));
#pragma unroll
        for (int32_t c = 0; c < 2; ++c) {
          if (c >= nc) break;
          const uint32_t slot = s * 2 + static_cast<uint32_t>(c);
          const uint64_t bdesc = sdesc_kmajor_sw128(sbase + SP::kBOff + slot * SP::kChunkB);
          const uint64_t adesc = sdesc_kmajor_sw128(sbase + SP::kAOff + slot * SP::kChunkA);
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            // B rows are the MMA's M side, A rows its N side; +32 bytes of K per MMA
            const uint32_t acc = (st > 0 || c > 0 || j > 0) ? 1u : 0u;
            if constexpr (KIND == 2)
              mma_f8f6f4<1>(tmem_base, bdesc + 2u * j, adesc + 2u * j, idesc, acc);
            else
              mma_f16<1>(tmem_base, bdesc + 2u * j, adesc + 2u * j, idesc, acc);
          }
        }
        tc_commit<1>(empty_bar(s));
      }
      // the accumulator is complete (or the CTA aborted) once every MMA issued is done
      tc_commit<1>(accf_bar);
      uint32_t spins = 0;
      while (!mbar_try_wait(accf_bar, 0) && spins < (1u << 22)) ++spins;
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const uint32_t quad = warp & 3u;
    const int32_t row = static_cast<int32_t>(quad * 32u + lane);  // row of the C^T tile
    const int32_t n = tile * 128 + row;                             // column of C
    const bool ok = __all_sync(0xffffffffu, skinny_wait(accf_bar, 0, abort_flag, p, B2G_SITE_ACC_FULL));
    // `has`: this warp's accumulator rows are complete. Warps decide it on
    // their own, so it gates only data movement; every epilogue warp passes
    // both named barriers below whatever it decided.
    const bool has = ok && n_stages > 0 && *abort_flag == 0u;
    constexpr int kPiece = BN < 32 ? BN : 32;  // accumulator columns per TMEM load
    constexpr int kPieces = BN / kPiece;
    const uint32_t taddr = tmem_base + ((quad * 32u) << 16);
    uint16_t* crow = static_cast<uint16_t*>(p.C) + n;  // C[m][n] = crow[m * ldc]
    const bool n_ok = n < p.N;
    auto store_c = [&](const float (&v)[kPiece], int m0) {
      if (!n_ok) return;
#pragma unroll
      for (int m = 0; m < kPiece; ++m)
        if (m0 + m < p.M) crow[static_cast<int64_t>(m0 + m) * p.ldc] = skinny_cvt<OUT_BF16>(v[m]);
    };
    auto load_piece = [&](int q, float (&v)[kPiece]) {
      if constexpr (kPiece == 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(q) * 16u, r);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 16; ++m) v[m] = __uint_as_float(r[m]);
      } else {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(q) * 32u, r);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 32; ++m) v[m] = __uint_as_float(r[m]);
      }
    };
    if (has) tc_fence_after();
    if (p.splits == 1) {
      if (has) {
        for (int q = 0; q < kPieces; ++q) {
          float v[kPiece];
          load_piece(q, v);
          store_c(v, q * kPiece);
        }
      }
    } else {
      // partial tile rows of this split, then the split that arrives last sums
      // all splits in split order. `has` is decided per warp, so it gates data
      // movement only: every epilogue warp passes both named barriers.
      const size_t tile_base = static_cast<size_t>(tile) * p.splits * 128u * BN;
      if (has) {
        float* mine = p.partials + tile_base + static_cast<size_t>(split) * 128u * BN +
                      static_cast<size_t>(row) * BN;
        for (int q = 0; q < kPieces; ++q) {
          float v[kPiece];
          load_piece(q, v);
#pragma unroll
          for (int m = 0; m < kPiece; m += 4)
            __stcg(reinterpret_cast<float4*>(mine + q * kPiece + m),
                   make_float4(v[m], v[m + 1], v[m + 2], v[m + 3]));
        }
      }
      __threadfence();
      epilogue_bar_sync();
      if (warp == 2 && lane == 0) {
        const uint32_t before = atomicAdd(p.counters + tile, 1u);
        const bool last = before == static_cast<uint32_t>(p.splits - 1);
        if (last) p.counters[tile] = 0u;  // every split has arrived: ready for the next call
        *last_flag = last ? 1u : 0u;
      }
      epilogue_bar_sync();
      if (has && *last_flag != 0u) {
        __threadfence();
        const float* base = p.partials + tile_base + static_cast<size_t>(row) * BN;
        for (int q = 0; q < kPieces; ++q) {
          float v[kPiece];
#pragma unroll
          for (int m = 0; m < kPiece; ++m) v[m] = 0.0f;
          for (int32_t sp = 0; sp < p.splits; ++sp) {
            const float* src = base + static_cast<size_t>(sp) * 128u * BN + q * kPiece;
#pragma unroll
            for (int m = 0; m < kPiece; m += 4) {
              const float4 t = __ldcg(reinterpret_cast<const float4*>(src + m));
              v[m] += t.x;
              v[m + 1] += t.y;
              v[m + 2] += t.z;
              v[m + 3] += t.w;
            }
          }
          store_c(v, q * kPiece);
        }
      }
    }
  }

  // ------------------------------------------------------------- teardown --
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, SP::kTmemCols);
  }
}

}  // namespace b2g
