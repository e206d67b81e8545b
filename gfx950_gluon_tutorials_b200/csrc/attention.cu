// Flash-attention forward (non-causal, GQA) for sm_100a: O = softmax(Q K^T * s) V
// and the row log-sum-exp, the reference's FMHA forward
// (kernels/attention/fmha_v4.py:343-758, launcher :761-790; torch oracle
// kernels/attention/common.py:115-138 sdpa_reference).
//
// Persistent: one CTA per SM loops over work items (256 query rows = two
// 128-row tiles, query head, batch). Per tile t and KV tile j of 128 keys:
//   S_t  = Q_t K_j^T          tcgen05.mma into tile t's TMEM score buffer
//   P_t  = exp2(S_t*s' - m)   softmax warpgroup t, one query row per thread; P is
//                             stored back to TMEM as 16-bit values over S_t's
//                             columns (the first half with the two-pass softmax,
//                             the upper half with the one-pass variant)
//   O_t += P_t V_j            tcgen05.mma with A = P read from TMEM and B = V as an
//                             MN-major shared-memory operand (no transpose pass)
// The MMA thread interleaves the tiles (PV_0, S_0 next, PV_1, S_1 next, ...) so
// one tile's softmax runs while the tensor pipe works on the other tile. The
// exponent offset m is kept in log2 units (s' = sm_scale * log2 e) and moves
// only when a row max grows by more than 2^8; O rows are then rescaled in TMEM
// before the next PV accumulates.
//
// CTA layout (320 threads): warp 0 one-thread TMA producer (Q once; K and V
// through two-stage rings), warp 1 one-thread MMA issuer (owns the 512 TMEM
// columns), warps 2-5 and 6-9 the softmax and epilogue of tiles 0 and 1. Q, K,
// V and O are addressed through 4-D views (d, sequence, head, batch) built
// from the caller's strides, so bhsd and bshd layouts and GQA (query head h
// reads key/value head h / (HQ / HK)) need no copies; keys and query rows
// past the sequence ends are zero-filled by TMA and masked.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "b2g.h"
#include "capi_internal.h"
#include "ptx.cuh"

// Exponential pairs per four computed by poly_exp2 on the FMA pipe instead of
// the MUFU unit (0..4).
#ifndef B2G_FMHA_POLY_PAIRS
#define B2G_FMHA_POLY_PAIRS 0
#endif

// Suspend-time hint of the slow path of the bounded waits (0: plain probes,
// which hand over between the roles a little sooner).
#ifndef B2G_FMHA_WAIT_HINT_NS
#define B2G_FMHA_WAIT_HINT_NS 0
#endif

namespace b2g {

struct alignas(64) FmhaParams {
  CUtensorMap tmQ, tmK, tmV;  // 4-D (d, seq, head, batch), 64 x 128 x 1 x 1 boxes, 128B swizzle
  void* O;                    // output, same element type as Q
  int64_t o_sb, o_sh, o_ss;   // element strides of O (d contiguous)
  float* lse;                 // [B][HQ][S_q] natural-log log-sum-exp, or null
  int* status;
  int32_t B, HQ, HK, S_q, S_k;
  float scale_log2;           // sm_scale * log2(e)
  uint64_t timeout_ns;
};

// Shared memory and TMEM plan of one CTA: two 128-row query tiles (Q0, Q1),
// K and V rings, and per tile one score buffer (P aliases half of it once
// the scores are in registers) and one O accumulator.
template <int D>
struct FmhaPlan {
  static constexpr uint32_t kSoftmaxWarps = 8;                  // two warpgroups, one per tile
  static constexpr uint32_t kThreads = 64 + 32 * kSoftmaxWarps;  // + producer and MMA warps
  static constexpr uint32_t kRegions = D / 64;             // 64-element (128-byte) column slabs
  static constexpr uint32_t kRegion = 128 * 128;           // 128 rows x 128 bytes
  static constexpr uint32_t kTile = kRegions * kRegion;    // one Q, K or V tile
  static constexpr uint32_t kStages = 2;                   // K ring and V ring depth
  static constexpr uint32_t kQOff = 0;                     // Q0, Q1
  static constexpr uint32_t kKOff = kQOff + 2 * kTile;
  static constexpr uint32_t kVOff = kKOff + kStages * kTile;
  static constexpr uint32_t kBarOff = kVOff + kStages * kTile;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2][2]
  // (tile, key half), o_done[2], q_empty, o_free[2]
  static constexpr uint32_t kNumBars = 1 + 4 * kStages + 11;
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr uint32_t kBytes = kMiscOff + 16;
  static constexpr uint32_t kDynBytes = kBytes + 1024;  // + alignment slack
  // TMEM columns: S_t = 128 t (128 fp32), P_t = S_t + 64 (128 x 16-bit),
  // O_t = 256 + 128 t (D fp32)
  // P from column 0: each 16-column P chunk lands on scores already reloaded
  static constexpr uint32_t kS = 0, kP = 0, kO = 256, kTileCols = 128;
  static_assert(D == 64 || D == 128, "head dim");
  static_assert(kDynBytes <= 232448, "shared memory");
};

// exp2 on the FMA pipe for x <= 8 (a share of the softmax exponentials, so that
// they do not all queue on the MUFU unit): x = i + f with i = round(x) and
// f in [-0.5, 0.5]; 2^f from a cubic fitted here to minimise the relative error
// on that interval (iteratively reweighted least squares; max relative error
// 7.5e-5 in fp32 for x in [-125.5, 8], below half an fp16 ULP); 2^i added to
// the exponent field. Inputs below -126 (masked keys are -inf) are clamped
// there: with 2^f in [0.70, 1.42] the biased exponent 126 or 127 plus
// i >= -126 stays >= 0, so the result is a tiny non-negative number, never a
// carry into the sign bit (at the clamp the exponent field reaches 0, so the
// result is the subnormal 0.99986 * 2^-126 rather than 0.99993 * 2^-126).
// b2g_selftest_poly_exp2 evaluates it on caller data for the tests.
__device__ __forceinline__ float poly_exp2(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
  x = fmaxf(x, -126.0f);
  const float t = x + kRound;
  const float fi = t - kRound;
  const float f = x - fi;
  float p = fmaf(0.05517134442925453f, f, 0.24261033535003662f);
  p = fmaf(p, f, 0.6932609677314758f);
  p = fmaf(p, f, 0.9999281167984009f);
  const int32_t i = static_cast<int32_t>(__float_as_uint(t) - __float_as_uint(kRound));
  return __uint_as_float(static_cast<uint32_t>(static_cast<int32_t>(__float_as_uint(p)) + (i << 23)));
}

// poly_exp2 on a pair, with the packed (two-lane) fp32 add and FMA: per pair
// two clamps, five packed operations and two integer adds.
__device__ __forceinline__ float2 poly_exp2x2(float2 x) {
  constexpr float kRound = 12582912.0f;
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 fi = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(fi, make_float2(-1.0f, -1.0f), x);
  float2 q = __ffma2_rn(make_float2(0.05517134442925453f, 0.05517134442925453f), f,
                        make_float2(0.24261033535003662f, 0.24261033535003662f));
  q = __ffma2_rn(q, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = __ffma2_rn(q, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
  // t's bit pattern is that of 1.5 * 2^23 plus round(x), and the former ends in
  // nine zero bits: shifted left by 23 it leaves round(x) * 2^23, the exponent step
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

// After tcgen05.wait::ld: ties these registers to this point, so that no use
// of a value loaded asynchronously is scheduled before the wait (no code).
__device__ __forceinline__ void regs_ready(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

template <int D, bool kBF16>
__host__ __device__ constexpr uint32_t fmha_idesc_s() {
  // D fp32 | A, B fmt | both K-major | N = 128 keys | M = 128 rows
  constexpr uint32_t f = kBF16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

template <int D, bool kBF16>
__host__ __device__ constexpr uint32_t fmha_idesc_pv() {
  // D fp32 | A, B fmt | A K-major (TMEM), B MN-major (V, d contiguous) | N = D | M = 128
  constexpr uint32_t f = kBF16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | (1u << 16) | ((static_cast<uint32_t>(D) >> 3) << 17) |
         ((128u >> 4) << 24);
}

__device__ __forceinline__ void fmha_report(const FmhaParams& p, int code) {
  if (p.status != nullptr) atomicCAS(p.status, 0, code);
}

// Bounded mbarrier wait: sleeping probes, then the deadline and the CTA's
// abort flag between them.
template <bool kClusterScope = false>
__device__ __noinline__ bool fmha_wait_slow(uint32_t bar, uint32_t parity,
                                            volatile uint32_t* abort_flag, const FmhaParams& p,
                                            int site) {
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
#if B2G_FMHA_WAIT_HINT_NS > 0
    if (mbar_try_wait_sleep(bar, parity, B2G_FMHA_WAIT_HINT_NS)) return true;
#else
    if (mbar_try_wait(bar, parity)) return true;
#endif
    if (*abort_flag != 0u) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      fmha_report(p, B2G_STATUS_TIMEOUT | site);
      *abort_flag = 1u;
      return false;
    }
  }
}

__device__ __forceinline__ bool fmha_wait(uint32_t bar, uint32_t parity,
                                          volatile uint32_t* abort_flag, const FmhaParams& p,
                                          int site) {
  if (mbar_try_wait(bar, parity)) return true;
  return fmha_wait_slow(bar, parity, abort_flag, p, site);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <int D, bool kBF16>
__global__ void __launch_bounds__(FmhaPlan<D>::kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ FmhaParams p) {
  using FP = FmhaPlan<D>;
  constexpr uint32_t KS = FP::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t n_kv = (p.S_k + 127) / 128;
  // Persistent: work items are (256-row query block, query head, batch), the
  // query block fastest, so the CTAs working at one time share K and V in L2.
  const int32_t n_mblk = (p.S_q + 255) / 256;
  const int32_t n_items = n_mblk * p.HQ * p.B;
  struct Item {
    int32_t m0, h, b, hk;
    uint32_t tiles;  // query tiles holding rows (1 or 2)
  };
  auto item_at = [&](int32_t it) {
    Item w;
    w.m0 = (it % n_mblk) * 256;
    w.h = (it / n_mblk) % p.HQ;
    w.b = it / (n_mblk * p.HQ);
    w.hk = w.h / (p.HQ / p.HK);
    w.tiles = p.S_q - w.m0 > 128 ? 2u : 1u;
    return w;
  };

  const uint32_t bar0 = sbase + FP::kBarOff;
  const uint32_t q_full = bar0;
  auto k_full = [&](uint32_t s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](uint32_t s) { return bar0 + 8u * (1 + KS + s); };
  auto v_full = [&](uint32_t s) { return bar0 + 8u * (1 + 2 * KS + s); };
  auto v_empty = [&](uint32_t s) { return bar0 + 8u * (1 + 3 * KS + s); };
  auto s_full = [&](uint32_t t) { return bar0 + 8u * (1 + 4 * KS + t); };
  auto p_full = [&](uint32_t t, uint32_t half) { return bar0 + 8u * (3 + 4 * KS + 2 * t + half); };
  auto o_done = [&](uint32_t t) { return bar0 + 8u * (7 + 4 * KS + t); };
  // q_empty: the item's last S MMAs are done with Q; o_free(t): the epilogue
  // has read tile t's O, so the next item's first PV may overwrite it
  const uint32_t q_empty = bar0 + 8u * (9 + 4 * KS);
  auto o_free = [&](uint32_t t) { return bar0 + 8u * (10 + 4 * KS + t); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FP::kMiscOff);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + FP::kMiscOff + 4);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (uint32_t s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (uint32_t t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t, 0), 4);  // one arrival per softmax warp of the tile
      mbar_init(p_full(t, 1), 4);
      mbar_init(o_done(t), 1);
      mbar_init(o_free(t), 4);
    }
    *abort_flag = 0u;
    fence_mbarrier_init();
    prefetch_tensormap(&p.tmQ);
    prefetch_tensormap(&p.tmK);
    prefetch_tensormap(&p.tmV);
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(tmem_slot), 512);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    // Q once per item (after the previous item's last S is done with it); K
    // and V through the rings, whose step count runs on across items.
    if (lane == 0) {
      uint32_t jg = 0, ic = 0;  // K/V steps and items issued
      uint32_t nk = 0, nv = 0;  // K and V loads issued
      bool alive = true;
      for (int32_t item = static_cast<int32_t>(blockIdx.x); alive && item < n_items;
           item += static_cast<int32_t>(gridDim.x), ++ic) {
        const Item w = item_at(item);
        if (ic > 0 && !fmha_wait(q_empty, (ic - 1u) & 1u, abort_flag, p, B2G_SITE_EMPTY)) break;
        mbar_arrive_expect_tx(q_full, w.tiles * FP::kTile);
        for (uint32_t t = 0; t < w.tiles; ++t)
          for (uint32_t r = 0; r < FP::kRegions; ++r)
            tma_load_4d(sbase + FP::kQOff + t * FP::kTile + r * FP::kRegion, &p.tmQ, q_full,
                        r * 64, w.m0 + static_cast<int32_t>(t) * 128, w.h, w.b);
        for (int32_t j = 0; j < n_kv; ++j, ++jg) {
          const uint32_t s = jg % KS, ph = (jg / KS) & 1u;
          if (!fmha_wait(k_empty(s), ph ^ 1u, abort_flag, p, B2G_SITE_EMPTY)) {
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(k_full(s), FP::kTile);
          for (uint32_t r = 0; r < FP::kRegions; ++r)
            tma_load_4d(sbase + FP::kKOff + s * FP::kTile + r * FP::kRegion, &p.tmK, k_full(s),
                        r * 64, j * 128, w.hk, w.b);
          ++nk;
          if (!fmha_wait(v_empty(s), ph ^ 1u, abort_flag, p, B2G_SITE_EMPTY)) {
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(v_full(s), FP::kTile);
          for (uint32_t r = 0; r < FP::kRegions; ++r)
            tma_load_4d(sbase + FP::kVOff + s * FP::kTile + r * FP::kRegion, &p.tmV, v_full(s),
                        r * 64, j * 128, w.hk, w.b);
          ++nv;
        }
      }
      // every load issued lands before the CTA can exit: the last Q and the
      // K and V loads of the last KS steps (older ones were consumed)
      uint32_t spins = 0;
      if (ic > 0)
        while (!mbar_try_wait(q_full, (ic - 1u) & 1u) && spins < (1u << 20)) ++spins;
      for (uint32_t i = nk > KS ? nk - KS : 0u; i < nk; ++i) {
        spins = 0;
        while (!mbar_try_wait(k_full(i % KS), (i / KS) & 1u) && spins < (1u << 20)) ++spins;
      }
      for (uint32_t i = nv > KS ? nv - KS : 0u; i < nv; ++i) {
        spins = 0;
        while (!mbar_try_wait(v_full(i % KS), (i / KS) & 1u) && spins < (1u << 20)) ++spins;
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    // Per tile the order is S_0, PV_0, S_1, PV_1, ...: P_j lives in S's
    // columns, and the tensor pipe runs one thread's MMAs in issue order, so
    // S_{j+1} is issued only after PV_j. The two tiles interleave: while one
    // tile's softmax runs, the other tile's PV and next S keep the pipe busy.
    // Across items, the next item's first S and softmax overlap this item's
    // epilogue; only its first PV waits for the O columns to be read out.
    if (lane == 0) {
      constexpr uint32_t idesc_s = fmha_idesc_s<D, kBF16>();
      constexpr uint32_t idesc_pv = fmha_idesc_pv<D, kBF16>();
      uint32_t last_bar = 0, last_par = 0;  // the newest commit: all earlier MMAs precede it
      auto issue_s = [&](uint32_t t, uint32_t kslot) {
        const uint32_t k_base = sbase + FP::kKOff + kslot * FP::kTile;
        const uint32_t q_base = sbase + FP::kQOff + t * FP::kTile;
#pragma unroll
        for (uint32_t kk = 0; kk < D / 16; ++kk) {
          // 16 head-dim elements per MMA: slab kk / 4, +32 bytes inside the swizzled row
          const uint64_t ad = sdesc_kmajor_sw128(q_base + (kk >> 2) * FP::kRegion) + 2u * (kk & 3u);
          const uint64_t bd = sdesc_kmajor_sw128(k_base + (kk >> 2) * FP::kRegion) + 2u * (kk & 3u);
          mma_f16<1>(tmem_base + FP::kS + t * FP::kTileCols, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      uint32_t jg = 0, ic = 0;             // K/V steps and items
      uint32_t steps[2] = {0u, 0u};        // steps of each tile (phases of s_full, p_full)
      uint32_t titems[2] = {0u, 0u};       // items of each tile (phases of o_done, o_free)
      bool alive = true;
      for (int32_t item = static_cast<int32_t>(blockIdx.x); alive && item < n_items;
           item += static_cast<int32_t>(gridDim.x), ++ic) {
        const Item w = item_at(item);
        const uint32_t nt = w.tiles;
        if (!fmha_wait(q_full, ic & 1u, abort_flag, p, B2G_SITE_FULL) ||
            !fmha_wait(k_full(jg % KS), (jg / KS) & 1u, abort_flag, p, B2G_SITE_FULL))
          break;
        tc_fence_after();
        for (uint32_t t = 0; t < nt; ++t) {
          issue_s(t, jg % KS);
          tc_commit<1>(s_full(t));
        }
        last_bar = s_full(0);
        last_par = steps[0] & 1u;
        if (n_kv == 1) tc_commit<1>(q_empty);  // the item's last S MMAs are issued
        tc_commit<1>(k_empty(jg % KS));
        for (int32_t j = 0; j < n_kv; ++j, ++jg) {
          const uint32_t s = jg % KS, ph = (jg / KS) & 1u;
          const bool has_next = j + 1 < n_kv;
          const uint32_t s1 = (jg + 1) % KS, ph1 = ((jg + 1) / KS) & 1u;
          if (!fmha_wait(v_full(s), ph, abort_flag, p, B2G_SITE_FULL)) {
            alive = false;
            break;
          }
          const uint32_t v_base = sbase + FP::kVOff + s * FP::kTile;
          for (uint32_t t = 0; alive && t < nt; ++t) {
            const uint32_t p_col = tmem_base + FP::kS + t * FP::kTileCols + FP::kP;
            // the previous item's epilogue must have read this tile's O
            if (j == 0 && titems[t] > 0 &&
                !fmha_wait(o_free(t), (titems[t] - 1u) & 1u, abort_flag, p, B2G_SITE_ACC_EMPTY)) {
              alive = false;
              break;
            }
            // P arrives in two 64-key halves; the first half's MMAs run while
            // the softmax still computes the second
            for (uint32_t half = 0; half < 2; ++half) {
              if (!fmha_wait(p_full(t, half), steps[t] & 1u, abort_flag, p, B2G_SITE_ACC_FULL)) {
                alive = false;
                break;
              }
              tc_fence_after();
#pragma unroll
              for (uint32_t k4 = 0; k4 < 4; ++k4) {
                // 16 keys per MMA: two 8-row swizzle atoms; head-dim slabs are kRegion apart
                const uint32_t kk = half * 4u + k4;
                const uint64_t bd = sdesc_mnmajor_sw128(v_base + kk * 2048u, FP::kRegion, 1024u);
                mma_f16_ts(tmem_base + FP::kO + t * FP::kTileCols, p_col + kk * 8u, bd, idesc_pv,
                           (j > 0 || kk > 0) ? 1u : 0u);
              }
            }
            if (!alive) break;
            ++steps[t];
            if (!has_next) {
              tc_commit<1>(o_done(t));
              last_bar = o_done(t);
              last_par = titems[t] & 1u;
              ++titems[t];
              continue;
            }
            if (t == 0 && !fmha_wait(k_full(s1), ph1, abort_flag, p, B2G_SITE_FULL)) {
              alive = false;
              break;
            }
            tc_fence_after();
            issue_s(t, s1);
            tc_commit<1>(s_full(t));
            last_bar = s_full(t);
            last_par = steps[t] & 1u;
          }
          if (!alive) break;
          if (j + 2 == n_kv) tc_commit<1>(q_empty);  // the item's last S MMAs are issued
          tc_commit<1>(v_empty(s));
          if (has_next) tc_commit<1>(k_empty(s1));
        }
      }
      // all MMAs issued by this thread finish before TMEM can be freed
      if (last_bar != 0u) {
        uint32_t spins = 0;
        while (!mbar_try_wait(last_bar, last_par) && spins < (1u << 22)) ++spins;
      }
    }
  } else {
    // --------------------------------------------- softmax and epilogue --
    // Warpgroup t (warps 2 + 4t .. 5 + 4t) owns query tile t; thread i of warp w
    // owns row 32 * (w % 4) + i of it: the TMEM lane quarter a warp may touch
    // is fixed by its index in the warpgroup.
    const uint32_t t = (warp - 2u) >> 2;
    {
      const uint32_t quarter = warp & 3u;
      const uint32_t row = quarter * 32u + lane;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16);
      const uint32_t s_col = taddr + FP::kS + t * FP::kTileCols;
      const uint32_t p_col = s_col + FP::kP;
      const uint32_t o_col = taddr + FP::kO + t * FP::kTileCols;
      const float sl2 = p.scale_log2;
      uint32_t step = 0, ti = 0;  // this tile's steps and items (barrier phases)
      bool alive = true;
      for (int32_t item = static_cast<int32_t>(blockIdx.x); alive && item < n_items;
           item += static_cast<int32_t>(gridDim.x)) {
      const Item w = item_at(item);
      if (t >= w.tiles) continue;
      float m_run = -INFINITY;  // exponent offset, log2 units (a running max of s * sl2)
      float l_run = 0.0f;       // running sum of exp2(s * sl2 - m_run)
      for (int32_t j = 0; j < n_kv; ++j, ++step) {
        if (!__all_sync(0xffffffffu, fmha_wait(s_full(t), step & 1u,
                                               abort_flag, p, B2G_SITE_ACC_FULL))) {
          alive = false;
          break;
        }
        tc_fence_after();
        uint32_t s[128];
        {
          uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
          uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
          uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[64]);
          uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[96]);
          tmem_ld_32x32b_x32(s_col, s0);
          tmem_ld_32x32b_x32(s_col + 32u, s1);
          tmem_ld_32x32b_x32(s_col + 64u, s2);
          tmem_ld_32x32b_x32(s_col + 96u, s3);
          tmem_wait_ld();
        }
        // keys past S_k (zero-filled by TMA) take no part
        const int32_t valid = p.S_k - j * 128;
        if (valid < 128) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= valid) s[c] = __float_as_uint(-INFINITY);
        }
        // row max: eight independent chains of three-input maxima
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(__uint_as_float(s[i]), __uint_as_float(s[i + 8]));
#pragma unroll
        for (int c = 16; c < 128; c += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            m8[i] = fmax3(m8[i], __uint_as_float(s[c + i]), __uint_as_float(s[c + 8 + i]));
        const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                               fmaxf(m8[6], m8[7]));
        // The exponent offset moves only when the row max grows by more than
        // 2^kRescaleLog2 over it: P stays below 2^kRescaleLog2, the final 1/l
        // cancels the offset exactly, and most tiles skip the O rescale.
        constexpr float kRescaleLog2 = 8.0f;
        const float m_cand = mx * sl2;
        const bool move = m_cand > m_run + kRescaleLog2;
        const float m_new = move ? m_cand : m_run;
        // on the FMA pipe: the other tile may be holding the MUFU unit
        float alpha = 1.0f;
        if (move) alpha = poly_exp2(m_run - m_new);

        // O holds PV_0..PV_{j-1} (the S_j commit follows them); rows whose
        // offset moved are scaled by alpha before PV_j adds onto them
        if (j >= 1 && __any_sync(0xffffffffu, move)) {
#pragma unroll 1
          for (uint32_t c0 = 0; c0 < static_cast<uint32_t>(D); c0 += 16u) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(o_col + c0, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st_32x32b_x16(o_col + c0, o);
          }
        }

        const float2 sl2x2 = make_float2(sl2, sl2);
        const float2 negm = make_float2(-m_new, -m_new);
        // Exponentials, 32 columns at a time: chunks 0 and 1 straight from the
        // registers of the max pass, chunks 2 and 3 reloaded from TMEM (each load
        // in flight while the previous chunk is exponentiated), so that few
        // registers are live and many exponentials can be in flight. P chunk c
        // (16 columns) overwrites score columns 16c.., whose scores are in
        // registers already.
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        {
          uint32_t buf[2][32];
          tmem_ld_32x32b_x32(s_col + 64u, buf[0]);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c == 2) {
              tmem_wait_ld();
              regs_ready(buf[0]);
              tmem_ld_32x32b_x32(s_col + 96u, buf[1]);
            }
            if (c == 3) {
              tmem_wait_ld();
              regs_ready(buf[1]);
            }
            uint32_t cur[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) cur[i] = c < 2 ? s[32 * c + i] : buf[c - 2][i];
            if (c >= 2 && valid < 128) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (32 * c + i >= valid) cur[i] = __float_as_uint(-INFINITY);
            }
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(cur[2 * i]),
                                                      __uint_as_float(cur[2 * i + 1])),
                                          sl2x2, negm);
              float2 e;
              if ((i & 3) < B2G_FMHA_POLY_PAIRS) {
                e = poly_exp2x2(x);
              } else {
                e.x = fast_exp2(x.x);
                e.y = fast_exp2(x.y);
              }
              acc[i & 3] = __fadd2_rn(acc[i & 3], e);
              pk[i] = pack2<kBF16>(e.x, e.y);
            }
            tmem_st_32x32b_x16(p_col + 16u * static_cast<uint32_t>(c), pk);
            if (c == 1 || c == 3) {
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(p_full(t, static_cast<uint32_t>(c >> 1)));
            }
          }
        }
        const float2 a01 = __fadd2_rn(acc[0], acc[1]), a23 = __fadd2_rn(acc[2], acc[3]);
        const float2 a = __fadd2_rn(a01, a23);
        l_run = fmaf(l_run, alpha, a.x + a.y);
        m_run = m_new;
      }

      if (!alive) break;
      // epilogue: O into registers, the columns released to the next item's
      // first PV, then the scaled rows stored
      if (!__all_sync(0xffffffffu, fmha_wait(o_done(t), ti & 1u, abort_flag, p, B2G_SITE_ACC_FULL))) {
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t o[D];
#pragma unroll
      for (uint32_t c0 = 0; c0 < static_cast<uint32_t>(D); c0 += 32u)
        tmem_ld_32x32b_x32(o_col + c0, *reinterpret_cast<uint32_t(*)[32]>(&o[c0]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free(t));
      ++ti;
      const int32_t q_row = w.m0 + static_cast<int32_t>(t * 128u + row);
      if (q_row < p.S_q) {
        const float inv_l = 1.0f / l_run;
        using OutT = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
        OutT* orow = static_cast<OutT*>(p.O) + static_cast<int64_t>(w.b) * p.o_sb +
                     static_cast<int64_t>(w.h) * p.o_sh + static_cast<int64_t>(q_row) * p.o_ss;
        uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
          uint4 u;
          u.x = pack2<kBF16>(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l);
          u.y = pack2<kBF16>(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l);
          u.z = pack2<kBF16>(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l);
          u.w = pack2<kBF16>(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l);
          dst[v] = u;
        }
        if (p.lse != nullptr) {
          // natural-log log-sum-exp of the scaled scores of this row
          constexpr float kLn2 = 0.693147180559945309f;
          p.lse[(static_cast<int64_t>(w.b) * p.HQ + w.h) * p.S_q + q_row] =
              (m_run + __log2f(l_run)) * kLn2;
        }
      }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host --
namespace {

// 4-D view (d, sequence, head, batch) of one operand, 64 x 128 boxes.
bool encode_bshd_view(CUtensorMap* map, const void* base, int dtype, int D, int S, int H, int B,
                      const int64_t* st /* batch, head, seq, dim (elements) */) {
  auto enc = tma_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                              static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st[2]) * 2u,
                                 static_cast<cuuint64_t>(st[1]) * 2u,
                                 static_cast<cuuint64_t>(st[0]) * 2u};
  const cuuint32_t box[4] = {64, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dtype == B2G_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, t, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool kBF16>
int launch_fmha(const FmhaParams& prm, int batch, int heads_q, int seqlen_q, cudaStream_t stream) {
  using FP = FmhaPlan<D>;
  auto kern = fmha_fwd_kernel<D, kBF16>;
  // At least half the SM's shared memory, so that two CTAs never share an SM
  // (each holds all 512 TMEM columns).
  const uint32_t dyn = FP::kDynBytes > 120u * 1024u ? FP::kDynBytes : 120u * 1024u;
  static std::atomic<bool> attr_set[64];  // per instantiation and device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return B2G_ENODEVICE;
  }
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(dyn)) != cudaSuccess)
      return static_cast<int>(cudaGetLastError());
    attr_set[dev].store(true);
  }
  // persistent: one CTA per SM, looping over the (query block, head, batch) items
  const int64_t items = static_cast<int64_t>((seqlen_q + 255) / 256) * heads_q * batch;
  const int sms = current_device_sms();
  if (sms <= 0) return B2G_ENODEVICE;
  if (items > INT32_MAX) return B2G_ESHAPE;
  const dim3 grid(static_cast<unsigned>(items < sms ? items : sms), 1, 1);
  kern<<<grid, FP::kThreads, dyn, stream>>>(prm);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

}  // namespace

}  // namespace b2g

extern "C" int b2g_attention_fwd(const void* q, const void* k, const void* v, void* o,
                                 const int64_t* strides, int batch, int heads_q, int heads_k,
                                 int seqlen_q, int seqlen_k, int head_dim, int dtype,
                                 float sm_scale, float* lse, int* status, void* stream) {
  using namespace b2g;
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || strides == nullptr)
    return B2G_EINVAL;
  if (dtype != B2G_DT_F16 && dtype != B2G_DT_BF16) return B2G_EINVAL;
  if (!(sm_scale > 0.0f) || !std::isfinite(sm_scale)) return B2G_EINVAL;
  if (head_dim != 64 && head_dim != 128) return B2G_ESHAPE;
  if (batch < 1 || heads_q < 1 || heads_k < 1 || heads_q % heads_k != 0) return B2G_ESHAPE;
  if (batch > 65535 || heads_q > 65535 || seqlen_q < 0 || seqlen_k < 1) return B2G_ESHAPE;
  for (int t = 0; t < 4; ++t) {
    const int64_t* st = strides + 4 * t;
    if (st[3] != 1) return B2G_ESTRIDE;
    for (int i = 0; i < 3; ++i)
      if (st[i] <= 0) return B2G_ESTRIDE;
    // rows must not overlap within a head: the sequence stride covers the row
    if (st[2] < head_dim) return B2G_ESTRIDE;
    for (int i = 0; i < 3; ++i)
      if ((st[i] * 2) % 16 != 0) return B2G_EALIGN;
  }
  for (const void* ptr : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return B2G_EALIGN;
  if (reinterpret_cast<uintptr_t>(lse) % alignof(float) != 0) return B2G_EALIGN;
  if (current_device_sms() <= 0) return B2G_ENODEVICE;
  if (seqlen_q == 0) return B2G_OK;

  FmhaParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!encode_bshd_view(&prm.tmQ, q, dtype, head_dim, seqlen_q, heads_q, batch, strides) ||
      !encode_bshd_view(&prm.tmK, k, dtype, head_dim, seqlen_k, heads_k, batch, strides + 4) ||
      !encode_bshd_view(&prm.tmV, v, dtype, head_dim, seqlen_k, heads_k, batch, strides + 8))
    return B2G_ETENSORMAP;
  prm.O = o;
  prm.o_sb = strides[12];
  prm.o_sh = strides[13];
  prm.o_ss = strides[14];
  prm.lse = lse;
  prm.status = status;
  prm.B = batch;
  prm.HQ = heads_q;
  prm.HK = heads_k;
  prm.S_q = seqlen_q;
  prm.S_k = seqlen_k;
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  prm.timeout_ns = wait_timeout_ns();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == B2G_DT_BF16;
  if (head_dim == 128)
    return bf16 ? launch_fmha<128, true>(prm, batch, heads_q, seqlen_q, s)
                : launch_fmha<128, false>(prm, batch, heads_q, seqlen_q, s);
  return bf16 ? launch_fmha<64, true>(prm, batch, heads_q, seqlen_q, s)
              : launch_fmha<64, false>(prm, batch, heads_q, seqlen_q, s);
}

// Evaluates the FMHA's FMA-pipe exponential on caller data: y_scalar[i] =
// poly_exp2(x[i]), y_pair[i] = the paired form (elements 2j and 2j+1 of x go
// through one poly_exp2x2), y_exp2f[i] = exp2f(x[i]) for comparison.
__global__ void poly_exp2_probe_kernel(const float* __restrict__ x, float* __restrict__ y_scalar,
                                       float* __restrict__ y_pair, float* __restrict__ y_exp2f,
                                       int64_t n) {
  const int64_t pairs = (n + 1) / 2;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < pairs;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = 2 * j, i1 = 2 * j + 1;
    const float x0 = x[i0], x1 = i1 < n ? x[i1] : 0.0f;
    const float2 e = b2g::poly_exp2x2(make_float2(x0, x1));
    y_scalar[i0] = b2g::poly_exp2(x0);
    y_pair[i0] = e.x;
    y_exp2f[i0] = exp2f(x0);
    if (i1 < n) {
      y_scalar[i1] = b2g::poly_exp2(x1);
      y_pair[i1] = e.y;
      y_exp2f[i1] = exp2f(x1);
    }
  }
}

extern "C" int b2g_selftest_poly_exp2(const float* x, float* y_scalar, float* y_pair,
                                      float* y_exp2f, int64_t n, void* stream) {
  if (x == nullptr || y_scalar == nullptr || y_pair == nullptr || y_exp2f == nullptr)
    return B2G_EINVAL;
  if (n < 0) return B2G_ESHAPE;
  if (n == 0) return B2G_OK;
  const int64_t pairs = (n + 1) / 2;
  const int blocks = static_cast<int>(std::min<int64_t>((pairs + 255) / 256, 148 * 8));
  poly_exp2_probe_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y_scalar, y_pair, y_exp2f, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}
