// Persistent, warp-specialised C = A * B^T for sm_100a.
//
// Replaces the reference's per-tile Gluon kernels
//   a16w16  kernels/gemm/intra_wave/a16w16/v9_beyond_hotloop/matmul_kernel.py:32-388
//   a8w8    kernels/gemm/intra_wave/a8w8/matmul_kernel.py:33-435
//   a4w4    kernels/gemm/intra_wave/a4w4/v1_sliceMN/matmul_kernel.py:15-694
// with one template: A is M x K and B is N x K, both K-contiguous; C is M x N.
//
// CTA layout (192 threads, 224 for MXFP4):
//   warp 0      TMA producer: one thread fills a STAGES-deep shared-memory ring
//               (A tile, B tile and, for block-scaled kinds, the E8M0 scales,
//               pre-arranged in 512-byte blocks by a relayout pass).
//   warp 1      MMA issuer: allocates all 512 TMEM columns, one thread issues
//               tcgen05.mma into a double-buffered TMEM accumulator.
//   warps 2-5   epilogue: TMEM -> registers -> (split-tile fixup) -> bf16/fp16
//               -> swizzled smem -> TMA store. Warp w reads TMEM lanes
//               32*(w%4) .. 32*(w%4)+31.
//   warp 6      (MXFP4) scale copier: one thread copies each K chunk's scale
//               factors smem -> TMEM with tcgen05.cp into one of four per-chunk
//               TMEM slots, so the MMA thread's issue slots go to MMAs. A slot
//               is refilled as soon as the MMAs of the chunk that used it
//               complete (a commit per chunk), so the copier may run up to
//               three chunks ahead of the MMA thread. For scaled
//               e5m2 (half the scale bytes per stage) the MMA thread issues
//               the copies itself into a single slot, which measured faster.
//
// Tiles: cta_group::1 -> 128 x 256 per CTA; cta_group::2 -> 256 x 256 per CTA
// pair, each CTA loading its own 128 rows of A and its own 128 rows of B (the
// pair's MMA reads both halves; there is no multicast load anywhere). With
// block scales each CTA holds the scales of its own A rows and of all 256 B
// rows (two 512-byte blocks per group), which the pair's tcgen05.cp copies
// into each CTA's TMEM.
//
// Every K stage moves kKChunks chunks of 128 bytes of K per row (one TMA box
// per operand and chunk): a chunk is 64 fp16/bf16, 128 e5m2 or 256 packed
// e2m1 elements, i.e. four MMAs of 32 bytes of K. Two chunks per stage halve
// the per-K cost of the MMA thread's barrier wait, commit and loop control,
// which otherwise outlast the MMAs themselves.
//
// All waits are bounded (iteration probes plus a %globaltimer deadline). On a
// timeout the CTA records a status code, raises a CTA-wide abort flag, drains
// its in-flight copies and MMAs, frees TMEM and exits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "b2g.h"
#include "ptx.cuh"
#include "sched.h"

namespace b2g {

// 128-byte K chunks per pipeline stage (k-iterations count stages).
constexpr int kKChunks = 2;

enum : int {
  kKindF16 = 0,
  kKindBF16 = 1,
  kKindE5M2 = 2,    // unscaled e5m2 x e5m2 (kind::f8f6f4)
  kKindMXE5M2 = 3,  // e5m2 with E8M0 per 32 K (kind::mxf8f6f4.block_scale)
  kKindMXFP4 = 4,   // packed e2m1 with E8M0 per 32 K (kind::mxf4.block_scale)
};

struct alignas(64) GemmParams {
  CUtensorMap tmA;
  CUtensorMap tmB;
  CUtensorMap tmBh;     // B with half-height boxes, for half-width (N = 128) tiles
  CUtensorMap tmC;
  CUtensorMap tmSFA;    // blocked scales of A (u32 view: 128 words per 128-row group)
  CUtensorMap tmSFB;    // blocked scales of B
  CUtensorMap tmP;      // split-tile partials as fp32 rows of 256 (32 x 32 boxes, 128B swizzle)
  float* partials;      // split-tile partials, one 128 x 256 fp32 slot per CTA
  uint32_t* flags;      // split-tile flags, one per (unit, CTA of pair, epilogue warp)
  int* status;          // device status word, may be null
  SkPlan plan;
  int32_t M, N, K;
  int32_t inject;       // test hook: 1 = split-tile owners wait for a flag nobody raises
  // Launched with programmatic stream serialization. 1: right after this
  // library's scale relayout, which itself waited for every earlier kernel,
  // so A and B may be loaded at once and only the relaid scales wait;
  // 2: after an arbitrary kernel, so every thread waits for it to complete
  // before its first global memory access.
  int32_t pdl_mode;
  int32_t prefetch;     // k-iterations the producer pulls into L2 ahead of its loads
  int32_t has_tmp;      // tmP is valid
  int32_t k_chunks;     // 128-byte K chunks per row (the last stage may hold fewer)
  // Grouped GEMM (MoE experts): rows [groups[e], groups[e+1]) of A and C use
  // rows [e * group_rows, (e + 1) * group_rows) of B (and its scales). Null
  // for a plain GEMM.
  const int32_t* groups;
  int32_t n_groups;
  int32_t group_rows;
  uint64_t timeout_ns;
};

template <int KIND>
struct KindTraits {
  static constexpr bool kScaled = KIND == kKindMXE5M2 || KIND == kKindMXFP4;
  // 4-scale groups (one 512-byte atom per 128 rows) per stage: a stage holds
  // 128 bytes of K per row = 128 e5m2 (4 scales) or 256 e2m1 (8 scales).
  static constexpr int kGroupsPerStage = KIND == kKindMXFP4 ? 2 : 1;
  // a/b format field of the instruction descriptor.
  static constexpr uint32_t kFmt = KIND == kKindF16 ? 0u : 1u;
};

// Instruction descriptor of a half-width (N = 128) tile: the N field halved.
__device__ __forceinline__ uint32_t idesc_half(uint32_t idesc) {
  return (idesc & ~(0x3Fu << 17)) | ((128u >> 3) << 17);
}

template <int KIND, int CG>
__device__ __forceinline__ uint32_t make_idesc(uint32_t sf_id) {
  constexpr uint32_t kM = 128u * CG, kN = 256u;
  constexpr uint32_t f = KindTraits<KIND>::kFmt;
  if constexpr (!KindTraits<KIND>::kScaled) {
    // D fp32 | A fmt | B fmt | K-major both | N >> 3 | M >> 4
    return (1u << 4) | (f << 7) | (f << 10) | ((kN >> 3) << 17) | ((kM >> 4) << 24);
  } else {
    // B scale id | A fmt | B fmt | N >> 3 | scales are E8M0 | M >> 4 | A scale id
    return (sf_id << 4) | (f << 7) | (f << 10) | ((kN >> 3) << 17) | (1u << 23) |
           ((kM >> 4) << 24) | (sf_id << 29);
  }
}

template <int KIND, int CG, int STAGES>
struct SmemPlan {
  static constexpr bool kScaled = KindTraits<KIND>::kScaled;
  static constexpr int kGps = KindTraits<KIND>::kGroupsPerStage;
  // Block-scaled kinds: a scale-copy warp fills one TMEM scale slot per K
  // chunk; the slots belong to stages in pairs (stage it uses slots
  // 2 * (it % 2) + c), so a slot is free again once the MMAs of stage it - 2
  // have completed, which the ring's empty barrier of that stage already says.
  static constexpr uint32_t kSfSlots = kScaled ? 2 * kKChunks : 0;
  static constexpr uint32_t kThreads = kScaled ? 224 : 192;
  // per 128-byte K chunk
  static constexpr uint32_t kChunkA = 128 * 128;
  static constexpr uint32_t kBRows = CG == 1 ? 256 : 128;
  static constexpr uint32_t kChunkB = kBRows * 128;
  // scales for this CTA's 128 A rows and all 256 B rows of the tile
  static constexpr uint32_t kChunkSfa = kScaled ? kGps * 512 : 0;
  static constexpr uint32_t kChunkSfb = kScaled ? 2 * kGps * 512 : 0;
  // per stage
  static constexpr uint32_t kABytes = kKChunks * kChunkA;
  static constexpr uint32_t kBBytes = kKChunks * kChunkB;
  static constexpr uint32_t kSfaBytes = kKChunks * kChunkSfa;
  static constexpr uint32_t kSfbBytes = kKChunks * kChunkSfb;
  static constexpr uint32_t kEpiBufs = 2;
  static constexpr uint32_t kEpiBufBytes = 32 * 64;  // 32 rows x 32 cols x 2 B

  static constexpr uint32_t kAOff = 0;
  static constexpr uint32_t kBOff = kAOff + STAGES * kABytes;
  static constexpr uint32_t kSfaOff = kBOff + STAGES * kBBytes;
  static constexpr uint32_t kSfbOff = kSfaOff + STAGES * kSfaBytes;
  static constexpr uint32_t kEpiOff = ((kSfbOff + STAGES * kSfbBytes) + 1023u) & ~1023u;
  static constexpr uint32_t kBarOff = kEpiOff + 4 * kEpiBufs * kEpiBufBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], ovl, drain, fixup[4],
  // scale slots[4], copier drain + 3 spare, scales in smem[S]
  static constexpr uint32_t kNumBars = 3 * STAGES + 18;
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr uint32_t kBytes = kMiscOff + 16;
  // The carve-up starts on a 1024-byte boundary (128-byte-swizzled TMA tiles).
  // Up to 1 KB of slack is reserved for rounding the dynamic base up to it;
  // plans that fill the 227 KB limit reserve what is left, and the kernel
  // refuses to run if its base would need more.
  static constexpr uint32_t kMaxDyn = 232448;
  static constexpr uint32_t kSlack =
      kBytes + 1024 <= kMaxDyn ? 1024u : (kBytes <= kMaxDyn ? (kMaxDyn - kBytes) & ~15u : 0u);
  static constexpr uint32_t kDynBytes = kBytes + kSlack;

  // bytes the TMA lands per chunk on the leader's full barrier (A and B of
  // both CTAs) and on its scale barrier (both CTAs' scales)
  static constexpr uint32_t kChunkTx = CG * (kChunkA + kChunkB);
  static constexpr uint32_t kChunkTxHalf = CG * (kChunkA + kChunkB / 2);
  static constexpr uint32_t kChunkTxSf = CG * (kChunkSfa + kChunkSfb);

  // TMEM columns. Block-scaled kinds keep kSfSlots scale-factor slots (one K
  // chunk each) at the top of the 512 columns: per 4-scale group g, SFA (this
  // CTA's 128 rows) takes 4 columns at g * 4 and SFB (256 rows) 8 columns at
  // kSfaSlotCols + g * 8. SFA blocks sit on 4-column and SFB blocks on
  // 8-column boundaries, as in every layout this kernel has run with. The two
  // accumulators then overlap by kOvlChunks 32-column chunks, which the
  // epilogue drains first.
  static constexpr uint32_t kSfaSlotCols = kScaled ? (kGps * 4 + 7) / 8 * 8 : 0;
  static constexpr uint32_t kSfSlotCols = kScaled ? kSfaSlotCols + kGps * 8 : 0;
  static constexpr uint32_t kSfCols = (kSfSlots * kSfSlotCols + 31) / 32 * 32;
  static constexpr uint32_t kSfBase = 512 - kSfCols;
  static constexpr uint32_t kAccStride = kScaled ? kSfBase - 256 : 256;
  static constexpr uint32_t kOvlChunks = (256 - kAccStride) / 32;
  static_assert(kAccStride % 32 == 0 && kOvlChunks < 8, "TMEM column plan");
  static_assert(kSfBase % 8 == 0 && kSfSlotCols % 8 == 0 && kSfaSlotCols % 8 == 0,
                "scale-factor blocks on 8-column boundaries");
  static_assert(!kScaled || kKChunks == 2, "scale slots are paired with two-chunk stages");
  // the epilogue's last tile uses the idle A/B ring: 128 KB of split-tile
  // partials (4 warps x 32 KB) and 64 KB of output staging (4 warps x 16 KB)
  static_assert(STAGES * (kABytes + kBBytes) >= 196608, "operand ring holds the last-tile staging");
  __device__ static constexpr uint32_t sfa_col(uint32_t slot, int g) {
    return kSfBase + slot * kSfSlotCols + static_cast<uint32_t>(g) * 4;
  }
  __device__ static constexpr uint32_t sfb_col(uint32_t slot, int g) {
    return kSfBase + slot * kSfSlotCols + kSfaSlotCols + static_cast<uint32_t>(g) * 8;
  }
};

__device__ __forceinline__ void report_status(const GemmParams& p, int code) {
  if (p.status != nullptr) atomicCAS(p.status, 0, code);
}

// Bounded wait on an mbarrier phase. Returns false on timeout or when another
// warp of the CTA has aborted.
// `kSleep`: each probe may suspend the thread for up to 20 us (woken when the
// phase completes), for waits that normally last long; without it the probes
// use the hardware's own short suspend, for hand-offs on the critical path.
template <bool kClusterScope, bool kSleep = true>
__device__ __noinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                        const GemmParams& p, int site) {
  // the deadline and the abort flag are checked between probes
  constexpr uint32_t kHintNs = 20000;
  auto probe = [&]() {
    if constexpr (kSleep)
      return kClusterScope ? mbar_try_wait_cluster_sleep(bar, parity, kHintNs)
                           : mbar_try_wait_sleep(bar, parity, kHintNs);
    else
      return kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
  if (probe()) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (probe()) return true;
    if (*abort_flag != 0u) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      report_status(p, B2G_STATUS_TIMEOUT | site);
      *abort_flag = 1u;
      return false;
    }
  }
}

// wait_phase behind an inlined single probe. The ring's full barriers complete
// through TMA transaction bytes and are read only by tcgen05 operations, so
// the per-stage probe needs no cluster-scope acquire; a miss falls back to the
// bounded wait (with `kClusterScope` probes).
template <bool kClusterScope>
__device__ __forceinline__ bool wait_phase_fast(uint32_t bar, uint32_t parity,
                                                volatile uint32_t* abort_flag,
                                                const GemmParams& p, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_phase<kClusterScope>(bar, parity, abort_flag, p, site);
}

// Bounded wait that never suspends the thread, with CTA-scope probes: for the
// MMA thread at a tile boundary. The epilogue warps of both CTAs arrive on
// these barriers after their tcgen05.ld of the columns concerned has
// completed (tcgen05.wait::ld) and a tcgen05.fence::before_thread_sync; the
// MMA thread issues its next MMAs after tcgen05.fence::after_thread_sync. A
// probe with cluster-scope acquire was measured at 0.5-1.2 us per success
// while operand loads are in flight, a stall at every tile boundary.
__device__ __noinline__ bool wait_spin(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                       const GemmParams& p, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    if (*abort_flag != 0u) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      report_status(p, B2G_STATUS_TIMEOUT | site);
      *abort_flag = 1u;
      return false;
    }
  }
}

// Bounded wait for a global split-tile flag to reach `want`.
__device__ __noinline__ bool wait_flag(const uint32_t* flag, uint32_t want,
                                       volatile uint32_t* abort_flag, const GemmParams& p,
                                       int site) {
  if (ld_acquire_gpu(flag) == want) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (ld_acquire_gpu(flag) == want) return true;
      __nanosleep(64);
    }
    if (*abort_flag != 0u) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      report_status(p, B2G_STATUS_TIMEOUT | site);
      *abort_flag = 1u;
      return false;
    }
  }
}

// Grouped GEMM: the group whose rows [groups[e], groups[e+1]) contain `row`
// (the last of equal offsets, so empty groups are skipped).
__device__ __forceinline__ int32_t expert_of(const GemmParams& p, int32_t row) {
  int32_t lo = 0, hi = p.n_groups - 1;
  while (lo < hi) {
    const int32_t mid = (lo + hi + 1) >> 1;
    if (__ldg(p.groups + mid) <= row)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack_out(uint32_t lo, uint32_t hi) {
  const float a = __uint_as_float(lo), b = __uint_as_float(hi);
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

__device__ __forceinline__ size_t partial_slot(int32_t unit, uint32_t rank, int CG) {
  return (static_cast<size_t>(unit) * CG + rank) * (128u * 256u);
}

__device__ __forceinline__ size_t flag_index(int32_t unit, uint32_t rank, uint32_t quad, int CG) {
  return (static_cast<size_t>(unit) * CG + rank) * 4u + quad;
}

template <int KIND, int CG, int STAGES, bool OUT_BF16>
__global__ void __launch_bounds__((SmemPlan<KIND, CG, STAGES>::kThreads), 1)
    gemm_kernel(const __grid_constant__ GemmParams p) {
  using SP = SmemPlan<KIND, CG, STAGES>;
  constexpr bool kScaled = SP::kScaled;
  constexpr int kGps = SP::kGps;

  // The next kernel on the stream may be scheduled onto SMs as they free up
  // (it waits for this grid to complete before touching memory).
  if (threadIdx.x == 0) grid_launch_dependents();
  if (p.pdl_mode == 2) grid_dependency_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if (static_cast<uint32_t>(smem - smem_raw) > SP::kSlack) {
    // the same for every CTA of the launch: nothing has been touched yet
    if (threadIdx.x == 0) report_status(p, B2G_STATUS_SMEM_BASE);
    return;
  }
  if (p.groups != nullptr) {
    // Group offsets are read from device memory: every CTA checks them the
    // same way (0 first, M last, non-decreasing, multiples of the tile
    // height) and, if they are not, returns before touching anything.
    // a word of the misc area (tmem slot, abort flag, this) not yet in use
    volatile uint32_t& groups_ok = *reinterpret_cast<volatile uint32_t*>(smem + SP::kMiscOff + 8);
    if (threadIdx.x < 32) {
      bool ok = true;
      for (int32_t e = static_cast<int32_t>(threadIdx.x); e <= p.n_groups; e += 32) {
        const int32_t o = __ldg(p.groups + e);
        ok = ok && o >= 0 && o <= p.M && (o % (128 * CG)) == 0;
        if (e > 0) ok = ok && __ldg(p.groups + e - 1) <= o;
      }
      ok = __all_sync(0xffffffffu, ok);
      if (threadIdx.x == 0) {
        ok = ok && __ldg(p.groups) == 0 && __ldg(p.groups + p.n_groups) == p.M;
        groups_ok = ok ? 1u : 0u;
      }
    }
    __syncthreads();
    if (groups_ok == 0u) {
      if (threadIdx.x == 0) report_status(p, B2G_STATUS_BAD_GROUPS);
      return;
    }
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int32_t unit = CG == 2 ? static_cast<int32_t>(blockIdx.x >> 1)
                               : static_cast<int32_t>(blockIdx.x);

  const uint32_t bar0 = sbase + SP::kBarOff;
  auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
  auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (STAGES + s); };
  auto accf_bar = [&](uint32_t b) { return bar0 + 8u * (2 * STAGES + b); };
  auto acce_bar = [&](uint32_t b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  const uint32_t ovl_bar = bar0 + 8u * (2 * STAGES + 4);
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 5);
  auto fix_bar = [&](uint32_t q) { return bar0 + 8u * (2 * STAGES + 6 + q); };
  // scale slot `slot` filled (the copier's copies issued and ordered before
  // the MMA thread's next tcgen05 operations)
  auto sf_bar = [&](uint32_t slot) { return bar0 + 8u * (2 * STAGES + 10 + slot); };
  // the scale copier's own drain at exit
  const uint32_t cdrain_bar = bar0 + 8u * (2 * STAGES + 14);
  // stage s's scales landed in shared memory (loaded ahead of its A and B)
  auto sffull_bar = [&](uint32_t s) { return bar0 + 8u * (2 * STAGES + 18 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SP::kMiscOff);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + SP::kMiscOff + 4);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(sffull_bar(s), 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 4 * CG);
    }
    mbar_init(ovl_bar, 4 * CG);
    mbar_init(drain_bar, 1);
    for (uint32_t q = 0; q < 4; ++q) mbar_init(fix_bar(q), 1);
    for (uint32_t slot = 0; slot < 4; ++slot) mbar_init(sf_bar(slot), 1);
    mbar_init(cdrain_bar, 1);
    *abort_flag = 0u;
    fence_mbarrier_init();
    prefetch_tensormap(&p.tmA);
    prefetch_tensormap(&p.tmB);
    prefetch_tensormap(&p.tmBh);
    prefetch_tensormap(&p.tmC);
    if (p.has_tmp) prefetch_tensormap(&p.tmP);
    if constexpr (kScaled) {
      prefetch_tensormap(&p.tmSFA);
      prefetch_tensormap(&p.tmSFB);
    }
  }
  if (warp == 1) {
    tmem_alloc<CG>(smem_u32(tmem_slot), 512);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_arrive_wait();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const bool leader = (CG == 1) || rank == 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      uint32_t it = 0;
      bool sf_dep_done = false;
      WorkCursor cur = cursor_begin(p.plan, unit);
      WorkItem w;
      bool alive = true;
      // A second cursor runs `prefetch` k-iterations ahead and pulls those A/B
      // boxes into L2 (off by default).
      WorkCursor pf_cur = cur;
      WorkItem pf_w;
      bool pf_live = p.prefetch > 0 && cursor_next(p.plan, unit, pf_cur, pf_w);
      int32_t pf_k = pf_live ? pf_w.k_begin : 0;
      auto prefetch_one = [&]() {
        while (pf_live && pf_k >= pf_w.k_end) {
          pf_live = cursor_next(p.plan, unit, pf_cur, pf_w);
          pf_k = pf_live ? pf_w.k_begin : 0;
        }
        if (!pf_live) return;
        const int32_t ar = pf_w.tm * (128 * CG) + static_cast<int32_t>(rank) * 128;
        const int32_t br = pf_w.tn * 256 + (CG == 2 ? static_cast<int32_t>(rank) * 128 : 0);
        for (int32_t c = 0; c < kKChunks && pf_k * kKChunks + c < p.k_chunks; ++c) {
          tma_prefetch_l2_2d(&p.tmA, (pf_k * kKChunks + c) * 128, ar);
          tma_prefetch_l2_2d(&p.tmB, (pf_k * kKChunks + c) * 128, br);
        }
        ++pf_k;
      };
      for (int32_t i = 0; i < p.prefetch; ++i) prefetch_one();
      while (alive && cursor_next(p.plan, unit, cur, w)) {
        const int32_t a_row = w.tm * (128 * CG) + static_cast<int32_t>(rank) * 128;
        // grouped GEMM: the expert whose rows hold this M-tile picks B's rows
        const int32_t b_base = p.groups != nullptr ? expert_of(p, w.tm * (128 * CG)) * p.group_rows : 0;
        // a half-width tile (w.nh = 0 / 1) takes 128 of the tile's 256 B rows,
        // 64 per CTA of a pair, through the half-height tensor map
        const bool half = w.nh >= 0;
        const int32_t b_rows_cta = (CG == 2 ? 128 : 256) >> (half ? 1 : 0);
        const int32_t b_row = b_base + w.tn * 256 + (half ? w.nh * 128 : 0) +
                              (CG == 2 ? static_cast<int32_t>(rank) * b_rows_cta : 0);
        const CUtensorMap* tm_b = half ? &p.tmBh : &p.tmB;
        const uint32_t chunk_tx = half ? SP::kChunkTxHalf : SP::kChunkTx;
        // scales of B: the tile's first (or, for the second half, second)
        // 128-row block comes first in the box
        const int32_t sfb_row = (b_base >> 7) + w.tn * 2 + (half ? w.nh : 0);
        for (int32_t kk = w.k_begin; kk < w.k_end; ++kk, ++it) {
          const int32_t k = w.k_desc ? w.k_end - 1 - (kk - w.k_begin) : kk;
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1u;
          if (p.prefetch > 0) prefetch_one();
          if (!wait_phase_fast<false>(empty_bar(s), ph ^ 1u, abort_flag, p, B2G_SITE_EMPTY)) {
            alive = false;
            break;
          }
          // chunks past the end of K are neither loaded nor multiplied
          const int32_t nc = min(kKChunks, p.k_chunks - k * kKChunks);
          if constexpr (kScaled) {
            // the scale relayout launched just before this grid (programmatic
            // dependency) must have finished before the first scale load
            if (!sf_dep_done) {
              grid_dependency_wait();
              sf_dep_done = true;
            }
            // The stage's scales first, on their own barrier: they are small,
            // land well before A and B, and the copier can move them into TMEM
            // while the operands are still arriving.
            if (leader)
              mbar_arrive_expect_tx(sffull_bar(s), static_cast<uint32_t>(nc) * SP::kChunkTxSf);
            const uint32_t sb_ = CG == 1 ? sffull_bar(s) : map_to_cta(sffull_bar(s), 0);
            for (int32_t c = 0; c < nc; ++c) {
              const int32_t kc = k * kKChunks + c;
              // blocked scales: this CTA's 128-row group of A, both groups of the B tile
              const uint32_t sfa_dst = sbase + SP::kSfaOff + s * SP::kSfaBytes + c * SP::kChunkSfa;
              const uint32_t sfb_dst = sbase + SP::kSfbOff + s * SP::kSfbBytes + c * SP::kChunkSfb;
              const int32_t sx = kc * kGps * 128;
              if constexpr (CG == 1) {
                tma_load_2d(sfa_dst, &p.tmSFA, sb_, sx, a_row >> 7);
                tma_load_2d(sfb_dst, &p.tmSFB, sb_, sx, sfb_row);
              } else {
                tma_load_2d_pair(sfa_dst, &p.tmSFA, sb_, sx, a_row >> 7);
                tma_load_2d_pair(sfb_dst, &p.tmSFB, sb_, sx, sfb_row);
              }
            }
          }
          if (leader) mbar_arrive_expect_tx(full_bar(s), static_cast<uint32_t>(nc) * chunk_tx);
          const uint32_t fb = CG == 1 ? full_bar(s) : map_to_cta(full_bar(s), 0);
          for (int32_t c = 0; c < nc; ++c) {
            const int32_t kc = k * kKChunks + c;
            const uint32_t a_dst = sbase + SP::kAOff + s * SP::kABytes + c * SP::kChunkA;
            const uint32_t b_dst = sbase + SP::kBOff + s * SP::kBBytes + c * SP::kChunkB;
            if constexpr (CG == 1) {
              tma_load_2d(a_dst, &p.tmA, fb, kc * 128, a_row);
              tma_load_2d(b_dst, tm_b, fb, kc * 128, b_row);
            } else {
              tma_load_2d_pair(a_dst, &p.tmA, fb, kc * 128, a_row);
              tma_load_2d_pair(b_dst, tm_b, fb, kc * 128, b_row);
            }
          }
        }
      }
      // Drain: every load issued must have landed before the CTA can exit.
      if (leader) {
        const uint32_t first = it > STAGES ? it - STAGES : 0u;
        for (uint32_t i = first; i < it; ++i) {
          const uint32_t s = i % STAGES, ph = (i / STAGES) & 1u;
          uint32_t spins = 0;
          while (!mbar_try_wait(full_bar(s), ph) && spins < (1u << 20)) ++spins;
          if constexpr (kScaled) {
            spins = 0;
            while (!mbar_try_wait(sffull_bar(s), ph) && spins < (1u << 20)) ++spins;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    if (leader && lane == 0) {
      uint32_t it = 0, tcount = 0;
      WorkCursor cur = cursor_begin(p.plan, unit);
      WorkItem w;
      bool alive = true;
      while (alive && cursor_next(p.plan, unit, cur, w)) {
        const uint32_t b = tcount & 1u, aph = (tcount >> 1) & 1u;
        // tile boundary: the accumulator's previous tile drained (and, for the
        // scaled kinds, the columns shared with the other accumulator read)
        if (!wait_spin(acce_bar(b), aph ^ 1u, abort_flag, p, B2G_SITE_ACC_EMPTY)) break;
        if constexpr (kScaled) {
          if (tcount > 0 &&
              !wait_spin(ovl_bar, (tcount - 1) & 1u, abort_flag, p, B2G_SITE_OVERLAP))
            break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * SP::kAccStride;
        const bool half = w.nh >= 0;  // N = 128 instructions on the first 64 B rows per CTA
        for (int32_t kk = w.k_begin; kk < w.k_end; ++kk, ++it) {
          const int32_t k = w.k_desc ? w.k_end - 1 - (kk - w.k_begin) : kk;
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1u;
          if (!wait_phase_fast<false>(full_bar(s), ph, abort_flag, p, B2G_SITE_FULL)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const int32_t nc = min(kKChunks, p.k_chunks - k * kKChunks);
#pragma unroll
          for (int32_t c = 0; c < kKChunks; ++c) {
          if (c >= nc) break;
          [[maybe_unused]] const uint32_t slot = (it & 1u) * kKChunks + static_cast<uint32_t>(c);
          if constexpr (kScaled) {
            // this chunk's scale factors, copied into `slot` by the scale copier
            // (its copies precede these MMAs in the tensor pipe)
            if (!wait_phase_fast<false>(sf_bar(slot), (it >> 1) & 1u, abort_flag, p,
                                        B2G_SITE_SCALES)) {
              alive = false;
              break;
            }
            tc_fence_after();
          }
          const uint32_t a_addr = sbase + SP::kAOff + s * SP::kABytes + c * SP::kChunkA;
          const uint32_t b_addr = sbase + SP::kBOff + s * SP::kBBytes + c * SP::kChunkB;
          const uint64_t adesc = sdesc_kmajor_sw128(a_addr);
          const uint64_t bdesc = sdesc_kmajor_sw128(b_addr);
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            // +32 bytes of K per MMA inside the 128-byte swizzled row
            const uint64_t ad = adesc + 2u * j;
            const uint64_t bd = bdesc + 2u * j;
            const uint32_t acc = (kk > w.k_begin || c > 0 || j > 0) ? 1u : 0u;
            if constexpr (KIND == kKindF16 || KIND == kKindBF16) {
              const uint32_t id = make_idesc<KIND, CG>(0);
              mma_f16<CG>(d_tmem, ad, bd, half ? idesc_half(id) : id, acc);
            } else if constexpr (KIND == kKindE5M2) {
              const uint32_t id = make_idesc<KIND, CG>(0);
              mma_f8f6f4<CG>(d_tmem, ad, bd, half ? idesc_half(id) : id, acc);
            } else {
              const int g = KIND == kKindMXFP4 ? static_cast<int>(j >> 1) : 0;
              const uint32_t sf_id = KIND == kKindMXFP4 ? ((j & 1u) * 2u) : j;
              const uint32_t sfa_t = (tmem_base + SP::sfa_col(slot, g)) | (sf_id << 30);
              const uint32_t sfb_t = (tmem_base + SP::sfb_col(slot, g)) | (sf_id << 30);
              const uint32_t id = make_idesc<KIND, CG>(sf_id);
              if constexpr (KIND == kKindMXFP4)
                mma_mxf4<CG>(d_tmem, ad, bd, half ? idesc_half(id) : id, sfa_t, sfb_t, acc);
              else
                mma_mxf8f6f4<CG>(d_tmem, ad, bd, half ? idesc_half(id) : id, sfa_t, sfb_t, acc);
            }
          }
          }
          if (!alive) break;
          // frees the ring stage and, two stages later, this stage's scale slots
          if constexpr (CG == 1)
            tc_commit<1>(empty_bar(s));
          else
            tc_commit_pair(empty_bar(s), 0x3);
        }
        if (!alive) break;
        if constexpr (CG == 1)
          tc_commit<1>(accf_bar(b));
        else
          tc_commit_pair(accf_bar(b), 0x3);
        ++tcount;
      }
      // Drain: all MMAs issued by this thread complete before TMEM is freed.
      tc_commit<CG>(drain_bar);
      uint32_t spins = 0;
      while (!mbar_try_wait(drain_bar, 0) && spins < (1u << 22)) ++spins;
    }
  } else if (warp == 6) {
    // -------------------------------------------------------- scale copier --
    if constexpr (kScaled) {
      if (leader && lane == 0) {
        uint32_t it = 0;
        WorkCursor cur = cursor_begin(p.plan, unit);
        WorkItem w;
        bool alive = true;
        while (alive && cursor_next(p.plan, unit, cur, w)) {
          for (int32_t kk = w.k_begin; kk < w.k_end; ++kk, ++it) {
          const int32_t k = w.k_desc ? w.k_end - 1 - (kk - w.k_begin) : kk;
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1u;
            // this stage's scales are in shared memory ...
            if (!wait_phase_fast<false>(sffull_bar(s), ph, abort_flag, p, B2G_SITE_FULL)) {
              alive = false;
              break;
            }
            // ... and the MMAs of stage it - 2, the last readers of its slots, are done
            if (it >= 2) {
              const uint32_t pi = it - 2;
              if (!wait_phase_fast<false>(empty_bar(pi % STAGES), (pi / STAGES) & 1u, abort_flag, p,
                                          B2G_SITE_EMPTY)) {
                alive = false;
                break;
              }
            }
            tc_fence_after();
            const int32_t nc = min(kKChunks, p.k_chunks - k * kKChunks);
#pragma unroll
            for (int32_t c = 0; c < kKChunks; ++c) {
              const uint32_t slot = (it & 1u) * kKChunks + static_cast<uint32_t>(c);
              if (c < nc) {
                const uint32_t sfa_addr =
                    sbase + SP::kSfaOff + s * SP::kSfaBytes + c * SP::kChunkSfa;
                const uint32_t sfb_addr =
                    sbase + SP::kSfbOff + s * SP::kSfbBytes + c * SP::kChunkSfb;
#pragma unroll
                for (int g = 0; g < kGps; ++g) {
                  tmem_cp_32x128b_x4<CG>(tmem_base + SP::sfa_col(slot, g),
                                         sdesc_rows16(sfa_addr + g * 512));
#pragma unroll
                  for (int rb = 0; rb < 2; ++rb)
                    tmem_cp_32x128b_x4<CG>(tmem_base + SP::sfb_col(slot, g) + 4 * rb,
                                           sdesc_rows16(sfb_addr + (rb * kGps + g) * 512));
                }
              }
              // Every slot of the stage is signalled (also a chunk past the end
              // of K), so each slot's phase count stays it / 2. The fence orders
              // the copies before the arrival: a tcgen05.cp followed by a
              // tcgen05.mma that another thread issues after observing this
              // arrival (and its own tcgen05.fence::after_thread_sync) runs in
              // that order in the tensor pipe.
              tc_fence_before();
              mbar_arrive(sf_bar(slot));
            }
          }
        }
        // Drain: this thread's copies complete before TMEM can be freed.
        tc_commit<CG>(cdrain_bar);
        uint32_t spins = 0;
        while (!mbar_try_wait(cdrain_bar, 0) && spins < (1u << 22)) ++spins;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const uint32_t quad = warp & 3u;
    const uint32_t row = quad * 32u + lane;  // accumulator row inside the CTA
    uint8_t* stage_base = smem + SP::kEpiOff + (warp - 2) * SP::kEpiBufs * SP::kEpiBufBytes;
    uint32_t tcount = 0, nstore = 0;
    WorkCursor cur = cursor_begin(p.plan, unit);
    WorkItem w;
    while (cursor_next(p.plan, unit, cur, w)) {
      const uint32_t b = tcount & 1u, aph = (tcount >> 1) & 1u;
      const bool ok = wait_phase<false, false>(accf_bar(b), aph, abort_flag, p, B2G_SITE_ACC_FULL);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((quad * 32u) << 16) + b * SP::kAccStride;
      const int32_t m0 = w.tm * (128 * CG) + static_cast<int32_t>(rank) * 128 + quad * 32;
      const bool half = w.nh >= 0;  // a half-width tile fills chunks 0-3 only
      const int32_t n0 = w.tn * 256 + (half ? w.nh * 128 : 0);
      // With overlapping accumulators the shared chunks are drained first. A
      // piece of a two-piece split tile (always its unit's last item, so no
      // later tile waits for particular columns) starts with the four chunks
      // it hands to its peer: chunks pub_lo .. pub_lo + 3 are published, then
      // the other four reduced and stored.
      const uint32_t pub_lo = w.pair_half == 0 ? 4u : 0u;
      const uint32_t first_chunk =
          w.role == kRolePair ? pub_lo : (kScaled ? (b == 0 ? 8u - SP::kOvlChunks : 0u) : 0u);
      bool pair_ok = true;
      // A split item that is this unit's last one finds the operand ring idle
      // (all its loads were consumed): each epilogue warp then moves its 32 x
      // 256 fp32 partial through its own 32 KB of the ring with bulk TMA copies
      // instead of per-thread global loads / stores.
      const bool last_item = [&] {
        WorkCursor c2 = cur;
        WorkItem w2;
        return !cursor_next(p.plan, unit, c2, w2);
      }();
      const bool ring_fix = last_item && w.role != kRoleFull && p.has_tmp != 0;
      uint8_t* ring = smem + quad * 32768u;
      int32_t glob_first = w.first_contrib, glob_n = w.n_contrib;
      if (w.role == kRoleOwner) {
        bool fok = true;
        for (int32_t ci2 = 0, u2 = w.first_contrib; ci2 < w.n_contrib && fok;
             ++ci2, u2 += w.contrib_stride)
          fok = wait_flag(p.flags + flag_index(u2, rank, quad, CG), p.inject ? 2u : 1u,
                          abort_flag, p, B2G_SITE_FLAG);
        fok = __all_sync(0xffffffffu, fok);
        if (fok && ring_fix) {
          fence_proxy_async_all();  // partials seen by the flag acquire -> TMA reads
          if (lane == 0) {
            mbar_arrive_expect_tx(fix_bar(quad), 8u * 4096u);
            const int32_t y = (w.first_contrib * CG + static_cast<int32_t>(rank)) * 128 +
                              static_cast<int32_t>(quad) * 32;
            for (uint32_t c = 0; c < 8; ++c)
              tma_load_2d(smem_u32(ring) + c * 4096u, &p.tmP, fix_bar(quad),
                          static_cast<int32_t>(c * 32u), y);
          }
          fok = wait_phase<false>(fix_bar(quad), 0, abort_flag, p, B2G_SITE_FLAG);
          fok = __all_sync(0xffffffffu, fok);
          glob_first += w.contrib_stride;
          glob_n -= 1;
        }
        if (!fok) break;
      }
      // A unit's last tile stages all eight of its output chunks in the idle
      // operand ring (beyond the 128 KB the split-tile partials may occupy),
      // so its TMA stores go out back to back without waiting for one another.
      uint8_t* const stage_last = smem + 131072u + quad * 16384u;
      // Convert and stage 32 rows x 32 columns in the 64-byte swizzle, then
      // one TMA store per warp (the tensor map clips rows / columns past C).
      // Chunks wholly outside C are skipped without touching the staging
      // buffers. Other tiles alternate two buffers per store actually issued:
      // the buffer being written is never the one the newest store may still
      // be reading.
      auto store_c = [&](uint32_t c, const uint32_t (&v)[32]) {
        const int32_t x = n0 + static_cast<int32_t>(c * 32u);
        if (x >= p.N || m0 >= p.M) return;
        uint8_t* buf;
        if (last_item) {
          buf = stage_last + c * SP::kEpiBufBytes;
        } else {
          buf = stage_base + (nstore & 1u) * SP::kEpiBufBytes;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
        }
#pragma unroll
        for (uint32_t pc = 0; pc < 4; ++pc) {
          uint4 q4;
          q4.x = pack_out<OUT_BF16>(v[8 * pc + 0], v[8 * pc + 1]);
          q4.y = pack_out<OUT_BF16>(v[8 * pc + 2], v[8 * pc + 3]);
          q4.z = pack_out<OUT_BF16>(v[8 * pc + 4], v[8 * pc + 5]);
          q4.w = pack_out<OUT_BF16>(v[8 * pc + 6], v[8 * pc + 7]);
          const uint32_t off = lane * 64u + ((pc ^ ((lane >> 1) & 3u)) << 4);
          *reinterpret_cast<uint4*>(buf + off) = q4;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&p.tmC, smem_u32(buf), x, m0);
          bulk_commit_group();
        }
        ++nstore;
      };
      // One 32-column chunk: the split-tile part, then convert, stage and store.
      auto body = [&](uint32_t ci, uint32_t (&v)[32]) {
        const uint32_t c = (first_chunk + ci) & 7u;
        if (half && c >= 4u) return;
        if (w.role == kRolePair) {
          if (!pair_ok) return;
          const int32_t peer = w.first_contrib;
          if (ci < 4u) {
            // the peer's half: this piece's fp32 partial
            if (ring_fix) {
              // 32 rows x 32 fp32 in the 128-byte swizzle, one box per chunk
              uint8_t* box = ring + ci * 4096u + lane * 128u;
#pragma unroll
              for (uint32_t q = 0; q < 8; ++q)
                *reinterpret_cast<uint4*>(box + ((q ^ (lane & 7u)) << 4)) =
                    make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
              float4* dst = reinterpret_cast<float4*>(p.partials + partial_slot(unit, rank, CG) +
                                                      static_cast<size_t>(row) * 256u + c * 32u);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                __stcg(dst + i,
                       make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
            }
            if (ci < 3u) return;
            // all four published: raise this piece's flag, then take the peer's
            // partial of this piece's half (its flag) into the ring's upper 16 KB
            if (ring_fix) {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                const int32_t y = (unit * CG + static_cast<int32_t>(rank)) * 128 +
                                  static_cast<int32_t>(quad) * 32;
                for (uint32_t j = 0; j < 4; ++j)
                  tma_store_2d(&p.tmP, smem_u32(ring + j * 4096u),
                               static_cast<int32_t>(((pub_lo + j) & 7u) * 32u), y);
                bulk_commit_group();
                bulk_wait_group<0>();   // partial written to global memory
                fence_proxy_async_all();
              }
            } else {
              __threadfence();
            }
            __syncwarp();
            if (lane == 0) st_release_gpu(p.flags + flag_index(unit, rank, quad, CG), 1u);
            bool fok = wait_flag(p.flags + flag_index(peer, rank, quad, CG), p.inject ? 2u : 1u,
                                 abort_flag, p, B2G_SITE_FLAG);
            fok = __all_sync(0xffffffffu, fok);
            if (fok && ring_fix) {
              fence_proxy_async_all();  // partials seen by the flag acquire -> TMA reads
              if (lane == 0) {
                mbar_arrive_expect_tx(fix_bar(quad), 4u * 4096u);
                const int32_t y = (peer * CG + static_cast<int32_t>(rank)) * 128 +
                                  static_cast<int32_t>(quad) * 32;
                for (uint32_t j = 0; j < 4; ++j)
                  tma_load_2d(smem_u32(ring + 16384u + j * 4096u), &p.tmP, fix_bar(quad),
                              static_cast<int32_t>(((pub_lo + 4u + j) & 7u) * 32u), y);
              }
              fok = wait_phase<false>(fix_bar(quad), 0, abort_flag, p, B2G_SITE_FLAG);
              fok = __all_sync(0xffffffffu, fok);
            }
            pair_ok = fok;
            return;
          }
          // this piece's half: own accumulator + the peer's partial
          if (ring_fix) {
            const uint8_t* box = ring + 16384u + (ci - 4u) * 4096u + lane * 128u;
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q) {
              const float4 t = *reinterpret_cast<const float4*>(box + ((q ^ (lane & 7u)) << 4));
              v[4 * q + 0] = __float_as_uint(__uint_as_float(v[4 * q + 0]) + t.x);
              v[4 * q + 1] = __float_as_uint(__uint_as_float(v[4 * q + 1]) + t.y);
              v[4 * q + 2] = __float_as_uint(__uint_as_float(v[4 * q + 2]) + t.z);
              v[4 * q + 3] = __float_as_uint(__uint_as_float(v[4 * q + 3]) + t.w);
            }
          } else {
            const float4* src = reinterpret_cast<const float4*>(
                p.partials + partial_slot(peer, rank, CG) + static_cast<size_t>(row) * 256u +
                c * 32u);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 t = __ldcg(src + i);
              v[4 * i + 0] = __float_as_uint(__uint_as_float(v[4 * i + 0]) + t.x);
              v[4 * i + 1] = __float_as_uint(__uint_as_float(v[4 * i + 1]) + t.y);
              v[4 * i + 2] = __float_as_uint(__uint_as_float(v[4 * i + 2]) + t.z);
              v[4 * i + 3] = __float_as_uint(__uint_as_float(v[4 * i + 3]) + t.w);
            }
          }
          store_c(c, v);
          return;
        }
        if (w.role == kRoleContrib) {
          if (ring_fix) {
            // 32 rows x 32 fp32 in the 128-byte swizzle, one box per chunk
            uint8_t* box = ring + c * 4096u + lane * 128u;
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q)
              *reinterpret_cast<uint4*>(box + ((q ^ (lane & 7u)) << 4)) =
                  make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
            float4* dst = reinterpret_cast<float4*>(p.partials + partial_slot(unit, rank, CG) +
                                                    static_cast<size_t>(row) * 256u + c * 32u);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              __stcg(dst + i,
                     make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                 __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
          }
          return;
        }
        if (w.role == kRoleOwner) {
          if (ring_fix) {
            const uint8_t* box = ring + c * 4096u + lane * 128u;
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q) {
              const float4 t = *reinterpret_cast<const float4*>(box + ((q ^ (lane & 7u)) << 4));
              v[4 * q + 0] = __float_as_uint(__uint_as_float(v[4 * q + 0]) + t.x);
              v[4 * q + 1] = __float_as_uint(__uint_as_float(v[4 * q + 1]) + t.y);
              v[4 * q + 2] = __float_as_uint(__uint_as_float(v[4 * q + 2]) + t.z);
              v[4 * q + 3] = __float_as_uint(__uint_as_float(v[4 * q + 3]) + t.w);
            }
          }
          for (int32_t ci2 = 0, u2 = glob_first; ci2 < glob_n; ++ci2, u2 += w.contrib_stride) {
            const float4* src = reinterpret_cast<const float4*>(
                p.partials + partial_slot(u2, rank, CG) + static_cast<size_t>(row) * 256u +
                c * 32u);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 t = __ldcg(src + i);
              v[4 * i + 0] = __float_as_uint(__uint_as_float(v[4 * i + 0]) + t.x);
              v[4 * i + 1] = __float_as_uint(__uint_as_float(v[4 * i + 1]) + t.y);
              v[4 * i + 2] = __float_as_uint(__uint_as_float(v[4 * i + 2]) + t.z);
              v[4 * i + 3] = __float_as_uint(__uint_as_float(v[4 * i + 3]) + t.w);
            }
          }
        }
        store_c(c, v);
      };
      // The chunks shared with the other accumulator go to registers first and
      // are released at once, so the next tile's MMAs wait for three TMEM loads
      // rather than for the conversion and stores of the chunks before them.
      constexpr uint32_t kPre = kScaled ? SP::kOvlChunks : 0u;
      uint32_t pre[kPre > 0 ? kPre : 1][32];
      if constexpr (kPre > 0) {
#pragma unroll
        for (uint32_t k = 0; k < kPre; ++k)
          tmem_ld_32x32b_x32(tbase + ((first_chunk + k) & 7u) * 32u, pre[k]);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t k = 0; k < kPre; ++k) tmem_regs_ready(pre[k]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1)
            mbar_arrive(ovl_bar);
          else
            mbar_arrive_remote_relaxed(map_to_cta(ovl_bar, 0));
        }
      }
      // The drained chunks first, with compile-time indices so that each set of
      // registers dies once used; the first TMEM chunk after them is already
      // loading. Then two register buffers: the next chunk's TMEM load is in
      // flight while the current one is converted and stored.
      auto fetch = [&](uint32_t ci, uint32_t (&v)[32]) {
        tmem_ld_32x32b_x32(tbase + ((first_chunk + ci) & 7u) * 32u, v);
      };
      auto ready = [&](uint32_t (&v)[32]) {
        tmem_wait_ld();
        tmem_regs_ready(v);
      };
      uint32_t va[32], vb[32];
      fetch(kPre, va);
      if constexpr (kPre > 0) {
#pragma unroll
        for (uint32_t k = 0; k < kPre; ++k) body(k, pre[k]);
      }
      uint32_t ci = kPre;
#pragma unroll 1
      for (; ci + 1 < 8u; ci += 2) {
        ready(va);
        fetch(ci + 1, vb);
        body(ci, va);
        ready(vb);
        if (ci + 2 < 8u) fetch(ci + 2, va);
        body(ci + 1, vb);
      }
      if (ci < 8u) {
        ready(va);
        body(ci, va);
      }
      if (!pair_ok) break;
      if (w.role == kRoleContrib) {
        if (ring_fix) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int32_t y = (unit * CG + static_cast<int32_t>(rank)) * 128 +
                              static_cast<int32_t>(quad) * 32;
            for (uint32_t c = 0; c < 8; ++c)
              tma_store_2d(&p.tmP, smem_u32(ring + c * 4096u), static_cast<int32_t>(c * 32u), y);
            bulk_commit_group();
            bulk_wait_group<0>();   // partial written to global memory
            fence_proxy_async_all();
          }
        } else {
          __threadfence();
        }
        __syncwarp();
        if (lane == 0) st_release_gpu(p.flags + flag_index(unit, rank, quad, CG), 1u);
      } else if (w.role == kRoleOwner || w.role == kRolePair) {
        // the contributors' (the peer's) flags have been consumed: zero at rest
        __syncwarp();
        if (lane == 0)
          for (int32_t ci2 = 0, u2 = w.first_contrib; ci2 < w.n_contrib;
               ++ci2, u2 += w.contrib_stride)
            p.flags[flag_index(u2, rank, quad, CG)] = 0u;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 1)
          mbar_arrive(acce_bar(b));
        else
          mbar_arrive_remote_relaxed(map_to_cta(acce_bar(b), 0));
      }
      ++tcount;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------- teardown --
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_arrive_wait();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, 512);
  }
}

}  // namespace b2g
