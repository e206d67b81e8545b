// extern "C" entry points of libb2g.so: argument checks, TMA descriptors,
// workspace carving, scheduler planning and kernel launches.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

#include "b2g.h"
#include "capi_internal.h"
#include "gemm_kernel.cuh"
#include "pack.cuh"
#include "sched.h"
#include "skinny_kernel.cuh"

using namespace b2g;

// Ring depths (stages of kKChunks x 128 bytes of K) per CTA shape; the shared-memory
// plan must fit 227 KB (checked at compile time).
#ifndef B2G_STAGES_CG1
#define B2G_STAGES_CG1 2
#endif
#ifndef B2G_STAGES_CG2
#define B2G_STAGES_CG2 3
#endif
#ifndef B2G_STAGES_CG2_SCALED
#define B2G_STAGES_CG2_SCALED 3
#endif

namespace {

// ------------------------------------------------------------- options --
struct Options {
  std::atomic<int64_t> pair{1};          // cta_group::2 CTA pairs
  std::atomic<int64_t> sk_mode{3};       // see make_plan
  std::atomic<int64_t> group_m{0};       // 0: chosen from the operand sizes (auto_group_m)
  // a split piece must span 16 stages: the fixed cost of publishing and adding
  // a partial tile (~13 us at 4096 x 4096) must stay below the half tile it saves
  std::atomic<int64_t> min_sk_iters{16};
  std::atomic<int64_t> timeout_ms{2000};
  std::atomic<int64_t> inject{0};
  std::atomic<int64_t> max_units{0};     // 0 = one unit per SM (pair)
  std::atomic<int64_t> prefetch{0};      // k-iterations pulled into L2 ahead of the ring
  std::atomic<int64_t> skinny_max_m{128};  // swap-AB kernel up to this M (0 = never)
  std::atomic<int64_t> skinny_splits{0};   // K splits per tile for it (0 = automatic)
  std::atomic<int64_t> serpentine{1};      // odd waves walk K backwards
};
Options g_opt;

constexpr int kMaxDevices = 64;

int device_sms(int dev) {
  static std::atomic<int> cache[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return -1;
  int v = cache[dev].load();
  if (v > 0) return v;
  int sms = 0, major = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return -1;
  if (major != 10) return -1;
  cache[dev].store(sms);
  return sms;
}

int current_sms() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return device_sms(dev);
}

// Stream-K owners wait for higher-numbered units, so every unit of a launch
// must be resident at once: cap the CTA-pair count at what the device can
// co-schedule (GPCs may not split evenly into pairs).
int pair_capacity(int dev, int sms) {
  static std::atomic<int> cache[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return sms / 2;
  int v = cache[dev].load();
  if (v > 0) return v;
  constexpr int kStages = B2G_STAGES_CG2;
  using SP = SmemPlan<kKindF16, 2, kStages>;
  auto kern = gemm_kernel<kKindF16, 2, kStages, false>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(SP::kDynBytes)) == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
    cfg.blockDim = dim3(SP::kThreads, 1, 1);
    cfg.dynamicSmemBytes = SP::kDynBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a failed query must not leak into the caller's error state
  v = (n > 0 && n < sms / 2) ? n : sms / 2;
  if (n <= 0) v = sms / 2 - 2;  // unknown: leave headroom
  cache[dev].store(v);
  return v;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool is_scaled(int kind) { return kind == B2G_KIND_MXE5M2 || kind == B2G_KIND_MXFP4; }

int64_t row_bytes(int kind, int64_t K) {
  switch (kind) {
    case B2G_KIND_F16:
    case B2G_KIND_BF16: return 2 * K;
    case B2G_KIND_E5M2:
    case B2G_KIND_MXE5M2: return K;
    default: return K / 2;
  }
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Zero-at-rest flag words at the start of every workspace: four per SM
// (split-tile flags; the small-M kernel's per-tile counters).
size_t flag_words(int sms) { return static_cast<size_t>(sms) * 4; }
size_t flag_region_bytes(int sms) { return align256(flag_words(sms) * sizeof(uint32_t)); }

struct Geometry {
  int cg;
  SkPlan plan;
  int launched;
  int sf_groups;  // 4-scale groups per row of the blocked scale layout
  size_t flags_off, flags_bytes, partial_off, partial_bytes;
  size_t sfa_off, sfa_bytes, sfb_off, sfb_bytes, total;
};

int64_t blocked_scale_bytes(int64_t rows, int64_t K) {
  return ((rows + 127) / 128) * ((K / 32 + 3) / 4) * 512;
}

// Raster group height when B2G_OPT_GROUP_M is 0, chosen so that the panels a
// wave shares stay in the 126 MB L2 and each operand is read from DRAM as few
// times as possible:
//  - A and B together within 96 MiB: everything stays in L2; row-major;
//  - A within 64 MiB: whole column strips (A stays, B is read once);
//  - B within 64 MiB: row-major (B stays, A is read once);
//  - neither: bands of tile rows whose A panels total about 32 MiB, walked
//    column by column (B is read once per band).
// Grouped GEMMs keep row-major: consecutive tile rows belong to one expert.
// Measured (interleaved, one box): FP16 4096 x 4096 x 8192 193.4 us in column
// strips against 196.4 us row-major, 3840^2 178.0 against 180.0; MXFP4
// 16384 x 53248 x 16384 (2 MiB A panels) 6.46 ms row-major, 5.63 / 5.37 / 5.75
// ms in bands of 8 / 16 / 32 tile rows; the 8- and 4-bit kinds at 4096^2, which
// fit in L2, 0.1-0.5 us slower in column strips.
int auto_group_m(int64_t rb, int M, int b_rows, int N, int cg, int tiles_m) {
  constexpr double kMiB = 1024.0 * 1024.0;
  const double a_bytes = static_cast<double>(M) * rb, b_bytes = static_cast<double>(b_rows) * rb;
  if (b_rows != N || a_bytes + b_bytes <= 96 * kMiB) return 1;
  if (a_bytes <= 64 * kMiB) return tiles_m;
  if (b_bytes <= 64 * kMiB) return 1;
  const double panel = 128.0 * cg * rb;
  const int band = static_cast<int>(32 * kMiB / panel);
  return std::max(1, std::min(band, tiles_m));
}

// `pair_cap`: how many CTA pairs the device can hold at once (0 = sms / 2).
// `b_rows`: rows of B and its scales (N, or groups * N for a grouped GEMM).
Geometry geometry(int kind, int M, int N, int K, int sms, int pair_cap = 0, int b_rows = 0) {
  if (b_rows <= 0) b_rows = N;
  Geometry g{};
  g.cg = g_opt.pair.load() != 0 ? 2 : 1;
  int units = g.cg == 2 ? sms / 2 : sms;
  if (g.cg == 2 && pair_cap > 0 && pair_cap < units) units = pair_cap;
  const int64_t mu = g_opt.max_units.load();
  if (mu > 0 && mu < units) units = static_cast<int>(mu);
  if (units < 1) units = 1;
  const int tiles_m = (M + 128 * g.cg - 1) / (128 * g.cg);
  const int tiles_n = (N + 255) / 256;
  const int k_chunks = static_cast<int>((row_bytes(kind, K) + 127) / 128);
  const int k_iters = (k_chunks + kKChunks - 1) / kKChunks;
  int group_m = static_cast<int>(g_opt.group_m.load());
  if (group_m == 0) group_m = auto_group_m(row_bytes(kind, K), M, b_rows, N, g.cg, tiles_m);
  g.plan = make_plan(tiles_m, tiles_n, k_iters, units, group_m,
                     static_cast<int>(g_opt.sk_mode.load()),
                     static_cast<int>(g_opt.min_sk_iters.load()));
  // the leftover items too for fp16 / bf16 (196.2 against 197.1 us at 4096^2;
  // the 8- and 4-bit kinds measured 0.1-0.3 us slower with them)
  const bool wide = kind == B2G_KIND_F16 || kind == B2G_KIND_BF16;
  g.plan.serpentine = g_opt.serpentine.load() != 0 ? (wide ? 3 : 1) : 0;
  g.launched = std::min(units, std::max(g.plan.dp_tiles, g.plan.sk_units));
  if (g.launched < 1) g.launched = 1;
  // Every workspace starts with the same fixed-size flag region (every unit
  // of every plan fits: units * cta_group <= SMs), reserved even by calls that
  // use no flags, so nothing another call writes (partial sums, relaid scales)
  // can sit where a later call looks for its flags, which must read zero.
  size_t off = 0;
  g.flags_off = off;
  g.flags_bytes = flag_region_bytes(sms);
  off += g.flags_bytes;
  g.partial_off = off;
  g.partial_bytes = static_cast<size_t>(g.plan.sk_units) * g.cg * 128 * 256 * sizeof(float);
  off += align256(g.partial_bytes);
  // scale relayout targets (scaled kinds, unless the caller passes blocked scales)
  g.sf_groups = is_scaled(kind) ? (K / 32 + 3) / 4 : 0;
  g.sfa_off = off;
  g.sfa_bytes = is_scaled(kind) ? static_cast<size_t>(blocked_scale_bytes(M, K)) : 0;
  off += align256(g.sfa_bytes);
  g.sfb_off = off;
  g.sfb_bytes = is_scaled(kind) ? static_cast<size_t>(blocked_scale_bytes(b_rows, K)) : 0;
  off += align256(g.sfb_bytes);
  g.total = off;
  return g;
}

// ------------------------------------------------------- skinny (small M) --
// Its per-tile arrival counters live in the flag region, one word per
// 128-column tile: wider problems take the persistent kernel.
bool use_skinny(int kind, int M, int N, int sms) {
  const int64_t lim = g_opt.skinny_max_m.load();
  return (kind == B2G_KIND_F16 || kind == B2G_KIND_BF16 || kind == B2G_KIND_E5M2) && lim > 0 &&
         M <= lim && M <= 128 && static_cast<size_t>((N + 127) / 128) <= flag_words(sms);
}

struct SkinnyGeom {
  int bn, tiles, splits, cps, k_chunks;
  size_t partial_off, partial_bytes, total;
};

// About one wave of (128-column tile, K split) CTAs: as many K splits as fit
// next to the tiles on the SMs, each keeping at least 8 chunks (or
// B2G_OPT_SKINNY_SPLITS when set).
// Counters live in the workspace's flag region, partial tiles after it.
SkinnyGeom skinny_geometry(int kind, int M, int N, int K, int sms) {
  SkinnyGeom g{};
  g.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  g.k_chunks = static_cast<int>((row_bytes(kind, K) + 127) / 128);
  g.tiles = (N + 127) / 128;
  const int64_t forced = g_opt.skinny_splits.load();
  const int want = std::max(1, sms / g.tiles);
  const int splits = forced > 0 ? static_cast<int>(std::min<int64_t>(forced, g.k_chunks))
                                : std::min(want, std::max(1, g.k_chunks / 8));
  g.cps = (g.k_chunks + splits - 1) / splits;
  g.splits = (g.k_chunks + g.cps - 1) / g.cps;
  g.partial_off = flag_region_bytes(sms);
  g.partial_bytes = g.splits > 1 ? static_cast<size_t>(g.tiles) * g.splits * 128 * g.bn * 4 : 0;
  g.total = g.partial_off + align256(g.partial_bytes);
  return g;
}

int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
              uint64_t outer, uint64_t stride_bytes, uint32_t box_in, uint32_t box_out,
              CUtensorMapSwizzle sw) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return B2G_ETENSORMAP;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_in, box_out};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2G_OK : B2G_ETENSORMAP;
}

// The GEMM is always launched with programmatic stream serialization, so its
// launch overlaps the tail of the kernel before it. `after_relayout`: that
// kernel is this library's scale relayout; the GEMM then waits for it only
// before loading scales (pdl_mode 1), otherwise before any global access
// (pdl_mode 2).
template <int KIND, int CG, bool OB>
int launch_gemm_t(const GemmParams& prm, int units, bool after_relayout, cudaStream_t stream) {
  constexpr bool kScaled = KindTraits<KIND>::kScaled;
  constexpr int kStages = CG == 1 ? B2G_STAGES_CG1 : (kScaled ? B2G_STAGES_CG2_SCALED : B2G_STAGES_CG2);
  using SP = SmemPlan<KIND, CG, kStages>;
  static_assert(SP::kDynBytes <= SP::kMaxDyn, "shared memory plan exceeds 227 KB");
  auto kern = gemm_kernel<KIND, CG, kStages, OB>;
  static std::atomic<uint64_t> attr_done{0};  // bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_done.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SP::kDynBytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(units * CG), 1, 1);
  cfg.blockDim = dim3(SP::kThreads, 1, 1);
  cfg.dynamicSmemBytes = SP::kDynBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n_attr = 0;
  if (CG == 2) {
    attr[n_attr].id = cudaLaunchAttributeClusterDimension;
    attr[n_attr].val.clusterDim.x = 2;
    attr[n_attr].val.clusterDim.y = 1;
    attr[n_attr].val.clusterDim.z = 1;
    ++n_attr;
  }
  attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
  ++n_attr;
  cfg.attrs = attr;
  cfg.numAttrs = n_attr;
  GemmParams prm2 = prm;
  prm2.pdl_mode = after_relayout ? 1 : 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm2);
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

template <int KIND, int CG>
int launch_gemm_out(const GemmParams& prm, int units, int out_dtype, bool dep, cudaStream_t s) {
  return out_dtype == B2G_DT_BF16 ? launch_gemm_t<KIND, CG, true>(prm, units, dep, s)
                                  : launch_gemm_t<KIND, CG, false>(prm, units, dep, s);
}

int dispatch(int kind, int cg, const GemmParams& prm, int units, int out_dtype, bool dep,
             cudaStream_t s) {
  switch (kind) {
    case B2G_KIND_F16:
      return cg == 2 ? launch_gemm_out<kKindF16, 2>(prm, units, out_dtype, dep, s)
                     : launch_gemm_out<kKindF16, 1>(prm, units, out_dtype, dep, s);
    case B2G_KIND_BF16:
      return cg == 2 ? launch_gemm_out<kKindBF16, 2>(prm, units, out_dtype, dep, s)
                     : launch_gemm_out<kKindBF16, 1>(prm, units, out_dtype, dep, s);
    case B2G_KIND_E5M2:
      return cg == 2 ? launch_gemm_out<kKindE5M2, 2>(prm, units, out_dtype, dep, s)
                     : launch_gemm_out<kKindE5M2, 1>(prm, units, out_dtype, dep, s);
    case B2G_KIND_MXE5M2:
      return cg == 2 ? launch_gemm_out<kKindMXE5M2, 2>(prm, units, out_dtype, dep, s)
                     : launch_gemm_out<kKindMXE5M2, 1>(prm, units, out_dtype, dep, s);
    case B2G_KIND_MXFP4:
      return cg == 2 ? launch_gemm_out<kKindMXFP4, 2>(prm, units, out_dtype, dep, s)
                     : launch_gemm_out<kKindMXFP4, 1>(prm, units, out_dtype, dep, s);
    default: return B2G_EINVAL;
  }
}

template <int KIND, int BN, bool OB>
int launch_skinny_t(const SkinnyParams& prm, int blocks, cudaStream_t stream) {
  using SP = SkinnyPlan<BN>;
  auto kern = skinny_kernel<KIND, BN, OB>;
  static std::atomic<uint64_t> attr_done{0};  // bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_done.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SP::kDynBytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done.fetch_or(bit);
  }
  kern<<<blocks, SP::kThreads, SP::kDynBytes, stream>>>(prm);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

template <int KIND, int BN>
int launch_skinny_out(const SkinnyParams& prm, int blocks, int out_dtype, cudaStream_t s) {
  return out_dtype == B2G_DT_BF16 ? launch_skinny_t<KIND, BN, true>(prm, blocks, s)
                                  : launch_skinny_t<KIND, BN, false>(prm, blocks, s);
}

template <int KIND>
int launch_skinny_bn(const SkinnyParams& prm, int bn, int blocks, int out_dtype,
                     cudaStream_t s) {
  switch (bn) {
    case 16: return launch_skinny_out<KIND, 16>(prm, blocks, out_dtype, s);
    case 32: return launch_skinny_out<KIND, 32>(prm, blocks, out_dtype, s);
    case 64: return launch_skinny_out<KIND, 64>(prm, blocks, out_dtype, s);
    default: return launch_skinny_out<KIND, 128>(prm, blocks, out_dtype, s);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct GemmCall {
  int kind;
  const void* A;
  int64_t lda;  // elements of A's storage type
  const void* B;
  int64_t ldb;
  const uint8_t* sfa;
  int64_t sfa_s0, sfa_s1;
  const uint8_t* sfb;
  int64_t sfb_s0, sfb_s1;
  void* C;
  int64_t ldc;
  int M, N, K, out_dtype;
  void* ws;
  size_t ws_bytes;
  int* status;
  cudaStream_t stream;
  const int32_t* groups;  // grouped GEMM: device row offsets (n_groups + 1), else null
  int n_groups;
};

// Storage bytes per stored element of A/B (packed e2m1: one byte holds 2).
int64_t storage_elem_bytes(int kind) {
  return (kind == B2G_KIND_F16 || kind == B2G_KIND_BF16) ? 2 : 1;
}

int check_call(const GemmCall& c) {
  if (c.kind < B2G_KIND_F16 || c.kind > B2G_KIND_MXFP4) return B2G_EINVAL;
  if (c.out_dtype != B2G_DT_F16 && c.out_dtype != B2G_DT_BF16) return B2G_EINVAL;
  if (c.A == nullptr || c.B == nullptr || c.C == nullptr) return B2G_EINVAL;
  if (c.M < 1 || c.N < 1 || c.K < 1) return B2G_ESHAPE;
  if (is_scaled(c.kind) && (c.K % 32) != 0) return B2G_ESHAPE;
  if (c.kind == B2G_KIND_MXFP4 && (c.K % 2) != 0) return B2G_ESHAPE;
  if (c.M > (1 << 30) || c.N > (1 << 30) || c.K > (1 << 30)) return B2G_ESHAPE;
  if (is_scaled(c.kind) && (c.sfa == nullptr || c.sfb == nullptr)) return B2G_EINVAL;
  const int64_t eb = storage_elem_bytes(c.kind);
  const int64_t rb = row_bytes(c.kind, c.K);
  if (!aligned16(c.A) || !aligned16(c.B) || !aligned16(c.C)) return B2G_EALIGN;
  if ((c.lda * eb) % 16 != 0 || (c.ldb * eb) % 16 != 0 || (c.ldc * 2) % 16 != 0)
    return B2G_EALIGN;
  if (c.lda * eb < rb || c.ldb * eb < rb || c.ldc < c.N) return B2G_ESTRIDE;
  if (is_scaled(c.kind) && (c.sfa_s0 < 0 || c.sfa_s1 < 0 || c.sfb_s0 < 0 || c.sfb_s1 < 0))
    return B2G_ESTRIDE;
  if (is_scaled(c.kind) && ((c.sfa_s0 == 0) != (c.sfa_s1 == 0) || (c.sfb_s0 == 0) != (c.sfb_s1 == 0)))
    return B2G_ESTRIDE;
  if (c.groups != nullptr) {
    if (c.kind != B2G_KIND_MXFP4 || c.n_groups < 1) return B2G_EINVAL;
    if (c.N % 128 != 0 || static_cast<int64_t>(c.n_groups) * c.N > (1 << 30)) return B2G_ESHAPE;
  }
  return B2G_OK;
}

// Everything one GEMM call launches, planned and with its tensor maps
// encoded. Every entry point plans and launches once; a prepared call
// (b2g_prepare_gemm) plans once and launches on every b2g_prepared_run.
struct Launch {
  int path;  // 0: the persistent kernel, 1: the small-M kernel
  int kind, out_dtype, dev;
  // persistent kernel
  int cg, units;
  bool relayout;  // the caller's (rows, K/32) scales are relaid first
  const uint8_t* rl_sa;
  int64_t rl_sa0, rl_sa1;
  int rl_rows_a;
  uint8_t* rl_dst_a;
  const uint8_t* rl_sb;
  int64_t rl_sb0, rl_sb1;
  int rl_rows_b;
  uint8_t* rl_dst_b;
  int rl_kscales;
  GemmParams prm;
  // small-M kernel
  int bn, blocks;
  SkinnyParams sprm;
};

// C = A * B^T for M <= 128 with the swap-AB kernel (skinny_kernel.cuh).
int plan_skinny(const GemmCall& c, int sms, Launch* L) {
  const SkinnyGeom g = skinny_geometry(c.kind, c.M, c.N, c.K, sms);
  if (c.ws == nullptr || c.ws_bytes < g.total) return B2G_EWORKSPACE;
  if ((reinterpret_cast<uintptr_t>(c.ws) & 255u) != 0) return B2G_EALIGN;
  uint8_t* ws = static_cast<uint8_t*>(c.ws);
  SkinnyParams prm;
  std::memset(&prm, 0, sizeof(prm));
  const int64_t eb = storage_elem_bytes(c.kind);
  const uint64_t rb = static_cast<uint64_t>(row_bytes(c.kind, c.K));
  int rc = encode_2d(&prm.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, c.B, rb, static_cast<uint64_t>(c.N),
                     static_cast<uint64_t>(c.ldb * eb), 128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B2G_OK) return rc;
  rc = encode_2d(&prm.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, c.A, rb, static_cast<uint64_t>(c.M),
                 static_cast<uint64_t>(c.lda * eb), 128, static_cast<uint32_t>(g.bn),
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B2G_OK) return rc;
  prm.C = c.C;
  prm.ldc = c.ldc;
  prm.partials = g.partial_bytes ? reinterpret_cast<float*>(ws + g.partial_off) : nullptr;
  prm.counters = reinterpret_cast<uint32_t*>(ws);  // inside the zero-at-rest flag region
  prm.status = c.status;
  prm.M = c.M;
  prm.N = c.N;
  prm.k_chunks = g.k_chunks;
  prm.splits = g.splits;
  prm.chunks_per_split = g.cps;
  prm.timeout_ns = static_cast<uint64_t>(g_opt.timeout_ms.load()) * 1000000ull;
  L->path = 1;
  L->kind = c.kind;
  L->out_dtype = c.out_dtype;
  L->bn = g.bn;
  L->blocks = g.tiles * g.splits;
  L->sprm = prm;
  return B2G_OK;
}

// `fixed`: a geometry the caller already planned (and sized its scratch by);
// null plans here from the current options.
int plan_gemm(const GemmCall& c, const Geometry* fixed, Launch* L) {
  int rc = check_call(c);
  if (rc != B2G_OK) return rc;
  int dev = -1;
  cudaGetDevice(&dev);
  const int sms = current_sms();
  if (sms <= 0) return B2G_ENODEVICE;
  std::memset(L, 0, sizeof(*L));
  L->dev = dev;
  if (fixed == nullptr && c.groups == nullptr && use_skinny(c.kind, c.M, c.N, sms))
    return plan_skinny(c, sms, L);
  const int b_rows = c.groups != nullptr ? c.n_groups * c.N : c.N;
  const Geometry g = fixed != nullptr
                         ? *fixed
                         : geometry(c.kind, c.M, c.N, c.K, sms, pair_capacity(dev, sms), b_rows);
  if (g.total > 0 && (c.ws == nullptr || c.ws_bytes < g.total)) return B2G_EWORKSPACE;
  if (c.ws != nullptr && (reinterpret_cast<uintptr_t>(c.ws) & 255u) != 0) return B2G_EALIGN;
  uint8_t* ws = static_cast<uint8_t*>(c.ws);

  GemmParams& prm = L->prm;
  bool relayout = false;
  const int64_t eb = storage_elem_bytes(c.kind);
  const uint64_t rb = static_cast<uint64_t>(row_bytes(c.kind, c.K));
  rc = encode_2d(&prm.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, c.A, rb, static_cast<uint64_t>(c.M),
                 static_cast<uint64_t>(c.lda * eb), 128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B2G_OK) return rc;
  rc = encode_2d(&prm.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, c.B, rb, static_cast<uint64_t>(b_rows),
                 static_cast<uint64_t>(c.ldb * eb), 128, g.cg == 1 ? 256 : 128,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B2G_OK) return rc;
  // half-width tiles of the last partial wave load half as many B rows
  rc = encode_2d(&prm.tmBh, CU_TENSOR_MAP_DATA_TYPE_UINT8, c.B, rb, static_cast<uint64_t>(b_rows),
                 static_cast<uint64_t>(c.ldb * eb), 128, g.cg == 1 ? 128 : 64,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B2G_OK) return rc;
  rc = encode_2d(&prm.tmC, CU_TENSOR_MAP_DATA_TYPE_UINT16, c.C, static_cast<uint64_t>(c.N),
                 static_cast<uint64_t>(c.M), static_cast<uint64_t>(c.ldc * 2), 32, 32,
                 CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc != B2G_OK) return rc;
  if (is_scaled(c.kind)) {
    // scales in the caller's (rows, K/32) layout are relaid into the workspace
    // in one launch; strides (0, 0) mean the tensor is already blocked
    const bool a_blocked = c.sfa_s0 == 0 && c.sfa_s1 == 0;
    const bool b_blocked = c.sfb_s0 == 0 && c.sfb_s1 == 0;
    const uint8_t* sfa = a_blocked ? c.sfa : ws + g.sfa_off;
    const uint8_t* sfb = b_blocked ? c.sfb : ws + g.sfb_off;
    if (!aligned16(sfa) || !aligned16(sfb)) return B2G_EALIGN;
    if (!a_blocked || !b_blocked) {
      relayout = true;
      L->rl_sa = a_blocked ? nullptr : c.sfa;
      L->rl_sa0 = c.sfa_s0;
      L->rl_sa1 = c.sfa_s1;
      L->rl_rows_a = c.M;
      L->rl_dst_a = ws + g.sfa_off;
      L->rl_sb = b_blocked ? nullptr : c.sfb;
      L->rl_sb0 = c.sfb_s0;
      L->rl_sb1 = c.sfb_s1;
      L->rl_rows_b = b_rows;
      L->rl_dst_b = ws + g.sfb_off;
      L->rl_kscales = c.K / 32;
    }
    const uint32_t gwords = static_cast<uint32_t>(c.kind == B2G_KIND_MXFP4 ? 256 : 128);
    const uint64_t row_words = static_cast<uint64_t>(g.sf_groups) * 128;
    rc = encode_2d(&prm.tmSFA, CU_TENSOR_MAP_DATA_TYPE_UINT32, sfa, row_words,
                   static_cast<uint64_t>((c.M + 127) / 128), row_words * 4, gwords, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != B2G_OK) return rc;
    rc = encode_2d(&prm.tmSFB, CU_TENSOR_MAP_DATA_TYPE_UINT32, sfb, row_words,
                   static_cast<uint64_t>((b_rows + 127) / 128), row_words * 4, gwords, 2,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != B2G_OK) return rc;
  }
  prm.partials = g.partial_bytes ? reinterpret_cast<float*>(ws + g.partial_off) : nullptr;
  if (prm.partials != nullptr) {
    rc = encode_2d(&prm.tmP, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, prm.partials, 256,
                   static_cast<uint64_t>(g.plan.sk_units) * g.cg * 128, 1024, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != B2G_OK) return rc;
    prm.has_tmp = 1;
  }
  prm.flags = g.flags_bytes ? reinterpret_cast<uint32_t*>(ws + g.flags_off) : nullptr;
  prm.status = c.status;
  prm.plan = g.plan;
  prm.M = c.M;
  prm.N = c.N;
  prm.K = c.K;
  prm.inject = static_cast<int32_t>(g_opt.inject.load());
  prm.prefetch = c.groups != nullptr ? 0 : static_cast<int32_t>(g_opt.prefetch.load());
  prm.groups = c.groups;
  prm.n_groups = c.n_groups;
  prm.group_rows = c.N;
  prm.timeout_ns = static_cast<uint64_t>(g_opt.timeout_ms.load()) * 1000000ull;
  prm.k_chunks = static_cast<int32_t>((rb + 127) / 128);
  L->path = 0;
  L->kind = c.kind;
  L->out_dtype = c.out_dtype;
  L->cg = g.cg;
  L->units = g.launched;
  L->relayout = relayout;
  return B2G_OK;
}

int launch_planned(const Launch& L, cudaStream_t stream) {
  if (L.path == 1) {
    switch (L.kind) {
      case B2G_KIND_F16: return launch_skinny_bn<0>(L.sprm, L.bn, L.blocks, L.out_dtype, stream);
      case B2G_KIND_BF16: return launch_skinny_bn<1>(L.sprm, L.bn, L.blocks, L.out_dtype, stream);
      default: return launch_skinny_bn<2>(L.sprm, L.bn, L.blocks, L.out_dtype, stream);
    }
  }
  if (L.relayout) {
    const cudaError_t e =
        launch_sf_relayout(L.rl_sa, L.rl_sa0, L.rl_sa1, L.rl_rows_a, L.rl_dst_a, L.rl_sb,
                           L.rl_sb0, L.rl_sb1, L.rl_rows_b, L.rl_dst_b, L.rl_kscales, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return dispatch(L.kind, L.cg, L.prm, L.units, L.out_dtype, L.relayout, stream);
}

int run_gemm(const GemmCall& c, const Geometry* fixed = nullptr) {
  Launch L;
  const int rc = plan_gemm(c, fixed, &L);
  if (rc != B2G_OK) return rc;
  return launch_planned(L, c.stream);
}

}  // namespace

namespace b2g {

int gemm_mxf4_fixed_scratch(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                            const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1,
                            const uint8_t* sfb, int64_t sfb_s0, int64_t sfb_s1, void* C,
                            int64_t ldc, int M, int N, int K, int out_dtype, void* scratch,
                            size_t capacity, int* status, cudaStream_t stream) {
  GemmCall c{};
  c.kind = B2G_KIND_MXFP4;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb;
  c.sfa = sfa; c.sfa_s0 = sfa_s0; c.sfa_s1 = sfa_s1;
  c.sfb = sfb; c.sfb_s0 = sfb_s0; c.sfb_s1 = sfb_s1;
  c.C = C; c.ldc = ldc; c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = scratch; c.ws_bytes = capacity; c.status = status;
  c.stream = stream;
  int rc = check_call(c);
  if (rc != B2G_OK) return rc;
  int dev = -1;
  cudaGetDevice(&dev);
  const int sms = current_sms();
  if (sms <= 0) return B2G_ENODEVICE;
  // planned once: the capacity check, the flag clear and the launch all use
  // this geometry, whatever b2g_set_option calls other threads make meanwhile
  const Geometry g = geometry(c.kind, c.M, c.N, c.K, sms, pair_capacity(dev, sms));
  if (g.total > capacity) return B2G_ECAPACITY;
  if (g.flags_bytes > 0) {
    // the scratch is not the caller's to reset, so a call that timed out must
    // not leave flags behind for the next one: clear them in stream order
    const cudaError_t e =
        cudaMemsetAsync(static_cast<uint8_t*>(scratch) + g.flags_off, 0, g.flags_bytes, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return run_gemm(c, &g);
}


int current_device_sms() { return current_sms(); }

PFN_cuTensorMapEncodeTiled_v12000 tma_encoder() { return tensor_map_encoder(); }

uint64_t wait_timeout_ns() { return static_cast<uint64_t>(g_opt.timeout_ms.load()) * 1000000ull; }

}  // namespace b2g

// The opaque handle of a prepared call: the planned launch itself.
struct b2g_prepared {
  Launch launch;
};

extern "C" {

int b2g_version(void) { return 100; }

const char* b2g_strerror(int code) {
  if (code >= B2G_STATUS_TIMEOUT && code < B2G_STATUS_TIMEOUT + 0x100) {
    switch (code & 0xFF) {
      case B2G_SITE_EMPTY: return "timeout: producer waiting for a free ring slot";
      case B2G_SITE_FULL: return "timeout: MMA waiting for a filled ring slot";
      case B2G_SITE_ACC_EMPTY: return "timeout: MMA waiting for a drained accumulator";
      case B2G_SITE_ACC_FULL: return "timeout: epilogue waiting for an accumulator";
      case B2G_SITE_OVERLAP: return "timeout: MMA waiting for shared accumulator columns";
      case B2G_SITE_FLAG: return "timeout: stream-K owner waiting for a contributor";
      case B2G_SITE_SCALES: return "timeout: MMA waiting for scale factors in TMEM";
      default: return "timeout in a bounded wait";
    }
  }
  switch (code) {
    case B2G_OK: return "ok";
    case B2G_EINVAL: return "invalid argument (kind, dtype or null pointer)";
    case B2G_ESHAPE: return "unsupported shape (M, N, K range or K multiple)";
    case B2G_EALIGN: return "pointer or row stride not 16-byte aligned";
    case B2G_ESTRIDE: return "operand not K-contiguous or row stride too small";
    case B2G_EWORKSPACE: return "workspace missing or too small";
    case B2G_ETENSORMAP: return "TMA descriptor rejected by the driver";
    case B2G_ENODEVICE: return "no sm_100 device is current";
    case B2G_ECAPACITY: return "size exceeds the entry point's fixed capacity";
    case B2G_STATUS_BAD_GROUPS:
      return "grouped GEMM refused to run: group offsets must start at 0, end at M, not "
             "decrease and be multiples of the tile height";
    case B2G_STATUS_SMEM_BASE:
      return "kernel refused to run: dynamic shared memory base needs more alignment padding "
             "than was reserved";
    default: break;
  }
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "unknown error";
}

size_t b2g_gemm_workspace_bytes(int kind, int M, int N, int K) {
  if (kind < B2G_KIND_F16 || kind > B2G_KIND_MXFP4 || M < 1 || N < 1 || K < 1) return 0;
  int dev = -1;
  cudaGetDevice(&dev);
  const int sms = current_sms();
  if (sms <= 0) return 0;
  if (use_skinny(kind, M, N, sms)) return skinny_geometry(kind, M, N, K, sms).total;
  return geometry(kind, M, N, K, sms, pair_capacity(dev, sms)).total;
}

int b2g_workspace_reset(void* workspace, size_t bytes, void* stream) {
  if (workspace == nullptr || bytes == 0) return B2G_OK;
  const cudaError_t e = cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

int b2g_gemm_f16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                 int M, int N, int K, int in_dtype, int out_dtype, void* workspace,
                 size_t workspace_bytes, int* status, void* stream) {
  if (in_dtype != B2G_DT_F16 && in_dtype != B2G_DT_BF16) return B2G_EINVAL;
  GemmCall c{};
  c.kind = in_dtype == B2G_DT_F16 ? B2G_KIND_F16 : B2G_KIND_BF16;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb; c.C = C; c.ldc = ldc;
  c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.status = status;
  c.stream = static_cast<cudaStream_t>(stream);
  return run_gemm(c);
}

int b2g_gemm_f8(const void* A, int64_t lda, const void* B, int64_t ldb, const uint8_t* sfa,
                int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb, int64_t sfb_s0,
                int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K, int out_dtype,
                void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if ((sfa == nullptr) != (sfb == nullptr)) return B2G_EINVAL;
  GemmCall c{};
  c.kind = sfa == nullptr ? B2G_KIND_E5M2 : B2G_KIND_MXE5M2;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb;
  c.sfa = sfa; c.sfa_s0 = sfa_s0; c.sfa_s1 = sfa_s1;
  c.sfb = sfb; c.sfb_s0 = sfb_s0; c.sfb_s1 = sfb_s1;
  c.C = C; c.ldc = ldc; c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.status = status;
  c.stream = static_cast<cudaStream_t>(stream);
  return run_gemm(c);
}

int b2g_gemm_mxf4(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                  const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb,
                  int64_t sfb_s0, int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K,
                  int out_dtype, void* workspace, size_t workspace_bytes, int* status,
                  void* stream) {
  GemmCall c{};
  c.kind = B2G_KIND_MXFP4;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb;
  c.sfa = sfa; c.sfa_s0 = sfa_s0; c.sfa_s1 = sfa_s1;
  c.sfb = sfb; c.sfb_s0 = sfb_s0; c.sfb_s1 = sfb_s1;
  c.C = C; c.ldc = ldc; c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.status = status;
  c.stream = static_cast<cudaStream_t>(stream);
  return run_gemm(c);
}

int b2g_gemm_mxf4_grouped(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                          const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb,
                          int64_t sfb_s0, int64_t sfb_s1, void* C, int64_t ldc,
                          const int32_t* group_offsets, int groups, int M, int N, int K,
                          int out_dtype, void* workspace, size_t workspace_bytes, int* status,
                          void* stream) {
  if (group_offsets == nullptr || groups < 1) return B2G_EINVAL;
  GemmCall c{};
  c.kind = B2G_KIND_MXFP4;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb;
  c.sfa = sfa; c.sfa_s0 = sfa_s0; c.sfa_s1 = sfa_s1;
  c.sfb = sfb; c.sfb_s0 = sfb_s0; c.sfb_s1 = sfb_s1;
  c.C = C; c.ldc = ldc; c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.status = status;
  c.stream = static_cast<cudaStream_t>(stream);
  c.groups = group_offsets;
  c.n_groups = groups;
  return run_gemm(c);
}

size_t b2g_gemm_grouped_workspace_bytes(int M, int N, int K, int groups) {
  if (M < 1 || N < 1 || K < 1 || groups < 1) return 0;
  int dev = -1;
  cudaGetDevice(&dev);
  const int sms = current_sms();
  if (sms <= 0) return 0;
  return geometry(B2G_KIND_MXFP4, M, N, K, sms, pair_capacity(dev, sms), groups * N).total;
}

int b2g_prepare_gemm(int kind, const void* A, int64_t lda, const void* B, int64_t ldb,
                     const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb,
                     int64_t sfb_s0, int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K,
                     int out_dtype, void* workspace, size_t workspace_bytes, int* status,
                     b2g_prepared** out) {
  if (out == nullptr) return B2G_EINVAL;
  *out = nullptr;
  if (kind < B2G_KIND_F16 || kind > B2G_KIND_MXFP4) return B2G_EINVAL;
  if (!is_scaled(kind) && (sfa != nullptr || sfb != nullptr)) return B2G_EINVAL;
  GemmCall c{};
  c.kind = kind;
  c.A = A; c.lda = lda; c.B = B; c.ldb = ldb;
  c.sfa = sfa; c.sfa_s0 = sfa_s0; c.sfa_s1 = sfa_s1;
  c.sfb = sfb; c.sfb_s0 = sfb_s0; c.sfb_s1 = sfb_s1;
  c.C = C; c.ldc = ldc; c.M = M; c.N = N; c.K = K; c.out_dtype = out_dtype;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.status = status;
  auto* p = new (std::nothrow) b2g_prepared;
  if (p == nullptr) return B2G_ECAPACITY;
  const int rc = plan_gemm(c, nullptr, &p->launch);
  if (rc != B2G_OK) {
    delete p;
    return rc;
  }
  *out = p;
  return B2G_OK;
}

int b2g_prepared_run(const b2g_prepared* prepared, void* stream) {
  if (prepared == nullptr) return B2G_EINVAL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != prepared->launch.dev) return B2G_ENODEVICE;
  return launch_planned(prepared->launch, static_cast<cudaStream_t>(stream));
}

void b2g_prepared_free(b2g_prepared* prepared) { delete prepared; }

int b2g_quant_mxfp4(const float* src, int64_t ld, int rows, int K, uint8_t* q, int64_t ldq,
                    uint8_t* scales, int64_t sc_s0, int64_t sc_s1, void* stream) {
  if (src == nullptr || q == nullptr || scales == nullptr) return B2G_EINVAL;
  if (rows < 1 || K < 32 || K % 32 != 0) return B2G_ESHAPE;
  if (!aligned16(src) || (ld % 4) != 0 || (reinterpret_cast<uintptr_t>(q) & 3u) != 0 ||
      (ldq % 4) != 0)
    return B2G_EALIGN;
  if (ld < K || ldq < K / 2 || sc_s0 < 0 || sc_s1 < 0) return B2G_ESTRIDE;
  const cudaError_t e = launch_quant_mxfp4(src, ld, rows, K, q, ldq, scales, sc_s0, sc_s1,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

int b2g_quant_mxe5m2(const float* src, int64_t ld, int rows, int K, const uint8_t* scales,
                     int64_t sc_s0, int64_t sc_s1, uint8_t* q, int64_t ldq, void* stream) {
  if (src == nullptr || q == nullptr || scales == nullptr) return B2G_EINVAL;
  if (rows < 1 || K < 32 || K % 32 != 0) return B2G_ESHAPE;
  if (!aligned16(src) || (ld % 4) != 0 || (reinterpret_cast<uintptr_t>(q) & 7u) != 0 ||
      (ldq % 8) != 0)
    return B2G_EALIGN;
  if (ld < K || ldq < K || sc_s0 < 0 || sc_s1 < 0) return B2G_ESTRIDE;
  const cudaError_t e = launch_quant_mxe5m2(src, ld, rows, K, scales, sc_s0, sc_s1, q, ldq,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

int b2g_cast_e5m2(const void* src, int src_dtype, int64_t n, uint8_t* dst, void* stream) {
  if (src == nullptr || dst == nullptr) return B2G_EINVAL;
  if (src_dtype != B2G_DT_F16 && src_dtype != B2G_DT_BF16 && src_dtype != B2G_DT_F32)
    return B2G_EINVAL;
  if (n < 0) return B2G_ESHAPE;
  if (n == 0) return B2G_OK;
  const cudaError_t e =
      launch_cast_e5m2(src, src_dtype, n, dst, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

size_t b2g_scales_blocked_bytes(int rows, int K) {
  if (rows < 1 || K < 32 || K % 32 != 0) return 0;
  return static_cast<size_t>(blocked_scale_bytes(rows, K));
}

int b2g_scales_to_blocked(const uint8_t* src, int64_t s0, int64_t s1, int rows, int K,
                          uint8_t* dst, void* stream) {
  if (src == nullptr || dst == nullptr) return B2G_EINVAL;
  if (rows < 1 || K < 32 || K % 32 != 0) return B2G_ESHAPE;
  if (s0 < 0 || s1 < 0 || (s0 == 0 && s1 == 0)) return B2G_ESTRIDE;
  if (!aligned16(dst)) return B2G_EALIGN;
  const cudaError_t e = launch_sf_relayout(src, s0, s1, rows, dst, nullptr, 0, 0, 0, nullptr,
                                           K / 32, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2G_OK : static_cast<int>(e);
}

int b2g_set_option(int key, int64_t value) {
  switch (key) {
    case B2G_OPT_PAIR: g_opt.pair.store(value != 0); return B2G_OK;
    case B2G_OPT_SK_MODE:
      if (value < 0 || value > 4) return B2G_EINVAL;
      g_opt.sk_mode.store(value);
      return B2G_OK;
    case B2G_OPT_GROUP_M:
      if (value < 0 || value > 64) return B2G_EINVAL;
      g_opt.group_m.store(value);
      return B2G_OK;
    case B2G_OPT_MIN_SK_ITERS:
      if (value < 1) return B2G_EINVAL;
      g_opt.min_sk_iters.store(value);
      return B2G_OK;
    case B2G_OPT_TIMEOUT_MS:
      if (value < 1 || value > 60000) return B2G_EINVAL;
      g_opt.timeout_ms.store(value);
      return B2G_OK;
    case B2G_OPT_INJECT_FLAG_TIMEOUT: g_opt.inject.store(value != 0); return B2G_OK;
    case B2G_OPT_MAX_UNITS:
      if (value < 0) return B2G_EINVAL;
      g_opt.max_units.store(value);
      return B2G_OK;
    case B2G_OPT_L2_PREFETCH:
      if (value < 0 || value > 64) return B2G_EINVAL;
      g_opt.prefetch.store(value);
      return B2G_OK;
    case B2G_OPT_SKINNY_MAX_M:
      if (value < 0 || value > 128) return B2G_EINVAL;
      g_opt.skinny_max_m.store(value);
      return B2G_OK;
    case B2G_OPT_SKINNY_SPLITS:
      if (value < 0 || value > 64) return B2G_EINVAL;
      g_opt.skinny_splits.store(value);
      return B2G_OK;
    case B2G_OPT_SERPENTINE:
      if (value < 0 || value > 1) return B2G_EINVAL;
      g_opt.serpentine.store(value);
      return B2G_OK;
    default: return B2G_EINVAL;
  }
}

int64_t b2g_get_option(int key) {
  switch (key) {
    case B2G_OPT_PAIR: return g_opt.pair.load();
    case B2G_OPT_SK_MODE: return g_opt.sk_mode.load();
    case B2G_OPT_GROUP_M: return g_opt.group_m.load();
    case B2G_OPT_MIN_SK_ITERS: return g_opt.min_sk_iters.load();
    case B2G_OPT_TIMEOUT_MS: return g_opt.timeout_ms.load();
    case B2G_OPT_INJECT_FLAG_TIMEOUT: return g_opt.inject.load();
    case B2G_OPT_MAX_UNITS: return g_opt.max_units.load();
    case B2G_OPT_L2_PREFETCH: return g_opt.prefetch.load();
    case B2G_OPT_SKINNY_MAX_M: return g_opt.skinny_max_m.load();
    case B2G_OPT_SKINNY_SPLITS: return g_opt.skinny_splits.load();
    case B2G_OPT_SERPENTINE: return g_opt.serpentine.load();
    default: return -1;
  }
}

int b2g_plan_query(int kind, int M, int N, int K, int num_sms, int32_t* out, int out_len) {
  if (out == nullptr || out_len < 11) return B2G_EINVAL;
  if (kind < B2G_KIND_F16 || kind > B2G_KIND_MXFP4 || M < 1 || N < 1 || K < 1 || num_sms < 2)
    return B2G_EINVAL;
  const Geometry g = geometry(kind, M, N, K, num_sms);
  out[0] = g.cg;
  out[1] = g.plan.tiles_m;
  out[2] = g.plan.tiles_n;
  out[3] = g.plan.k_iters;
  out[4] = g.plan.units;
  out[5] = g.plan.dp_tiles;
  out[6] = g.plan.sk_units;
  out[7] = g.launched;
  out[8] = g.plan.group_m;
  out[9] = g.plan.splits;
  out[10] = g.plan.half;
  return B2G_OK;
}

int b2g_plan_items(int kind, int M, int N, int K, int num_sms, int unit, int32_t* items,
                   int max_items) {
  if (kind < B2G_KIND_F16 || kind > B2G_KIND_MXFP4 || M < 1 || N < 1 || K < 1 || num_sms < 2)
    return B2G_EINVAL;
  const Geometry g = geometry(kind, M, N, K, num_sms);
  if (unit < 0 || unit >= g.launched) return 0;
  WorkCursor cur = cursor_begin(g.plan, unit);
  WorkItem w;
  int n = 0;
  while (cursor_next(g.plan, unit, cur, w)) {
    if (items != nullptr && n < max_items) {
      int32_t* o = items + 11 * n;
      o[0] = w.tile; o[1] = w.tm; o[2] = w.tn; o[3] = w.k_begin; o[4] = w.k_end;
      o[5] = w.role; o[6] = w.first_contrib; o[7] = w.n_contrib; o[8] = w.contrib_stride;
      o[9] = w.nh;
      o[10] = w.pair_half;
    }
    ++n;
  }
  return n;
}

}  // extern "C"
