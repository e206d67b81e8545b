/*
 * b2g.h - C ABI of the B200 (sm_100a) GEMM hot path: C = A * B^T in
 * FP16/BF16 (a16w16), BF8 = E5M2 (a8w8, unscaled or with E8M0 per-32-K scales)
 * and MXFP4 = packed E2M1 with E8M0 per-32-K scales (a4w4), plus the
 * quantise-and-pack kernels that produce the low-precision operands.
 *
 * Conventions (all entry points):
 *   - Plain device pointers, element strides in elements of the operand's own
 *     storage type (bytes for e5m2, packed e2m1 and E8M0 scales), `stream` is a
 *     cudaStream_t passed as void*.
 *   - A is M x K and B is N x K, both K-contiguous (row stride lda / ldb);
 *     C is M x N row-major with row stride ldc. This is the layout the
 *     reference's kernels see when its bench passes `b` as a (K, N) view of an
 *     (N, K) K-contiguous tensor.
 *   - Launches are asynchronous on `stream`. Nothing synchronises.
 *   - Return value: 0 on success, a negative B2G_E* code when an argument is
 *     rejected before launch (nothing was launched), or a positive CUDA error.
 *   - `status` (nullable) is a device int the kernel sets to a nonzero
 *     B2G_STATUS_* code when a bounded wait expired. Zero it before use; read
 *     it after synchronising. After a nonzero status the workspace flags may be
 *     stale: clear the workspace with b2g_workspace_reset before reuse.
 *   - `workspace` is caller-owned device memory of at least
 *     b2g_gemm_workspace_bytes(...) bytes, zeroed once when allocated
 *     (b2g_workspace_reset). The kernels leave it zeroed after a successful
 *     run. Calls that share a workspace must not overlap on the GPU.
 *
 * Reference interfaces replaced (paths inside jamesbowley/gfx950-gluon-tutorials):
 *   a16w16 matmul(a, b, c=None)
 *       kernels/gemm/intra_wave/a16w16/v9_beyond_hotloop/matmul_kernel.py:390-424
 *       kernels/gemm/inter_wave/a16w16/matmul_kernel.py:335-379 (matmul_kernel_only)
 *   a8w8 matmul(a, b)
 *       kernels/gemm/intra_wave/a8w8/matmul_kernel.py:437-470
 *       kernels/gemm/inter_wave/a8w8/matmul_kernel.py:343-388
 *   a4w4 matmul(a, b, a_scales, b_scales)
 *       kernels/gemm/intra_wave/a4w4/v1_sliceMN/matmul_kernel.py:696-742
 *       kernels/gemm/inter_wave/a4w4/v2_mfma32x32x64/matmul_kernel.py:614-668
 */
#ifndef B2G_H_
#define B2G_H_

#include <stddef.h>
#include <stdint.h>

#if defined(B2G_EXPORT) && defined(__GNUC__)
#define B2G_API __attribute__((visibility("default")))
#else
#define B2G_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- operand kinds (b2g_gemm_workspace_bytes `kind`) ---- */
#define B2G_KIND_F16 0    /* fp16 x fp16, kind::f16 */
#define B2G_KIND_BF16 1   /* bf16 x bf16, kind::f16 */
#define B2G_KIND_E5M2 2   /* e5m2 x e5m2, no scales, kind::f8f6f4 */
#define B2G_KIND_MXE5M2 3 /* e5m2 x e5m2 with E8M0 per 32 K, kind::mxf8f6f4 */
#define B2G_KIND_MXFP4 4  /* packed e2m1 x e2m1 with E8M0 per 32 K, kind::mxf4 */

/* ---- element types ---- */
#define B2G_DT_F16 0
#define B2G_DT_BF16 1
#define B2G_DT_F32 2

/* ---- argument errors (returned before any launch) ---- */
#define B2G_OK 0
#define B2G_EINVAL -1        /* bad kind / dtype / null pointer */
#define B2G_ESHAPE -2        /* M, N or K out of range or K not a multiple of the kind's unit */
#define B2G_EALIGN -3        /* pointer or row stride not 16-byte aligned */
#define B2G_ESTRIDE -4       /* operand not K-contiguous / overlapping rows */
#define B2G_EWORKSPACE -5    /* workspace missing or too small */
#define B2G_ETENSORMAP -6    /* the driver refused a TMA descriptor */
#define B2G_ENODEVICE -7     /* no sm_100 device current */
#define B2G_ECAPACITY -8     /* a size exceeds a fixed capacity of the entry point */

/* ---- device status word codes (set by kernels, read by the caller) ---- */
#define B2G_STATUS_TIMEOUT 0x1000 /* a bounded wait expired; low byte = wait site */
#define B2G_SITE_EMPTY 1          /* producer waiting for a free ring slot */
#define B2G_SITE_FULL 2           /* MMA waiting for a filled ring slot */
#define B2G_SITE_ACC_EMPTY 3      /* MMA waiting for a drained accumulator */
#define B2G_SITE_ACC_FULL 4       /* epilogue waiting for a finished accumulator */
#define B2G_SITE_OVERLAP 5        /* MMA waiting for the shared accumulator columns */
#define B2G_SITE_FLAG 6           /* stream-K owner waiting for a contributor */
#define B2G_SITE_SCALES 7         /* MMA waiting for scale factors copied into TMEM */
#define B2G_STATUS_SMEM_BASE 0x2000 /* kernel returned at entry: shared memory base misaligned */
#define B2G_STATUS_BAD_GROUPS 0x3000 /* grouped GEMM returned at entry: group offsets invalid */

/* Library ABI version (major * 100 + minor). */
B2G_API int b2g_version(void);

/* Human-readable text for a return code or a status word. */
B2G_API const char* b2g_strerror(int code);

/* Bytes of workspace the GEMM entry points need on the current device. */
B2G_API size_t b2g_gemm_workspace_bytes(int kind, int M, int N, int K);

/* Zero `bytes` of workspace on `stream` (once after allocation, and after a
 * nonzero status). */
B2G_API int b2g_workspace_reset(void* workspace, size_t bytes, void* stream);

/* a16w16: C = A * B^T, A/B fp16 or bf16 (`in_dtype`), C fp16 or bf16
 * (`out_dtype`). lda, ldb and ldc must be multiples of 8 elements (16-byte
 * rows); K itself is free. */
B2G_API int b2g_gemm_f16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                 int M, int N, int K, int in_dtype, int out_dtype, void* workspace,
                 size_t workspace_bytes, int* status, void* stream);

/* a8w8: C = A * B^T with A/B e5m2 bytes. With sfa == sfb == NULL the product
 * is unscaled (the reference's a8w8 contract, usually out_dtype = fp16).
 * Otherwise both scale tensors are E8M0 bytes of logical shape (rows, K/32)
 * with element strides (s0, s1) - any order, e.g. the reference's
 * M-contiguous (1, rows_pad) - and K must be a multiple of 32. Such scales are
 * relaid into the workspace by an extra launch on `stream`; strides (0, 0)
 * instead mean the pointer already holds the blocked layout written by
 * b2g_scales_to_blocked (16-byte aligned), and that tensor is used as is. */
B2G_API int b2g_gemm_f8(const void* A, int64_t lda, const void* B, int64_t ldb, const uint8_t* sfa,
                int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb, int64_t sfb_s0,
                int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K, int out_dtype,
                void* workspace, size_t workspace_bytes, int* status, void* stream);

/* a4w4: C = dequant(A) * dequant(B)^T with A (M, K/2) and B (N, K/2) packed
 * e2m1 bytes (low nibble = even k), lda/ldb in bytes, E8M0 scales as in
 * b2g_gemm_f8. K is the logical (unpacked) depth, a multiple of 32. */
B2G_API int b2g_gemm_mxf4(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                  const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1, const uint8_t* sfb,
                  int64_t sfb_s0, int64_t sfb_s1, void* C, int64_t ldc, int M, int N, int K,
                  int out_dtype, void* workspace, size_t workspace_bytes, int* status,
                  void* stream);

/* a4w4 without a workspace. This entry point has no counterpart in the
 * reference (whose launchers always let torch allocate); it serves callers
 * that cannot allocate device memory per call: a process that reserves HBM
 * for its own pool up front, or an FFI host with no caching allocator, for
 * which cudaMalloc / cudaFree around each call would fail or stall the device.
 * It computes what b2g_gemm_mxf4 computes, with the same arguments minus the
 * workspace, and allocates nothing: its scratch (stream-K flag words, split
 * partial sums, relaid scales) is a static device array of
 * B2G_NOALLOC_SCRATCH_BYTES inside the library, one copy per device.
 * - Limit: a call needs b2g_gemm_workspace_bytes(B2G_KIND_MXFP4, M, N, K)
 *   bytes (4096 x 4096 x 8192 needs about 19 MiB on a 148-SM B200); above
 *   the capacity it returns B2G_ECAPACITY and launches nothing.
 * - Zero state: the flag words must be zero when a GEMM launch starts. The
 *   array is zero when the library's module is loaded on a device, and each
 *   call also clears its flag words on `stream` (a memset, no allocation)
 *   before the launch; partial sums and relaid scales need no initial value.
 * - Set-up: the first call in each CUDA context, made while that context is
 *   current, looks up the scratch address (cudaGetSymbolAddress, which may
 *   load the module into the context) together with the set-up every entry
 *   point does once per device. The address is cached per device with the
 *   context's unique ID, so a call in another context (after
 *   cudaDeviceReset, or in a context a driver-API host made current) looks
 *   it up again rather than reuse an address of a destroyed context; the
 *   array's contents do not survive a context's destruction. Make the first
 *   call of each context before any stream capture begins.
 * - Races: one scratch per device means calls on the same device must not
 *   overlap on the GPU (use one stream, or order streams with events);
 *   overlapping calls corrupt each other's flags and partial sums. */
#define B2G_NOALLOC_SCRATCH_BYTES 33554432 /* 32 MiB per device */
B2G_API int b2g_gemm_mxf4_noalloc(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                                  const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1,
                                  const uint8_t* sfb, int64_t sfb_s0, int64_t sfb_s1, void* C,
                                  int64_t ldc, int M, int N, int K, int out_dtype, int* status,
                                  void* stream);

/* MoE grouped a4w4: rows [g[e], g[e+1]) of A and C belong to expert e and are
 * multiplied by expert e's weights, rows [e * N, (e + 1) * N) of B (`groups`
 * experts stacked, (groups * N) x K/2 packed bytes, scales (groups * N, K/32)).
 * `group_offsets` is a DEVICE array of groups + 1 int32: g[0] = 0,
 * g[groups] = M, non-decreasing, every entry a multiple of the tile height
 * (256 rows; 128 with B2G_OPT_PAIR = 0) - tokens sorted by expert with each
 * expert's segment padded (padding rows of C are written with the products of
 * whatever A holds there). Empty experts are allowed. N must be a multiple of
 * 128. Offsets that break these rules set B2G_STATUS_BAD_GROUPS and nothing is
 * written. Workspace: b2g_gemm_grouped_workspace_bytes. The reference has no
 * MoE kernel yet (its roadmap plans a 4-bit MoE GEMM); this is that row. */
B2G_API int b2g_gemm_mxf4_grouped(const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb,
                                  const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1,
                                  const uint8_t* sfb, int64_t sfb_s0, int64_t sfb_s1, void* C,
                                  int64_t ldc, const int32_t* group_offsets, int groups, int M,
                                  int N, int K, int out_dtype, void* workspace,
                                  size_t workspace_bytes, int* status, void* stream);
B2G_API size_t b2g_gemm_grouped_workspace_bytes(int M, int N, int K, int groups);

/* Prepared calls. Replaces the reference's PreparedKernel
 * (scripts/prepared_kernel.py:76-138: create() binds a launch's arguments once,
 * __call__ enters the compiled launcher directly), used by its kernel-only
 * timing (scripts/benchmark_prepared.py:255-260) to take launch overhead out of
 * back-to-back calls. b2g_prepare_gemm checks the arguments, plans the schedule
 * and encodes every tensor map of one GEMM call (the arguments of
 * b2g_gemm_f16 / _f8 / _mxf4, the operand kind given by `kind`; scales null for
 * the unscaled kinds, both set for the scaled ones); each b2g_prepared_run then
 * launches that call on `stream` with no further host work than the launch
 * itself. The plan keeps the pointers, the workspace, the status word and the
 * b2g_set_option values of the moment it was made: the buffers must stay
 * allocated (their contents may change between runs), and calls that share the
 * workspace must not overlap on the GPU. Runs must be made with the device
 * current that was current at preparation (else B2G_ENODEVICE). Free the
 * handle with b2g_prepared_free; *out is null when preparation fails. */
typedef struct b2g_prepared b2g_prepared;
B2G_API int b2g_prepare_gemm(int kind, const void* A, int64_t lda, const void* B, int64_t ldb,
                             const uint8_t* sfa, int64_t sfa_s0, int64_t sfa_s1,
                             const uint8_t* sfb, int64_t sfb_s0, int64_t sfb_s1, void* C,
                             int64_t ldc, int M, int N, int K, int out_dtype, void* workspace,
                             size_t workspace_bytes, int* status, b2g_prepared** out);
B2G_API int b2g_prepared_run(const b2g_prepared* prepared, void* stream);
B2G_API void b2g_prepared_free(b2g_prepared* prepared);

/* Attention forward, non-causal, with grouped-query heads:
 *   O[b, h] = softmax(Q[b, h] K[b, g]^T * sm_scale) V[b, g],  g = h / (heads_q / heads_k)
 * Replaces run_gluon_attention (kernels/attention/fmha_v4.py:761-790) and the
 * gluon_attn_fwd launch it makes; reference numerics kernels/attention/common.py:115
 * (sdpa_reference). `strides` holds 16 element strides, four per tensor in the
 * order q, k, v, o and, inside each, (batch, head, sequence, dim) -- the order of
 * get_strides_from_layout (common.py:79), so bhsd and bshd layouts are both plain
 * strides. The dim stride must be 1 and the other strides positive multiples of
 * 8 elements; q, k, v and o 16-byte aligned. head_dim 64 or 128; dtype B2G_DT_F16
 * or B2G_DT_BF16 for all four tensors; heads_q a multiple of heads_k; seqlen_k >= 1
 * and any seqlen_q >= 0 (unlike the reference, neither needs to be a multiple of
 * a block size, nor equal). `lse`, when not null, receives the natural-log
 * log-sum-exp of each row's scaled scores as float [batch][heads_q][seqlen_q]
 * (the reference keeps this in its internal M buffer). Accumulation is fp32;
 * P is rounded to the input type before the PV product. */
B2G_API int b2g_attention_fwd(const void* q, const void* k, const void* v, void* o,
                              const int64_t* strides, int batch, int heads_q, int heads_k,
                              int seqlen_q, int seqlen_k, int head_dim, int dtype,
                              float sm_scale, float* lse, int* status, void* stream);

/* Diagnostic, no counterpart in the reference: evaluates the FMHA's FMA-pipe
 * exponential (a cubic for 2^f, f in [-0.5, 0.5], plus an exponent-field add;
 * relative error <= 7.5e-5 for x in [-125.5, 8], inputs below -126 clamped) on
 * n device floats: y_scalar from the one-lane form, y_pair from the packed
 * two-lane form the softmax uses (elements 2j, 2j+1 together), y_exp2f from
 * CUDA's exp2f for comparison. Asynchronous on `stream`. */
B2G_API int b2g_selftest_poly_exp2(const float* x, float* y_scalar, float* y_pair,
                                   float* y_exp2f, int64_t n, void* stream);

/* Blocked E8M0 scale layout: for each 128-row block and each group of 4
 * k-blocks (4 scales), 512 bytes in which byte r0*16 + r1*4 + j holds the
 * scale of row 128*block + 32*r1 + r0 for k-block 4*group + j; blocks are
 * stored row-block major. Positions past the matrix hold 127. Static operands
 * (weights) can be converted once and passed with strides (0, 0). */
B2G_API size_t b2g_scales_blocked_bytes(int rows, int K);
B2G_API int b2g_scales_to_blocked(const uint8_t* src, int64_t s0, int64_t s1, int rows, int K,
                                  uint8_t* dst, void* stream);

/* Quantise fp32 `src` (rows x K, row stride ld) to MXFP4: per row and 32-K
 * block, scale exponent s = floor(log2(max|x|)) - 2 (E8M0 byte s + 127,
 * clamped to [0, 254]; an all-zero block gets byte 0; a block with a NaN or
 * an infinity gets byte 255 and zero codes), codes = E2M1 round-to-nearest-even
 * with saturation to +-6 of x * 2^-s, two per byte with the even k in the low
 * nibble. q is rows x K/2 bytes (row stride ldq); scales go to
 * scales[r * sc_s0 + j * sc_s1]. K must be a multiple of 32. */
B2G_API int b2g_quant_mxfp4(const float* src, int64_t ld, int rows, int K, uint8_t* q, int64_t ldq,
                    uint8_t* scales, int64_t sc_s0, int64_t sc_s1, void* stream);

/* Quantise fp32 `src` to e5m2 with given E8M0 scales: q = e5m2_rne(x * 2^-(e-127))
 * where e = scales[r * sc_s0 + (k/32) * sc_s1] (non-saturating, the rounding of
 * torch's float -> float8_e5m2 cast). K must be a multiple of 32. */
B2G_API int b2g_quant_mxe5m2(const float* src, int64_t ld, int rows, int K, const uint8_t* scales,
                     int64_t sc_s0, int64_t sc_s1, uint8_t* q, int64_t ldq, void* stream);

/* Elementwise cast of n contiguous values of `src_dtype` (B2G_DT_*) to e5m2,
 * round-to-nearest-even, non-saturating (torch's Tensor.to(float8_e5m2)). */
B2G_API int b2g_cast_e5m2(const void* src, int src_dtype, int64_t n, uint8_t* dst, void* stream);

/* ---- process-wide tuning and test options (b2g_set_option keys) ----
 * They change how later launches are planned; set them before computing a
 * workspace size and do not change them while GEMMs are in flight. */
#define B2G_OPT_PAIR 1        /* 1 (default): cta_group::2 CTA pairs (256 x 256 tiles);
                                 0: one CTA per tile (128 x 256) */
#define B2G_OPT_SK_MODE 2     /* tiles left after the full data-parallel waves:
                                 0: run as a partial wave; 1: stream-K (equal
                                 contiguous (tile, k) ranges per unit); 2: stream-K
                                 over the last full wave plus the partial one;
                                 3 (default): split each into two k-pieces
                                 (each piece reduces half of the tile), or, when
                                 the tiles are too short to split, run each as
                                 two half-width (N = 128) tiles if they fit;
                                 4: half-width tiles whenever they fit, else as 3 */
#define B2G_OPT_GROUP_M 3     /* raster group height in tiles (1: row-major); default 0
                                 picks it from the operand sizes: row-major when A and
                                 B fit in L2 together or B alone does, whole column
                                 strips when A alone does, else bands of tile rows
                                 holding about 32 MiB of A */
#define B2G_OPT_MIN_SK_ITERS 4 /* minimum k-iterations (256-byte stages) per stream-K unit
                                  or split piece (default 16) */
#define B2G_OPT_TIMEOUT_MS 5  /* bounded-wait deadline in ms (default 2000) */
#define B2G_OPT_INJECT_FLAG_TIMEOUT 6 /* test hook: stream-K owners wait for a flag
                                         value no contributor writes, so the wait
                                         expires and the status word is set */
#define B2G_OPT_MAX_UNITS 7   /* cap on persistent work units (0 = one per SM / pair) */
#define B2G_OPT_L2_PREFETCH 8 /* k-iterations of A/B the producer pulls into L2 ahead
                                 of its shared-memory loads (default 0 = off) */
#define B2G_OPT_SKINNY_MAX_M 9 /* fp16 / bf16 / unscaled e5m2 GEMMs with M up to this
                                  (default 128, at most 128; 0 = never) run the
                                  memory-bound swap-AB kernel: B's rows on the MMA's
                                  128-row side, A's rows on its N side */
#define B2G_OPT_SKINNY_SPLITS 10 /* K splits per 128-column tile in that kernel
                                    (default 0 = chosen from the SM count) */
#define B2G_OPT_SERPENTINE 11 /* 1 (default): the data-parallel tiles of odd waves run
                                 their K loop backwards, starting on the k-chunks the
                                 previous wave read last (still in L2); 0: every
                                 tile runs K forwards */

B2G_API int b2g_set_option(int key, int64_t value);
B2G_API int64_t b2g_get_option(int key);

/* Host-only view of the persistent schedule for a device with `num_sms` SMs
 * (no GPU needed). out[0..10] = {cta_group, tiles_m, tiles_n, k_iters, units,
 * dp_tiles, sk_units, launched_units, group_m, splits, half}; out_len >= 11. */
B2G_API int b2g_plan_query(int kind, int M, int N, int K, int num_sms, int32_t* out, int out_len);

/* Work items of one unit in execution order, 11 ints each: {tile, tm, tn,
 * k_begin, k_end, role (0 full, 1 split-tile owner, 2 contributor, 3 one of
 * the two pieces of a tile split in two), first_contrib (for role 3: the other
 * piece's unit), n_contrib, contrib_stride, nh (-1 whole tile, 0 / 1 first /
 * second 128 columns of a half-width tile), pair_half (role 3: the column
 * half this piece reduces, else -1)}. Returns the item count (items may be
 * NULL). */
B2G_API int b2g_plan_items(int kind, int M, int N, int K, int num_sms, int unit, int32_t* items,
                   int max_items);

#ifdef __cplusplus
}
#endif

#endif /* B2G_H_ */
