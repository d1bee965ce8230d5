/*
 * rouge-numerics-b200: C ABI of the B200 (sm_100a) implementation of the
 * rouge-numerics GEMM / convolution / quantization path.
 *
 * Two groups of entry points live here.
 *
 * 1. Drop-in symbols. Same names, argument order and meaning as the
 *    reference header software/rouge-numerics/include/rouge/numerics.h.
 *    They take HOST pointers (row-major, caller-owned), copy to the GPU,
 *    run the sm_100a kernels and copy back before returning. Invalid
 *    arguments keep the reference's behaviour: `void` entries return
 *    without writing, `int` quantizers return 0. A device failure (no GPU,
 *    launch error, a device-side wait that ran out) is not a silent CPU
 *    fallback: the call writes nothing further and the status is kept for
 *    rouge_b200_last_error().
 *
 * 2. rouge_b200_* extensions. DEVICE pointers, an explicit cudaStream_t
 *    passed as `void *stream` (NULL = legacy default stream), explicit
 *    layouts, fused scales and output types. Every one returns an int
 *    status (ROUGE_B200_OK == 0, negative on failure). Asynchronous with
 *    respect to the host unless stated otherwise.
 *
 * Nothing here falls back to the CPU: with no usable GPU every entry fails
 * with ROUGE_B200_ENODEV.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Types shared with the reference                                          */
/* ------------------------------------------------------------------------ */

/* A translation unit that also includes the reference header
 * rouge/numerics.h (which defines RougeGemmConfig and declares the drop-in
 * names) defines ROUGE_B200_WITH_REFERENCE_HEADER before including this
 * header; the shared type and the drop-in declarations are then taken from
 * the reference header. */
#ifndef ROUGE_B200_WITH_REFERENCE_HEADER

/* Replaces RougeGemmConfig, numerics.h:35-41. rouge_gemm_f32 reads it as a
 * tile-shape hint; the other GPU entries accept and ignore it. Garbage
 * values never cause out-of-bounds work (the reference normalises them at
 * gemm.cpp:254-275). */
typedef struct RougeGemmConfig {
  int tile_m;
  int tile_n;
  int tile_k;
  int unroll;
  int split_k;
} RougeGemmConfig;

/* Replaces RougeGemmProfile, numerics.h:44-48: the configuration a tuning
 * run chose, its GFLOP/s (2*M*N*K / best wall-clock of a whole call) and
 * the number of calls made. */
typedef struct RougeGemmProfile {
  RougeGemmConfig cfg;
  double gflops;
  long long iters;
} RougeGemmProfile;

#endif /* ROUGE_B200_WITH_REFERENCE_HEADER */

/* ------------------------------------------------------------------------ */
/* Status codes and library state                                           */
/* ------------------------------------------------------------------------ */

#define ROUGE_B200_OK 0
#define ROUGE_B200_EINVAL (-1)       /* bad pointer, size or enum value */
#define ROUGE_B200_ENODEV (-2)       /* no CUDA device / not an sm_100 part */
#define ROUGE_B200_ECUDA (-3)        /* a CUDA runtime call failed */
#define ROUGE_B200_EUNSUPPORTED (-4) /* shape or alignment outside the kernel's contract */
#define ROUGE_B200_ETIMEOUT (-5)     /* a bounded device-side wait ran out; results invalid */
#define ROUGE_B200_ENOMEM (-6)       /* device or pinned allocation failed */
#define ROUGE_B200_ETOOBIG (-7)      /* problem does not fit a fixed scratch area */

/* Status of the last failing call on this host thread (0 if none since the
 * last rouge_b200_clear_error). */
int rouge_b200_last_error(void);
void rouge_b200_clear_error(void);
const char *rouge_b200_status_string(int status);

/* Replaces rouge_gemm_isa_variant, numerics.h:331 (gemm.cpp:385-394).
 * Returns "sm_100a+tcgen05". */
const char *rouge_gemm_isa_variant(void);

/* Replaces rouge_gemm_default_config, numerics.h:307 (gemm.cpp:281-289).
 * Returns the reference's default {64,64,32,2,1}; the GPU path ignores it. */
RougeGemmConfig rouge_gemm_default_config(void);

/* 1 if a device usable by this library (compute capability 10.x) is
 * present, else 0. */
int rouge_b200_device_ok(void);

/* Caps the SMs the persistent kernels size their grids for (0 = all).
 * Leaving SMs free lets communication kernels on another stream overlap
 * (used by the sharded GEMM). Process-wide; returns the previous value. */
int rouge_b200_set_sm_budget(int sms);

/* GEMM / convolution tile shapes (no reference counterpart: the reference's
 * RougeGemmConfig blocking is a CPU cache blocking and is ignored).
 *   AUTO   256 x 256 tiles computed by 2-SM CTA pairs when 128 x 256 tiles
 *          would fill every SM, else 128 x 128 tiles on single CTAs
 *          (128 x 64 or 128 x 32 when those would fill at most half or a
 *          quarter of the SMs)
 *   SINGLE single-CTA tiles only (128 x 256 down to 128 x 32)
 *   PAIR   CTA-pair tiles only (256 x 256)
 * int8 results are identical in every mode (exact int32 accumulation).
 * Process-wide; returns the previous
 * mode, or ROUGE_B200_EINVAL for an unknown mode (nothing changed). */
#define ROUGE_B200_TILES_AUTO 0
#define ROUGE_B200_TILES_SINGLE 1
#define ROUGE_B200_TILES_PAIR 2
int rouge_b200_set_tile_mode(int mode);

/* Clock probe (a measurement aid; no reference counterpart). With `stamps`
 * non-NULL, every later GEMM / convolution launch on the current device
 * (the one current when this is called) has each of its first `ctas` CTAs
 * write four 64-bit words at stamps + 4 * cta: the SM cycle counter
 * (%clock64) and the global nanosecond timer (%globaltimer) when the CTA
 * starts, then both again when it ends. (w[2] - w[0]) / (w[3] - w[1]) is
 * the SM clock in GHz that the CTA ran at -- under the power cap often
 * well below the clock that nvidia-smi samples between launches.
 * `stamps`: 32 * ctas bytes of that device's memory; every launch
 * overwrites it, so read it after the launch of interest. NULL or ctas == 0
 * switches the probe off (the default). Process-wide; change it only while
 * no launch is being issued. Returns ROUGE_B200_OK, or ROUGE_B200_EINVAL
 * for ctas < 0. */
int rouge_b200_set_clock_probe(unsigned long long *stamps, int ctas);

/* Synchronises `stream`, then reads and clears the current device's error
 * word, which kernels set when a bounded device-side wait runs out.
 * Returns ROUGE_B200_OK or the failure (e.g. ROUGE_B200_ETIMEOUT). */
int rouge_b200_sync_status(void *stream);

/* Failure-detection check of the bounded device waits: launches one CTA on
 * `stream` that waits on an mbarrier nothing arrives at, bounded by
 * limit_ns (1e6..2e9 ns, else ROUGE_B200_EINVAL). The launch ends by itself
 * after about limit_ns; the next rouge_b200_sync_status(stream) returns
 * ROUGE_B200_ETIMEOUT and clears it, and the context stays usable.
 * Returns the launch status. */
int rouge_b200_check_wait_limit(unsigned long long limit_ns, void *stream);

/* Layout of the B operand of a GEMM. */
#define ROUGE_B200_B_KN 0 /* B[K][N] row-major (the reference's layout)  */
#define ROUGE_B200_B_NK 1 /* B[N][K] row-major (column-major B, K-major) */

/* Output element type of a GEMM / conv epilogue. */
#define ROUGE_B200_OUT_F32 0
#define ROUGE_B200_OUT_BF16 1 /* RNE, NaN -> 0x7fc0 (fp16.cpp:101-112) */
#define ROUGE_B200_OUT_I32 2  /* raw int32 accumulators (int8 GEMM only) */

/* ------------------------------------------------------------------------ */
/* Drop-in scalar format conversions (host functions, identical results)    */
/* ------------------------------------------------------------------------ */

/* Replace numerics.h:251-252 (fp8.cpp:42-106, 112-114). */
uint8_t rouge_quantize_e4m3(float f);
float rouge_dequantize_e4m3(uint8_t u);
/* Replace numerics.h:293-296 (fp16.cpp:31-121). */
uint16_t rouge_quantize_f16(float f);
float rouge_dequantize_f16(uint16_t u);
uint16_t rouge_quantize_bf16(float f);
float rouge_dequantize_bf16(uint16_t u);

/* ------------------------------------------------------------------------ */
/* Drop-in host-pointer entries (synchronous, GPU-backed)                   */
/* ------------------------------------------------------------------------ */

/* Replaces rouge_quantize_i8_tensor, numerics.h:144-145
 * (quant_int8.cpp:54-68). Returns 1 on success, 0 on bad arguments or a
 * device failure. */
int rouge_quantize_i8_tensor(const float *x, int n, float *scale_out, int8_t *out);

/* Replaces rouge_quantize_i8_channel, numerics.h:146-147
 * (quant_int8.cpp:72-90). One symmetric scale per row of x[rows][cols]. */
int rouge_quantize_i8_channel(const float *x, int rows, int cols, float *scales,
                              int8_t *out);

/* Replace rouge_dequantize_i8_tensor / _channel, numerics.h:150-153
 * (quant_int8.cpp:145-160). */
void rouge_dequantize_i8_tensor(const int8_t *q, int n, float scale, float *out);
void rouge_dequantize_i8_channel(const int8_t *q, int rows, int cols,
                                 const float *scales, float *out);

/* Replace rouge_quantize_i8_group / rouge_dequantize_i8_group,
 * numerics.h:148-149,154-156 (quant_int8.cpp:94-142, 162-179): asymmetric
 * 0..255 codes per group of cols/groups consecutive elements, scale and
 * zero point per group (scales/zeros[rows*groups]). cols % groups != 0 is
 * refused as in the reference. */
int rouge_quantize_i8_group(const float *x, int rows, int cols, int groups, float *scales,
                            uint8_t *zeros, uint8_t *out);
void rouge_dequantize_i8_group(const uint8_t *q, int rows, int cols, int groups,
                               const float *scales, const uint8_t *zeros, float *out);

/* Replaces rouge_gemm_i8, numerics.h:160-162 (quant_int8.cpp:189-211).
 * A[M][K] s8, B[K][N] s8 row-major; exact int32 accumulation, then
 * C[m][n] = ((float)acc * sa) * sb. */
void rouge_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B,
                   const float *scales_a, int a_rows, const float *scales_b,
                   int b_cols, float *C);

/* No counterpart in the reference. rouge_gemm_i8 (same arguments, same
 * results) for callers that cannot let the library allocate device memory,
 * such as a process that reserves the GPU's memory for its own allocator at
 * start-up or a loop that must not allocate once it runs. Host pointers,
 * synchronous. Stages operands, scales and output in a fixed 64 MiB device
 * array (one per GPU, held until exit) instead of an allocated workspace:
 * M*Kp + Kp*Np + 4*(M+N) + 4*M*N bytes (Kp, Np = K, N rounded up to 16, plus
 * alignment) must fit, otherwise ROUGE_B200_ETOOBIG and C is not written.
 * The first call on a device does a one-time set-up (the device address of
 * the array); make it before any stream capture. Memory is still reserved
 * once, by the CUDA driver, outside the calls that follow: the array when
 * the driver loads its module and the GEMM kernel's code when it is first
 * launched, which under CUDA's default lazy loading is during the first
 * call on a device (and the first call of a shape that needs another kernel
 * variant: single-CTA tiles for small problems, CTA pairs for large ones).
 * Make one call of each shape class before reserving the GPU's memory for
 * another allocator or entering a loop that must not allocate (or set
 * CUDA_MODULE_LOADING=EAGER). Calls share the array:
 * they are serialised by a lock and synchronise before returning; GPU work
 * that overlapped a call's use of the array would race with it. Returns a
 * status (ROUGE_B200_OK on success). */
int rouge_gemm_i8_noalloc(int M, int N, int K, const int8_t *A, const int8_t *B,
                          const float *scales_a, int a_rows, const float *scales_b,
                          int b_cols, float *C);

/* Replaces rouge_gemm_f32, numerics.h:54-55 (gemm.cpp:291-383).
 * C[M][N] = A[M][K] * B[K][N], all f32 row-major; C is overwritten, not
 * accumulated. Computed on tf32 tensor cores with split operands (hi + lo,
 * three products per element pair: f32 accuracy). cfg selects the tile
 * shape: tile_m >= 256 CTA pairs on 256 x 256 tiles; tile_m >= 128 one CTA
 * per 128 x 256 tile (tile_n >= 256) or 128 x 128 tile; otherwise, or NULL,
 * the library's choice. Every shape gives identical results. Sizes <= 0 or
 * NULL pointers: no-op. */
void rouge_gemm_f32(int M, int N, int K, const float *A, const float *B, float *C,
                    const RougeGemmConfig *cfg);

/* Replace the tuner, numerics.h:311-324 (autotune.cpp:32-127).
 * rouge_gemm_candidate_count / rouge_gemm_candidate: the candidate
 * configurations (the default one and the three tile shapes above); an
 * index out of range gives rouge_gemm_default_config().
 * rouge_gemm_flops_per_sec: one warm-up call of rouge_gemm_f32 with cfg,
 * then 2*M*N*K / the best wall-clock of three calls, in GFLOP/s (host
 * copies included: the time a caller of the drop-in waits); the product is
 * left in C. 0.0 on invalid arguments or a device failure.
 * rouge_gemm_tuned: every candidate timed the same way (each call counted in
 * iters), then the best one's result computed again into C; its config and
 * GFLOP/s are returned. Invalid arguments: the default config, 0 GFLOP/s,
 * 0 iterations, C untouched. */
int rouge_gemm_candidate_count(void);
RougeGemmConfig rouge_gemm_candidate(int index);
double rouge_gemm_flops_per_sec(int M, int N, int K, const float *A, const float *B, float *C,
                                const RougeGemmConfig *cfg);
RougeGemmProfile rouge_gemm_tuned(int M, int N, int K, const float *A, const float *B, float *C);

/* Replaces rouge_gemm_e4m3, numerics.h:68-69 (fp8.cpp:116-124).
 * A[M][K], B[K][N] OCP E4M3 codes; C f32 = dec(A) * dec(B), f32 accumulate. */
void rouge_gemm_e4m3(int M, int N, int K, const uint8_t *A, const uint8_t *B,
                     float *C, const RougeGemmConfig *cfg);

/* Replace rouge_gemm_f16 / rouge_gemm_bf16, numerics.h:301-304
 * (fp16.cpp:123-141). A[M][K], B[K][N] half / bf16 codes; C f32. */
void rouge_gemm_f16(int M, int N, int K, const uint16_t *A, const uint16_t *B,
                    float *C, const RougeGemmConfig *cfg);
void rouge_gemm_bf16(int M, int N, int K, const uint16_t *A, const uint16_t *B,
                     float *C, const RougeGemmConfig *cfg);

/* Replace rouge_conv2d_f32, numerics.h:76-79 (conv.cpp:26-66), and
 * rouge_conv_implicit_f32, numerics.h:106-109 (conv_implicit.cpp:24-79):
 * Y[N][Cout][OH][OW] = conv(X[N][Cin][H][W], Wt[Cout][Cin][KH][KW]) + bias,
 * all NCHW f32, OH = (H + 2*pad - KH)/stride + 1; bias may be NULL; NULL
 * X/Wt/Y or invalid sizes -> no-op. Computed on tf32 tensor cores with
 * split operands (hi + lo, three products) for f32 accuracy. Not
 * expressible by the im2col tensor map (no-op, status
 * ROUGE_B200_EUNSUPPORTED): pad > 128, stride > 8, KH or KW above 256, above
 * pad + 129 or above the padded input. cfg is accepted and ignored. */
void rouge_conv2d_f32(int N, int Cin, int H, int W, int Cout, int KH, int KW,
                      int stride, int pad, const float *X, const float *Wt,
                      const float *bias, float *Y, const RougeGemmConfig *cfg);
void rouge_conv_implicit_f32(int N, int Cin, int H, int W, int Cout, int KH,
                             int KW, int stride, int pad, const float *X,
                             const float *Wt, const float *bias, float *Y,
                             const RougeGemmConfig *cfg);

/* ------------------------------------------------------------------------ */
/* rouge_b200_* device-pointer extensions                                   */
/* ------------------------------------------------------------------------ */

/* Per-row symmetric int8 quantization of x[rows][cols] (f32, device).
 * Bit-exact with quant_int8.cpp:72-90: amax in double, scale =
 * (float)(amax/127.0) or 1.0f for an all-zero row, code =
 * clamp(rne((double)x * (1.0/(double)scale)), -127, 127).
 * scales[rows] f32, out[rows][cols] s8. Requires cols % 4 == 0 and 16-byte
 * aligned x, 4-byte aligned out. */
int rouge_b200_quantize_i8_rows(const float *x, int rows, int cols, float *scales,
                                int8_t *out, void *stream);

/* out[r][c] = (float)q[r][c] * scales[r]   (quant_int8.cpp:151-160).
 * scales == NULL with scale != 0 uses one scale for the whole tensor
 * (quant_int8.cpp:145-149). */
int rouge_b200_dequantize_i8_rows(const int8_t *q, int rows, int cols,
                                  const float *scales, float scale, float *out,
                                  void *stream);

/* Device-pointer per-group quantization / dequantization (same semantics
 * as rouge_quantize_i8_group / rouge_dequantize_i8_group). */
int rouge_b200_quantize_i8_group(const float *x, int rows, int cols, int groups, float *scales,
                                 uint8_t *zeros, uint8_t *out, void *stream);
int rouge_b200_dequantize_i8_group(const uint8_t *q, int rows, int cols, int groups,
                                   const float *scales, const uint8_t *zeros, float *out,
                                   void *stream);

/* Per-tensor absolute maximum of x[n] (f32, device) into *amax (device f32).
 * NaNs are ignored, as std::fabs/operator> ignore them on the host. */
int rouge_b200_absmax_f32(const float *x, size_t n, float *amax, void *stream);

/* E4M3 codes of x[n] under a per-tensor scale:
 *   s = amax / 448.0f (1.0f when amax == 0), out[i] = e4m3(x[i] / s),
 * with the encoder of fp8.cpp:75-106 (RNE, satfinite, |v| < 2^-10 -> +0).
 * amax is read from device memory (as written by rouge_b200_absmax_f32);
 * s is written to *scale_out (device f32) when scale_out != NULL. */
int rouge_b200_quantize_e4m3_scaled(const float *x, size_t n, const float *amax,
                                    float *scale_out, uint8_t *out, void *stream);

/* absmax + scaled encode in one call (two kernels, no host round trip).
 * *amax_out (device) receives the tensor's absolute maximum, *scale_out
 * (device, may be NULL, must differ from amax_out) receives s. */
int rouge_b200_quantize_e4m3_tensor(const float *x, size_t n, float *amax_out,
                                    float *scale_out, uint8_t *out, void *stream);

/* Elementwise f32 <-> narrow conversions on device (fp16.cpp:61-112,
 * fp8.cpp:42-106). */
int rouge_b200_convert_f32_to_f16(const float *x, size_t n, uint16_t *out, void *stream);
int rouge_b200_convert_f32_to_bf16(const float *x, size_t n, uint16_t *out, void *stream);
int rouge_b200_convert_e4m3_to_f32(const uint8_t *x, size_t n, float *out, void *stream);

/* int8 GEMM on tcgen05 (kind::i8), exact int32 accumulation in TMEM.
 * A[M][K] s8 row-major; B per b_layout (ROUGE_B200_B_KN or _NK).
 * Epilogue (fused): out_type F32:  C = ((float)acc * sa) * sb
 *                   out_type BF16: bf16_rne(((float)acc * sa) * sb)
 *                   out_type I32:  C = acc (scales ignored, may be NULL)
 * sa = a_rows ? scales_a[m] : scales_a[0]; sb = b_cols ? scales_b[n] : scales_b[0].
 * ldc = row pitch of C in elements (>= N). Requires K % 16 == 0 and
 * (for B_KN) N % 16 == 0, 16-byte aligned A/B. */
int rouge_b200_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B,
                       int b_layout, const float *scales_a, int a_rows,
                       const float *scales_b, int b_cols, void *C, int ldc,
                       int out_type, void *stream);

/* The W8A8 linear step -- rouge_quantize_i8_channel of the activations
 * followed by rouge_gemm_i8 with per-row and per-column scales
 * (quant_int8.cpp:72-90, 189-211) -- as one device call:
 *   Aq[M][K], sa[M] = rouge_b200_quantize_i8_rows(X[M][K])
 *   C = rouge_b200_gemm_i8(Aq, Wq, ROUGE_B200_B_NK, sa, 1, sw, 1, out_type)
 * with identical results. Wq[N][K] holds the weights' int8 codes (one row
 * per output channel), sw[N] their scales. When K <= 4096 and the problem
 * takes CTA-pair tiles the quantization runs inside the GEMM launch (the
 * first round of tiles starts as soon as its rows are coded; the other
 * rows are coded while the tiles run); otherwise two launches.
 * `workspace`: rouge_b200_w8a8_workspace_bytes(M) bytes of device memory,
 * 4-byte aligned, zeroed before its first use; every call leaves it zeroed.
 * Calls that may run at the same time need separate workspaces.
 * Alignment: X 16 bytes, K % 16 == 0, plus those of rouge_b200_gemm_i8. */
size_t rouge_b200_w8a8_workspace_bytes(int M);
int rouge_b200_w8a8_linear(int M, int N, int K, const float *X, const int8_t *Wq,
                           const float *sw, int8_t *Aq, float *sa, void *C, int ldc,
                           int out_type, void *workspace, void *stream);

/* Column-major BLAS GEMM (the semantics of cublasSgemm / cublasGemmEx; the
 * reference implements them on its CPU GEMM, cublas_shim.cpp:36-65,199-211):
 *   C (m x n, column-major, ldc) = alpha * op(A) * op(B) + beta * C
 * transa / transb: 0 = N, 1 = T. Operand type ab_type (A and B alike) and
 * output c_type:
 *   F32  -> F32  tf32 tensor cores with split operands (3xTF32: hi*hi +
 *                hi*lo + lo*hi), f32-accurate
 *   F16 / BF16 / E4M3 -> F32   f32 accumulation
 *   I8   -> I32  exact int32 (alpha must be 1, beta 0)
 * The operands are packed (transposed as needed) into `workspace`
 * (256-byte aligned, at least rouge_b200_gemm_colmajor_workspace bytes;
 * ROUGE_B200_ETOOBIG otherwise). beta == 0 never reads C. Asynchronous on
 * `stream`. Device pointers. */
#define ROUGE_B200_T_F32 0
#define ROUGE_B200_T_F16 1
#define ROUGE_B200_T_BF16 2
#define ROUGE_B200_T_E4M3 3
#define ROUGE_B200_T_I8 4
#define ROUGE_B200_T_I32 5
size_t rouge_b200_gemm_colmajor_workspace(int ab_type, int m, int n, int k);
int rouge_b200_gemm_colmajor(int transa, int transb, int m, int n, int k, int ab_type,
                             float alpha, const void *A, int lda, const void *B, int ldb,
                             float beta, void *C, int c_type, int ldc, void *workspace,
                             size_t workspace_bytes, void *stream);

/* rouge_b200_gemm_i8 with its output broadcast to every GPU of a sharded
 * job (no reference counterpart: the reference has no multi-GPU code; this
 * is the all-gather of the N-sharded W8A8 GEMM fused into the epilogue).
 * Each output element (m, n) of this rank's M x N block is written to
 * element (m, col_off + n) of every rank's [M][ldc] output:
 *   C_mc != NULL: one multimem store per 16 bytes to the NVLink multicast
 *                 address C_mc (the switch writes every bound GPU's copy);
 *   C_mc == NULL: one store per entry of C_peers[0..npeers) (1..8 device
 *                 pointers, this GPU's own output included).
 * Requires N % 8 == 0, 16-byte row pitch and column offset, K % 16 == 0.
 * The kernel ends with a system-scope fence; the caller synchronises the
 * ranks (a device-side barrier) before anyone reads the output. */
int rouge_b200_gemm_i8_bcast(int M, int N, int K, const int8_t *A, const int8_t *B,
                             int b_layout, const float *scales_a, int a_rows,
                             const float *scales_b, int b_cols, void *C_mc,
                             void *const *C_peers, int npeers, long long ldc, int col_off,
                             int out_type, void *stream);

/* E4M3 GEMM on tcgen05 (kind::f8f6f4), f32 accumulation in TMEM.
 * C = acc * (scale_a[0] * scale_b[0]) when the scale pointers (device f32
 * scalars) are non-NULL, else acc. out_type F32 or BF16. Same layout and
 * alignment rules as rouge_b200_gemm_i8. */
int rouge_b200_gemm_e4m3(int M, int N, int K, const uint8_t *A, const uint8_t *B,
                         int b_layout, const float *scale_a, const float *scale_b,
                         void *C, int ldc, int out_type, void *stream);

/* f16 / bf16 GEMM on tcgen05 (kind::f16), f32 accumulation in TMEM.
 * is_bf16 selects the input format. C f32 (out_type F32) or bf16.
 * Requires K % 8 == 0 and (for B_KN) N % 8 == 0. */
int rouge_b200_gemm_f16(int M, int N, int K, const uint16_t *A, const uint16_t *B,
                        int b_layout, int is_bf16, void *C, int ldc, int out_type,
                        void *stream);

/* Implicit-GEMM 2-D convolution on tcgen05 (kind::f16), the B200 form of
 * rouge_conv2d_f32 / rouge_conv_implicit_f32 (numerics.h:76-79,106-109;
 * conv.cpp:26-66): cross-correlation with symmetric stride and zero
 * padding, OH = (H + 2*pad - KH)/stride + 1, then + bias[co].
 *   X  [N][H][W][Cin]      f16 (is_bf16 = 0) or bf16 codes, NHWC
 *   Wt [Cout][KH][KW][Cin] same type
 *   bias [Cout] f32 or NULL; Y [N][OH][OW][Cout] f32, f32 accumulation.
 * Requires Cin % 64 == 0, Cout % 4 == 0, 16-byte aligned X / Wt, an input
 * of at least 128 KB, KH, KW <= 256, pad <= 128, stride <= 8. */
int rouge_b200_conv2d_nhwc_f16(int N, int H, int W, int Cin, int Cout, int KH, int KW,
                               int stride, int pad, const uint16_t *X, const uint16_t *Wt,
                               const float *bias, float *Y, int is_bf16, void *stream);

/* ------------------------------------------------------------------------ */
/* Narrow formats and MX / NVFP4 block quantization (narrow.cpp)            */
/* ------------------------------------------------------------------------ */
/* Replace numerics.h:257-264 (narrow.cpp:166-198): single-value codecs,
 * codes in the low bits (e2m1: 4-bit field, sign in bit 3). */
uint8_t rouge_quantize_e5m2(float f);
float rouge_dequantize_e5m2(uint8_t u);
uint8_t rouge_quantize_e3m2(float f);
float rouge_dequantize_e3m2(uint8_t u);
uint8_t rouge_quantize_e2m3(float f);
float rouge_dequantize_e2m3(uint8_t u);
uint8_t rouge_quantize_e2m1(float f);
float rouge_dequantize_e2m1(uint8_t u);

/* Replace numerics.h:278-289 (narrow.cpp:200-331), host pointers,
 * synchronous: MXFP8 (elem_bytes 1: e4m3, 2: e5m2) and MXFP4 (e2m1) in
 * blocks of 32 with E8M0 scales, NVFP4 (e2m1) in blocks of 16 with e4m3
 * block scales and a global scale. Return the block count (0 and nothing
 * written on invalid arguments or a device failure). */
int rouge_mx_quantize_f32(const float *x, int n, int elem_bytes, uint8_t *out,
                          uint8_t *scale_out);
int rouge_mx_quantize_f32_e2m1(const float *x, int n, uint8_t *out, uint8_t *scale_out);
int rouge_nvfp4_quantize_f32(const float *x, int n, float global_scale, uint8_t *out,
                             uint8_t *scale_out);
void rouge_mx_dequantize_f32(const uint8_t *in, const uint8_t *scales, int n, int elem_bytes,
                             float *out);
void rouge_mx_dequantize_f32_e2m1(const uint8_t *in, const uint8_t *scales, int n, float *out);

/* Device-pointer forms (asynchronous on `stream`); fmt ROUGE_B200_FMT_*. */
#define ROUGE_B200_FMT_E4M3 0
#define ROUGE_B200_FMT_E5M2 1
#define ROUGE_B200_FMT_E2M1 4
int rouge_b200_mx_quantize(const float *x, size_t n, int fmt, uint8_t *codes, uint8_t *scales,
                           void *stream);
int rouge_b200_nvfp4_quantize(const float *x, size_t n, float global_scale, uint8_t *codes,
                              uint8_t *scales, void *stream);
int rouge_b200_mx_dequantize(const uint8_t *codes, const uint8_t *scales, size_t n, int fmt,
                             float *out, void *stream);

/* Block-scaled MXFP8 GEMM on tcgen05 (kind::mxf8f6f4.block_scale; no
 * reference counterpart: the reference has the formats but no GEMM on
 * them). C[M][N] (f32 or bf16, row pitch ldc) = sum_k A'[m][k] B'[n][k]
 * with A' = decode(A) * 2^(sfa - 127) per 32-element K-block of each row,
 * likewise B'; f32 accumulation. A [M][K] and B [N][K] are e4m3
 * (ROUGE_B200_FMT_E4M3) or e5m2 codes, K-major, K % 32 == 0, 16-byte
 * aligned; sfa / sfb are their E8M0 scales in the tensor-core atom layout
 * made by rouge_b200_mx_scale_atoms from the block quantizer's [rows][K/32]
 * scales. */
size_t rouge_b200_mx_scale_atoms_bytes(int rows, int K);
int rouge_b200_mx_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                              void *stream);
int rouge_b200_gemm_mx(int M, int N, int K, const uint8_t *A, int fmt_a, const uint8_t *sfa,
                       const uint8_t *B, int fmt_b, const uint8_t *sfb, void *C, int ldc,
                       int out_type, void *stream);

/* Block-scaled NVFP4 GEMM (kind::mxf4nvf4.block_scale.scale_vec::4X):
 * C[M][N] = gs_a * gs_b * sum_k (a * sa)(b * sb), a / b the e2m1 codes of
 * rouge_nvfp4_quantize packed two per byte by rouge_b200_fp4_pack (A
 * [M][K/2], B [N][K/2] bytes, K % 32 == 0), sa / sb their UE4M3 block
 * scales (one per 16 K, [rows][K/16]) laid out by
 * rouge_b200_nvfp4_scale_atoms, gs_a / gs_b device pointers to the global
 * scales (both null: 1). f32 accumulation; f32 or bf16 output. */
size_t rouge_b200_nvfp4_scale_atoms_bytes(int rows, int K);
int rouge_b200_nvfp4_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                                 void *stream);
int rouge_b200_fp4_pack(const uint8_t *codes, size_t n, uint8_t *packed, void *stream);
/* rouge_b200_nvfp4_quantize with the codes written packed (n % 16 == 0,
 * 16-byte aligned x, 8-byte aligned packed[n/2]): the GEMM's operand in one
 * pass. */
int rouge_b200_nvfp4_quantize_packed(const float *x, size_t n, float global_scale,
                                     uint8_t *packed, uint8_t *scales, void *stream);
int rouge_b200_gemm_nvfp4(int M, int N, int K, const uint8_t *A, const uint8_t *sfa,
                          const float *gs_a, const uint8_t *B, const uint8_t *sfb,
                          const float *gs_b, void *C, int ldc, int out_type, void *stream);

/* Block-scaled MXFP4 GEMM (kind::mxf4.block_scale.scale_vec::2X): the e2m1
 * codes of the MXFP4 quantizer (rouge_b200_mx_quantize, ROUGE_B200_FMT_E2M1)
 * packed by rouge_b200_fp4_pack, their E8M0 scales (one per 32 K,
 * [rows][K/32]) laid out by rouge_b200_mxfp4_scale_atoms; otherwise as
 * rouge_b200_gemm_nvfp4 without global scales. */
size_t rouge_b200_mxfp4_scale_atoms_bytes(int rows, int K);
int rouge_b200_mxfp4_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                                 void *stream);
int rouge_b200_gemm_mxfp4(int M, int N, int K, const uint8_t *A, const uint8_t *sfa,
                          const uint8_t *B, const uint8_t *sfb, void *C, int ldc, int out_type,
                          void *stream);

/* ------------------------------------------------------------------------ */
/* Attention and the transformer block (the GEMM's in-library consumers)     */
/* ------------------------------------------------------------------------ */
/* Replace numerics.h:125-137,173-183 (attention.cpp:27-88,
 * attention_gqa.cpp:52-269, transformer.cpp:33-161), host pointers,
 * synchronous, same layouts: Q [Hq][S][Dh], K / V [Hkv][Skv][Dh] (f32 or
 * e4m3 codes with per-head scales), O [Hq][S][Dh]; scale <= 0 means
 * 1/sqrt(Dh); causal masks t > s + kv_off, window > 0 masks
 * t < s + kv_off - window + 1; fully masked rows give 0. Scores and the
 * weighted sums run on the tf32 tensor cores with split operands
 * (f32-accurate); softmax per row on the device. */
void rouge_attention_f32(int S, int Skv, int D, const float *Q, const float *K, const float *V,
                         float *O, float scale, int causal, int kv_off);
void rouge_attention_gqa(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q, const float *K,
                         const float *V, float *O, float scale, int causal, int window,
                         int kv_off);
void rouge_attention_gqa_fp8kv(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q,
                               const uint8_t *Kq, const uint8_t *Vq, const float *scales_k,
                               const float *scales_v, float *O, float scale, int causal,
                               int window, int kv_off);
void rouge_rmsnorm(const float *x, int n, const float *w, float eps, float *out);
void rouge_rope(float *x, int heads, int head_dim, int pos, float theta);
void rouge_swiglu(const float *gate, const float *up, int n, float *out);
void rouge_transformer_block(int S, int D, int Hq, int Hkv, int Dq, int Dk, const float *x,
                             const float *wrms1, const float *wq, const float *wk, const float *wv,
                             const float *wo, const float *wrms2, const float *wgate,
                             const float *wup, const float *wdown, int Dff, float rope_theta,
                             float rms_eps, float *out);

/* Device-pointer forms (asynchronous on `stream`; workspace 256-byte
 * aligned, at least the *_workspace bytes, else ROUGE_B200_ETOOBIG).
 * Attention: f32 K / V, or (Kq != NULL) e4m3 K / V with device scales. */
size_t rouge_b200_attention_workspace(int S, int Skv, int Dh, int Hq, int Hkv, int fp8_kv);
int rouge_b200_attention_gqa(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q,
                             const float *K, const float *V, const uint8_t *Kq, const uint8_t *Vq,
                             const float *scales_k, const float *scales_v, float *O, float scale,
                             int causal, int window, int kv_off, void *workspace,
                             size_t workspace_bytes, void *stream);
size_t rouge_b200_transformer_block_workspace(int S, int D, int Hq, int Hkv, int Dq, int Dff);
int rouge_b200_transformer_block(int S, int D, int Hq, int Hkv, int Dq, int Dk, const float *x,
                                 const float *wrms1, const float *wq, const float *wk,
                                 const float *wv, const float *wo, const float *wrms2,
                                 const float *wgate, const float *wup, const float *wdown, int Dff,
                                 float rope_theta, float rms_eps, float *out, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* Convolution forward with cuDNN's semantics (the operation the reference
 * runs in cudnnConvolutionForward, cudnn_shim.cpp:188-232, on its CPU
 * conv): Y = alpha * conv(X, Wt) + beta * Y, cross-correlation, symmetric
 * stride and zero padding, OH = (H + 2*pad - KH)/stride + 1. X, Wt and Y
 * are device arrays of one element type `type`: ROUGE_B200_T_F32 (tf32
 * tensor cores with split operands, f32-accurate), ROUGE_B200_T_F16 or
 * ROUGE_B200_T_BF16 (f32 accumulation, result rounded to nearest even).
 * Layouts: X [N][Cin][H][W] (NCHW) or [N][H][W][Cin] (NHWC); Wt
 * [Cout][Cin][KH][KW] (NCHW) or [Cout][KH][KW][Cin] (NHWC); Y likewise.
 * Y is read only when beta != 0. Workspace: at least
 * rouge_b200_conv2d_forward_workspace(...) bytes, 256-byte aligned (0 for
 * 16-bit NHWC data with Cin % 64 == 0, Cout % 8 == 0, X of at least
 * 128 KB and 16-byte aligned pointers: the kernel then reads X and Wt as
 * they are and writes Y from its epilogue); too little -> ROUGE_B200_ETOOBIG.
 * Limits (EUNSUPPORTED): pad <= 128, KH, KW <= min(256, pad + 129),
 * stride <= 8. Asynchronous on `stream`. */
#define ROUGE_B200_NCHW 0
#define ROUGE_B200_NHWC 1
size_t rouge_b200_conv2d_forward_workspace(int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                           int stride, int pad, int type, int x_layout,
                                           int w_layout, int y_layout);
int rouge_b200_conv2d_forward(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride,
                              int pad, int type, float alpha, const void *X, int x_layout,
                              const void *Wt, int w_layout, float beta, void *Y, int y_layout,
                              void *workspace, size_t workspace_bytes, void *stream);

/* N-sharded GEMM, layout step after the all-gather:
 * rank r of g owns output columns [r*ns, (r+1)*ns); shards gathered in
 * bands of R rows arrive as src[M/R][g][R][ns]; this writes them to
 * dst[M][ldd] row-major (columns >= N dropped). esize = 1, 2 or 4 bytes;
 * ns, N, ldd multiples of 16/esize; M % R == 0; 16-byte aligned buffers.
 * No reference counterpart: the reference has no multi-GPU code. */
int rouge_b200_unshard_columns(const void *src, void *dst, int M, int N, int g, int ns, int R,
                               int ldd, int esize, void *stream);

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs (host, multi-threaded)                           */
/* ------------------------------------------------------------------------ */
/* Counterparts of the reference's splitmix64 + Box-Muller generator
 * (rouge_rng_*, numerics.h:237-246): counter-based splitmix64, so a fill is
 * identical for any thread count. Return 0 (count for _outliers) or -1. */
int rouge_b200_synth_uniform(uint64_t seed, size_t n, float lo, float hi, float *out);
int rouge_b200_synth_normal(uint64_t seed, size_t n, float mean, float stddev, float *out);
long long rouge_b200_synth_outliers(uint64_t seed, size_t n, float frac, float mult, float *x);
/* The same streams from element `offset` on (offset even for _normal), so
 * a rank can generate only its own shard of a tensor. */
int rouge_b200_synth_normal_at(uint64_t seed, size_t offset, size_t n, float mean, float stddev,
                               float *out);
long long rouge_b200_synth_outliers_at(uint64_t seed, size_t offset, size_t n, float frac,
                                       float mult, float *x);

#ifdef __cplusplus
} /* extern "C" */
#endif
