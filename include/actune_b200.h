/*
 * actune_b200 -- C ABI of the B200 (sm_100a) group-64 packed-integer linear.
 *
 * Plain pointers and sizes only.  Every pointer argument is a device pointer on
 * the CUDA device that is current on the calling thread, unless noted.  The
 * caller owns every buffer; no function allocates device memory.  The functions
 * other than actune_grouped_linear_noalloc can be captured into a CUDA graph
 * (the first call of each kernel on a device also sets its shared-memory
 * attribute, so make one call before capturing).
 * `stream` is a cudaStream_t (NULL = legacy default stream).  All functions are
 * asynchronous with respect to the host and return an actune_status; a kernel
 * that fails on the device records the failure in a device word read by
 * actune_device_error() instead of hanging.
 *
 * Bit layouts follow the reference project (paths relative to its root):
 *   packed activations  uint8 [M, K*A/8], element k of a row at byte k*A/8,
 *                       bits (k mod 8/A)*A, little-endian    (actune/kernels/grouped.py:55-71)
 *   activation scales   float [M, K/64]                      (grouped.py:131)
 *   packed weights      uint8 [N, K*W/8], same bit order     (grouped.py:108-111, 121)
 *   weight scales       float [N] (one per output row)       (actune/kernels/quantizers.py:23-94)
 *   bias                [N] bf16/f16/f32, optional           (grouped.py:123-125)
 *   output              [M, N] bf16/f16/f32                  (grouped.py:138, grouped_native.cu:106)
 * Constraints: W, A in {2, 4, 8}; K a positive multiple of 64; 0 <= M, N < 2^31;
 * packed operands 16-byte aligned.
 */
#ifndef ACTUNE_B200_H
#define ACTUNE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ACTUNE_ABI_VERSION 1

typedef enum actune_status {
  ACTUNE_OK = 0,
  ACTUNE_ERR_INVALID_VALUE = 1,  /* shape, bit width, dtype code or null pointer rejected */
  ACTUNE_ERR_MISALIGNED = 2,     /* a pointer violates its alignment requirement */
  ACTUNE_ERR_DEVICE = 3,         /* the current device is not an sm_100 (B200-class) GPU */
  ACTUNE_ERR_CUDA = 4,           /* a CUDA runtime or driver call failed (launch, attribute, tensor map) */
  ACTUNE_ERR_WORKSPACE = 5       /* the workspace passed is smaller than actune_grouped_linear_workspace_size */
} actune_status;

typedef enum actune_dtype {
  ACTUNE_DTYPE_NONE = 0,
  ACTUNE_DTYPE_F32 = 1,
  ACTUNE_DTYPE_F16 = 2,
  ACTUNE_DTYPE_BF16 = 3
} actune_dtype;

/* GEMM kernel and tile choice (the reference's `config` argument of
 * grouped_big_m.cu:92-93 selects among its tile geometries the same way).  All
 * variants compute the identical fp32 chain, so their outputs are bit-identical.
 * BN*: token rows on the MMA M side (128 per tile), BN weight rows per tile, both
 * operands staged in shared memory.  WT*: weights-in-tensor-memory form, 128
 * weight rows per tile expanded straight into TMEM, WT tokens per tile.  GEMV:
 * warp-level integer MMAs streaming 32 weight rows per CTA, for up to 32 tokens. */
typedef enum actune_variant {
  ACTUNE_VARIANT_AUTO = 0,
  ACTUNE_VARIANT_BN32 = 1,
  ACTUNE_VARIANT_BN64 = 2,
  ACTUNE_VARIANT_BN128 = 3,
  ACTUNE_VARIANT_WT16 = 4,
  ACTUNE_VARIANT_WT32 = 5,
  ACTUNE_VARIANT_WT64 = 6,
  ACTUNE_VARIANT_WT128 = 7,
  ACTUNE_VARIANT_GEMV = 8, /* weight-streaming kernel for M <= 32 (AUTO picks it there) */
  ACTUNE_VARIANT_BN32X2 = 9, /* BN* tiles at two CTAs per SM (half the tensor memory each) */
  ACTUNE_VARIANT_BN64X2 = 10,
  ACTUNE_VARIANT_BN128X2 = 11,
  ACTUNE_VARIANT_BN64P = 12, /* BN64 / BN128 tiles in a persistent kernel (one CTA per SM walking the tiles, */
  ACTUNE_VARIANT_BN128P = 13 /* TMA-store epilogue); bf16/f16 outputs with N % 8 == 0, else the BN kernel */
} actune_variant;

/* Device error codes reported by actune_device_error(). */
#define ACTUNE_DEV_OK 0
#define ACTUNE_DEV_TIMEOUT 1 /* a pipeline wait exceeded its time limit; outputs are invalid */

/* Per-token, per-64-group symmetric activation quantizer and bit packer.
 * Replaces the Triton `_quantize_groups` launch in GroupedLinear.forward
 * (actune/kernels/grouped.py:130-133; kernel grouped.py:55-71).
 * x: [M, K] row-major, dtype x_dtype (BF16, F16 or F32), 16-byte aligned.
 * packed: uint8 [M, K*A/8] (8-byte aligned); scales: float [M, K/64]. */
int actune_quantize_group64(const void* x, int x_dtype, int64_t M, int64_t K, int A, uint8_t* packed, float* scales,
                            void* stream);

/* The same A-bit quantization written as one int8 code per element (codes: [M, K],
 * 8-byte aligned), i.e. the W=8 / A=8 operand layout: actune_packed_linear with
 * A = 8 on these codes and W = 8 on int8 weight codes gives bit-for-bit the output
 * of the A-bit (and W-bit) packed call, since the integer group dots and scales are
 * the same.  No reference counterpart (a host that keeps decoded weight codes for
 * calls of many token rows pairs them with these). */
int actune_quantize_group64_codes(const void* x, int x_dtype, int64_t M, int64_t K, int A, uint8_t* codes,
                                  float* scales, void* stream);

/* The packed-integer linear: out = ws * sum_g(float(dot_g) * as[:, g]) (+ bias).
 * Replaces the native op `linear(a, as, w, ws, bias, source, W, A[, config])`
 * (actune/kernels/grouped_native.cu:90-115, grouped_big_m.cu:162-205) and the
 * Triton `_group_gemm` launch (grouped.py:137-142) for all nine W x A pairs.
 * bias may be NULL (bias_dtype NONE); out_dtype is BF16, F16 or F32. */
int actune_packed_linear(const uint8_t* a, const float* a_scale, const uint8_t* w, const float* w_scale,
                         const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                         int W, int A, int variant, void* stream);

/* Tokenwise backends (replace actune/kernels/w4a8_triton.py, w8a8_triton.py,
 * w2a8_triton.py).
 *
 * actune_quantize_rows_a8: per-row dynamic INT8 activations of x [M, K] (bf16 /
 * f16 / f32, K % 8 == 0, 16-byte aligned): scale[m] = max(row absmax, 1e-8) *
 * fp32(1/127), codes = clamp(rint(x / scale), -128, 127); replaces
 * _quantize_rows_kernel, w4a8_triton.py:161-201.
 *
 * actune_tokenwise_linear: out[M, N] = float(sum_k a[m,k] w[n,k]) * a_scale[m] *
 * w_scale[n] (+ bias[n], fused with the last multiply) for int8 activations
 * [M, K] and weight codes of W bits packed as rows [N, K*W/8] (the layout of
 * actune_pack_rows; the Python modules derive it from the reference's K-major
 * buffers).  K % 64 == 0.  variant: AUTO or BN32/BN64/BN128.  Replaces
 * _w4a8_gemm_kernel (w4a8_triton.py:57-114), _w8a8_gemm_kernel
 * (w8a8_triton.py:22-77), _w2a8_gemm_kernel (w2a8_triton.py:25-112). */
int actune_quantize_rows_a8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* codes, float* scales,
                            void* stream);
int actune_tokenwise_linear(const int8_t* a, const float* a_scale, const uint8_t* w, const float* w_scale,
                            const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                            int W, int variant, void* stream);

/* Per-row A4 backends (replace actune/kernels/wxa4_native.py).
 *
 * actune_quantize_rows_a4: per-row dynamic signed INT4 activations of x [M, K]:
 * scale[m] = max(row absmax, 1e-8) * fp32(1/7), codes = clamp(rint(x / scale), -8, 7),
 * packed two per byte (even k in the low nibble) into packed [M, K/2]; replaces
 * _quantize_rows_a4_kernel, wxa4_native.py:27-64.
 *
 * actune_rowwise_linear: actune_tokenwise_linear for A-bit activations packed as
 * rows [M, K*A/8] (A = 8: int8; A = 4: actune_quantize_rows_a4 layout) and the
 * epilogue order of the replaced kernel: order 0 = (float(acc) * as[m]) * ws[n]
 * (+ bias), the Triton kernels (W8A4 runs _w8a8_gemm_kernel, wxa4_native.py:
 * 370-389); order 1 = float(acc) * (as[m] * ws[n]) (+ bias), the native S4 CUDA
 * kernels (native_s4_extension_kernel.cu:229-233).  K % 64 == 0. */
int actune_quantize_rows_a4(const void* x, int x_dtype, int64_t M, int64_t K, uint8_t* packed, float* scales,
                            void* stream);
int actune_rowwise_linear(const uint8_t* a, int A, const float* a_scale, const uint8_t* w, int W, const float* w_scale,
                          const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                          int order, int variant, void* stream);

/* Debug export of the exact per-group int32 dots: dots[m, n, g] =
 * sum_{k in group g} a[m,k]*w[n,k], int32 [M, N, K/64].  These are the integer
 * accumulators of grouped_native.cu:70-74 / grouped.py:89, computed by the same
 * tensor-core kernel as actune_packed_linear. */
int actune_packed_linear_dots(const uint8_t* a, const uint8_t* w, int32_t* dots, int64_t M, int64_t N, int64_t K,
                              int W, int A, int variant, void* stream);

/* Per-row weight codebook (install time).  Replaces
 * actune/kernels/quantizers.py:83-94 `weight_codes(weight, w, a, clip_ratios)`.
 * weight: [N, K] dtype BF16/F16/F32; clip: NULL or float [N] ratios in (0, 1]
 * (validated by the caller as quantizers.py:4-21 does); codes: int8 [N, K];
 * scale: float [N]. */
int actune_weight_codes(const void* weight, int dtype, int64_t N, int64_t K, int W, int A, const float* clip,
                        int8_t* codes, float* scale, void* stream);

/* Nested W8 refinement for given int4 codes and scales.  Replaces
 * actune/kernels/quantizers.py:42-57 `signed_r4_refine(weight, q4, scale4)`.
 * weight: [N, K] BF16/F16/F32; q4: int8 [N, K]; scale4: float [N];
 * residual, q8: int8 [N, K]. */
int actune_r4_refine(const void* weight, int dtype, int64_t N, int64_t K, const int8_t* q4, const float* scale4,
                     int8_t* residual, int8_t* q8, void* stream);

/* Little-endian sub-byte row packing.  Replaces actune/kernels/grouped.py:108-111
 * `pack_rows(q, bits)`.  codes: int8 [R, K]; packed: uint8 [R, K*bits/8]. */
int actune_pack_rows(const int8_t* codes, int64_t R, int64_t K, int bits, uint8_t* packed, void* stream);

/* Bytes of device workspace actune_grouped_linear needs for (M, K, A). */
size_t actune_grouped_linear_workspace_size(int64_t M, int64_t K, int A);

/* Whole GroupedLinear.forward for a row-major [M, K] input (quantize + packed
 * GEMM).  Replaces actune/kernels/grouped.py:127-143.  The packed activations
 * and their scales live in the caller's `workspace` (256-byte aligned, at least
 * actune_grouped_linear_workspace_size(M, K, A) bytes). */
int actune_grouped_linear(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* w, const float* w_scale,
                          const void* bias, int bias_dtype, int64_t N, int W, int A, void* out, int out_dtype,
                          void* workspace, size_t workspace_bytes, int variant, void* stream);

/* Bytes of the fixed device scratch used by actune_grouped_linear_noalloc. */
#define ACTUNE_NOALLOC_SCRATCH_BYTES (8u << 20)

/* actune_grouped_linear for callers that cannot allocate device memory (no
 * counterpart in the reference; its GroupedLinear.forward allocates its
 * temporaries with torch).  Hosts whose device memory is owned by another
 * allocator, or loops that must not allocate once running, pass only inputs and
 * outputs: the packed activations and scales live in a fixed array of
 * ACTUNE_NOALLOC_SCRATCH_BYTES (8 MiB) in this library's device memory, held on
 * every device that loads the library until the process exits.  Requests with
 * actune_grouped_linear_workspace_size(M, K, A) above that size return
 * ACTUNE_ERR_WORKSPACE without launching.  Every call looks up the array's
 * device address (cudaGetSymbolAddress) with the device current, so it stays
 * valid across a device reset; the first call on a device also loads this
 * library's device code there, so make that first call before any stream
 * capture.  The function allocates
 * nothing.  All calls share the one array and it keeps the last call's contents
 * (no part of it needs to start at zero): calls that overlap on the GPU (other
 * streams, other threads) race on it and must be serialised by the caller. */
int actune_grouped_linear_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* w,
                                  const float* w_scale, const void* bias, int bias_dtype, int64_t N, int W, int A,
                                  void* out, int out_dtype, int variant, void* stream);

/* Failure detection (no counterpart in the reference, whose kernels have no
 * bounded waits).  Every pipeline wait of this library's kernels gives up after a
 * time limit, records ACTUNE_DEV_TIMEOUT and the wait site in the device error
 * word (actune_device_error) and lets the kernel finish, so a broken pipeline
 * never hangs the GPU and the context stays usable.
 *
 * actune_set_wait_limit_ns: sets that limit on the current device (default 2 s;
 * accepted range 1 ms .. 60 s) for kernels launched afterwards.  Synchronous.
 * actune_wait_limit_ns: reads it.
 * actune_selftest_wait_timeout: launches a one-warp kernel that waits, with the
 * same bounded primitive, on a barrier nothing arrives on; it records
 * ACTUNE_DEV_TIMEOUT with `site` (> 0) once the limit passes and returns.  It
 * holds no tensor memory and no copies in flight.  For tests of the error path. */
int actune_set_wait_limit_ns(uint64_t ns);
int actune_wait_limit_ns(uint64_t* ns);
int actune_selftest_wait_timeout(int site, void* stream);

/* Human-readable text for an actune_status (static storage). */
const char* actune_status_string(int status);

/* Reads (and with reset != 0 clears) the device error word of the current
 * device.  Synchronous: waits for the device's pending work first.
 * code / site may be NULL. */
int actune_device_error(int* code, int* site, int reset);

/* ACTUNE_ABI_VERSION of the loaded library. */
int actune_abi_version(void);

/* The cudaError_t value behind the last ACTUNE_ERR_CUDA returned on the calling
 * thread (0 if none), for diagnostics; the reference surfaces the same detail in
 * its TORCH_CHECK / CUDA error messages. */
int actune_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* ACTUNE_B200_H */
