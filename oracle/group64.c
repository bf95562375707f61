/*
 * CPU oracle for the group-64 packed-integer linear.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
 * file's shared library; the product path (actune_b200) never does.
 *
 * Parity: pinned.  tests/test_oracle.py checks every function below against the
 * golden vectors in tests/golden/, which tests/golden/gen_golden.py produced by
 * running the reference's own code (Triton kernels under TRITON_INTERPRET=1 and
 * the torch weight codebooks).
 *
 * It restates, in plain C, the arithmetic of (paths relative to the reference
 * project root):
 *   actune/kernels/grouped.py:55-71   _quantize_groups (activation quantizer/packer)
 *   actune/kernels/grouped.py:74-94   _group_gemm      (unpack, per-group int dot,
 *                                                       fp32 rescale, epilogue)
 *   actune/kernels/grouped.py:108-111 pack_rows        (little-endian sub-byte pack)
 *   actune/kernels/quantizers.py:23-94 weight codebooks (W2/W4/W8, nested W8 for A4)
 *   actune/kernels/grouped_native.cu:8-17,70-85 (S2->S4 sign extension, epilogue)
 *
 * Floating point: every operation is a single IEEE-754 binary32 operation in
 * round-to-nearest-even (compile with -ffp-contract=off and without
 * -ffast-math).  `fma_mode` selects how `acc += dot*scale` and `acc*ws + bias`
 * are rounded:
 *   fma_mode = 0: separate multiply and add (two roundings) -- what the
 *                 reference computes under the Triton interpreter (numpy);
 *   fma_mode = 1: fused multiply-add (one rounding) -- what the reference's GPU
 *                 kernels compute (Triton enable_fp_fusion and nvcc --fmad=true
 *                 both contract these expressions) and what the CUDA kernels of
 *                 this project compute with explicit fmaf().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_EINVAL 1

static float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* Round-to-nearest-even fp32 -> bf16 (NaN kept quiet). */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

void oracle_f32_to_bf16_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_bf16(src[i]);
}

static int valid_bits(int b) { return b == 2 || b == 4 || b == 8; }

/* Quantize one group of 64 fp32 values (grouped.py:59-71):
 *   scale = max(absmax, 1e-8) / (2^(A-1)-1)          (IEEE division)
 *   code  = clamp(rint(x / scale), -2^(A-1), 2^(A-1)-1)  (IEEE division, RNE)
 *   byte j = sum_i (code[j*P+i] & (2^A-1)) << (i*A),  P = 8/A
 */
static void quantize_one_group(const float* v, int A, uint8_t* packed, float* scale_out) {
    const float positive = (float)((1 << (A - 1)) - 1);
    float absmax = 0.0f;
    for (int i = 0; i < 64; ++i) {
        float a = fabsf(v[i]);
        if (a > absmax) absmax = a;
    }
    float scale = (absmax > 1e-8f ? absmax : 1e-8f) / positive;
    *scale_out = scale;
    const int P = 8 / A;
    const int lo = -(1 << (A - 1)), hi = (1 << (A - 1)) - 1;
    for (int j = 0; j < 64 / P; ++j) {
        unsigned byte = 0;
        for (int i = 0; i < P; ++i) {
            float q = rintf(v[j * P + i] / scale);
            int c = (int)q;
            if (q < (float)lo) c = lo;
            if (q > (float)hi) c = hi;
            byte |= ((unsigned)c & ((1u << A) - 1u)) << (i * A);
        }
        packed[j] = (uint8_t)byte;
    }
}

/* x: [M, K] bf16 bits (row-major). packed: [M, K*A/8]. scales: [M, K/64]. */
int oracle_quantize_group64_bf16(const uint16_t* x, int64_t M, int64_t K, int A,
                                 uint8_t* packed, float* scales) {
    if (!valid_bits(A) || K % 64 || M < 0) return ORACLE_EINVAL;
    float v[64];
    const int64_t G = K / 64;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g = 0; g < G; ++g) {
            for (int i = 0; i < 64; ++i) v[i] = bf16_to_f32(x[m * K + g * 64 + i]);
            quantize_one_group(v, A, packed + m * (K * A / 8) + g * (64 * A / 8), scales + m * G + g);
        }
    return ORACLE_OK;
}

/* Same as above for fp32 input values. */
int oracle_quantize_group64_f32(const float* x, int64_t M, int64_t K, int A,
                                uint8_t* packed, float* scales) {
    if (!valid_bits(A) || K % 64 || M < 0) return ORACLE_EINVAL;
    const int64_t G = K / 64;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g = 0; g < G; ++g)
            quantize_one_group(x + m * K + g * 64, A, packed + m * (K * A / 8) + g * (64 * A / 8),
                               scales + m * G + g);
    return ORACLE_OK;
}

/* Signed field extraction (grouped.py:84-88): element k of a row packed with
 * `bits` bits sits in byte k*bits/8 at bit (k mod 8/bits)*bits; the field is
 * sign-extended as (v ^ 2^(b-1)) - 2^(b-1). */
static int field(const uint8_t* row, int64_t k, int bits) {
    const int per = 8 / bits;
    int v = (row[k / per] >> ((k % per) * bits)) & ((1 << bits) - 1);
    return (v ^ (1 << (bits - 1))) - (1 << (bits - 1));
}

/* Unpack one packed row of K codes into int8. */
int oracle_unpack_rows(const uint8_t* packed, int64_t R, int64_t K, int bits, int8_t* codes) {
    if (!valid_bits(bits) || K % (8 / bits)) return ORACLE_EINVAL;
    for (int64_t r = 0; r < R; ++r)
        for (int64_t k = 0; k < K; ++k)
            codes[r * K + k] = (int8_t)field(packed + r * (K * bits / 8), k, bits);
    return ORACLE_OK;
}

/* pack_rows (grouped.py:108-111): q int8 [R, K] -> [R, K*bits/8]. */
int oracle_pack_rows(const int8_t* q, int64_t R, int64_t K, int bits, uint8_t* packed) {
    if (!valid_bits(bits) || K % (8 / bits)) return ORACLE_EINVAL;
    const int per = 8 / bits;
    for (int64_t r = 0; r < R; ++r)
        for (int64_t j = 0; j < K / per; ++j) {
            unsigned byte = 0;
            for (int i = 0; i < per; ++i)
                byte += ((unsigned)(q[r * K + j * per + i]) & ((1u << bits) - 1u)) << (i * bits);
            packed[r * (K / per) + j] = (uint8_t)byte;
        }
    return ORACLE_OK;
}

/* Per-64-group int32 dots: dots[m, n, g] = sum_{k in group g} a[m,k]*w[n,k]. */
int oracle_group_dots(const uint8_t* a, const uint8_t* w, int64_t M, int64_t N, int64_t K,
                      int W, int A, int32_t* dots) {
    if (!valid_bits(W) || !valid_bits(A) || K % 64) return ORACLE_EINVAL;
    const int64_t G = K / 64;
    int8_t* ac = (int8_t*)malloc((size_t)(M * K > 0 ? M * K : 1));
    int8_t* wc = (int8_t*)malloc((size_t)(N * K > 0 ? N * K : 1));
    if (!ac || !wc) { free(ac); free(wc); return ORACLE_EINVAL; }
    oracle_unpack_rows(a, M, K, A, ac);
    oracle_unpack_rows(w, N, K, W, wc);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            for (int64_t g = 0; g < G; ++g) {
                int32_t d = 0;
                const int8_t* ar = ac + m * K + g * 64;
                const int8_t* wr = wc + n * K + g * 64;
                for (int i = 0; i < 64; ++i) d += (int32_t)ar[i] * (int32_t)wr[i];
                dots[(m * N + n) * G + g] = d;
            }
    free(ac);
    free(wc);
    return ORACLE_OK;
}

/* The whole linear (grouped.py:80-94, grouped_native.cu:70-85):
 *   acc = 0; for g ascending: acc += float(dot_g) * as[m,g]
 *   y = acc * ws[n] (+ bias[n])
 * bias may be NULL.  out: fp32 [M, N] (convert with oracle_f32_to_bf16_array). */
int oracle_packed_linear(const uint8_t* a, const float* as, const uint8_t* w, const float* ws,
                         const float* bias, int64_t M, int64_t N, int64_t K, int W, int A,
                         int fma_mode, float* out) {
    if (!valid_bits(W) || !valid_bits(A) || K % 64) return ORACLE_EINVAL;
    const int64_t G = K / 64;
    int8_t* ac = (int8_t*)malloc((size_t)(M * K > 0 ? M * K : 1));
    int8_t* wc = (int8_t*)malloc((size_t)(N * K > 0 ? N * K : 1));
    if (!ac || !wc) { free(ac); free(wc); return ORACLE_EINVAL; }
    oracle_unpack_rows(a, M, K, A, ac);
    oracle_unpack_rows(w, N, K, W, wc);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                int32_t d = 0;
                const int8_t* ar = ac + m * K + g * 64;
                const int8_t* wr = wc + n * K + g * 64;
                for (int i = 0; i < 64; ++i) d += (int32_t)ar[i] * (int32_t)wr[i];
                const float s = as[m * G + g];
                if (fma_mode) {
                    acc = fmaf((float)d, s, acc);
                } else {
                    volatile float prod = (float)d * s;
                    acc = acc + prod;
                }
            }
            float y;
            if (bias) {
                if (fma_mode) {
                    y = fmaf(acc, ws[n], bias[n]);
                } else {
                    volatile float prod = acc * ws[n];
                    y = prod + bias[n];
                }
            } else {
                y = acc * ws[n];
            }
            out[m * N + n] = y;
        }
    free(ac);
    free(wc);
    return ORACLE_OK;
}

/* Weight codebooks (quantizers.py:23-94).  weight: fp32 [N, K]; clip: NULL or
 * per-row ratios in (0, 1] (already validated by the caller).  codes: int8
 * [N, K]; scale: fp32 [N].
 *   W4:            scale = max(absmax,1e-8)*clip / 7,  q = clamp(rint(v/scale), -8, 7)
 *   W2:            scale = max(absmax,1e-8)*clip,      q = clamp(rint(v/scale), -2, 1)
 *   W8, A != 4:    scale = max(absmax,1e-8) / 127 (clip ignored), q = clamp(rint(v/scale), -128, 127)
 *   W8, A == 4:    nested code q8 = 16*q4 + r4 with r4 = clamp(rint(16*(v/s4 - q4)), lo, hi),
 *                  lo = max(-8, -128-16*q4), hi = min(7, 127-16*q4), scale = s4/16.
 */
int oracle_weight_codes(const float* weight, int64_t N, int64_t K, int W, int A, const float* clip,
                        int8_t* codes, float* scale) {
    if (!valid_bits(W) || !valid_bits(A)) return ORACLE_EINVAL;
    for (int64_t n = 0; n < N; ++n) {
        const float* v = weight + n * K;
        float absmax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float t = fabsf(v[k]);
            if (t > absmax) absmax = t;
        }
        float rowmax = absmax > 1e-8f ? absmax : 1e-8f;
        int8_t* q = codes + n * K;
        if (W == 8 && A != 4) {
            float s = rowmax / 127.0f;
            scale[n] = s;
            for (int64_t k = 0; k < K; ++k) {
                float r = rintf(v[k] / s);
                r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
                q[k] = (int8_t)r;
            }
            continue;
        }
        if (clip) rowmax = rowmax * clip[n];
        const float s = (W == 2) ? rowmax : rowmax / 7.0f;
        const float lo = (W == 2) ? -2.0f : -8.0f, hi = (W == 2) ? 1.0f : 7.0f;
        for (int64_t k = 0; k < K; ++k) {
            float r = rintf(v[k] / s);
            r = r < lo ? lo : (r > hi ? hi : r);
            q[k] = (int8_t)r;
        }
        if (W == 8) { /* A == 4: nested refinement (signed_r4_refine) */
            for (int64_t k = 0; k < K; ++k) {
                const int q4 = q[k];
                volatile float quotient = v[k] / s;
                volatile float diff = quotient - (float)q4;
                float rf = rintf(16.0f * diff);
                rf = rf < -8.0f ? -8.0f : (rf > 7.0f ? 7.0f : rf);
                int r = (int)rf;
                int rlo = -128 - 16 * q4, rhi = 127 - 16 * q4;
                if (rlo < -8) rlo = -8;
                if (rhi > 7) rhi = 7;
                if (r < rlo) r = rlo;
                if (r > rhi) r = rhi;
                q[k] = (int8_t)(16 * q4 + r);
            }
            scale[n] = s / 16.0f;
        } else {
            scale[n] = s;
        }
    }
    return ORACLE_OK;
}

/* ---- tokenwise backends (reference actune/kernels/w4a8_triton.py,
 * w8a8_triton.py, w2a8_triton.py) --------------------------------------------
 *
 * Per-row dynamic INT8 activation quantizer, w4a8_triton.py:161-201:
 *   scale = max(row absmax, 1e-8) * fp32(1/127)   -- a multiply by the binary32
 *           reciprocal, as torch lowers CUDA tensor/scalar division (the
 *           reference reproduces that on purpose, w4a8_triton.py:179-184)
 *   code  = clamp(rint(x / scale), -128, 127)      -- IEEE division, RNE */
int oracle_quantize_rows_a8(const uint16_t* x, int64_t M, int64_t K, int8_t* codes, float* scales) {
    if (M < 0 || K <= 0) return 1;
    const float recip = 1.0f / 127.0f;
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* row = x + m * K;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float v = fabsf(bf16_to_f32(row[k]));
            if (v > amax) amax = v;
        }
        const float scale = (amax > 1e-8f ? amax : 1e-8f) * recip;
        scales[m] = scale;
        for (int64_t k = 0; k < K; ++k) {
            float q = rintf(bf16_to_f32(row[k]) / scale);
            if (q < -128.0f) q = -128.0f;
            if (q > 127.0f) q = 127.0f;
            codes[m * K + k] = (int8_t)(int)q;
        }
    }
    return 0;
}

/* Tokenwise linear, w4a8_triton.py:57-114 (and the W8/W2 kernels): exact int32
 * dot over all of K, then out = float(acc) * as[m]; out *= ws[n]; out += bias[n]
 * in that order (fma_mode 1 fuses the last multiply and add, as GPU compilers
 * do; 0 rounds twice).  codes is [N, K] int8. */
int oracle_tokenwise_linear(const int8_t* a, const float* as, const int8_t* codes, const float* ws,
                            const float* bias, int64_t M, int64_t N, int64_t K, int fma_mode, float* out) {
    if (M < 0 || N < 0 || K <= 0) return 1;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            int64_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int64_t)a[m * K + k] * (int64_t)codes[n * K + k];
            const float t = (float)(int32_t)acc * as[m];
            float y;
            if (bias) {
                y = fma_mode ? fmaf(t, ws[n], bias[n]) : t * ws[n] + bias[n];
            } else {
                y = t * ws[n];
            }
            out[m * N + n] = y;
        }
    }
    return 0;
}

/* ---- per-row A4 backends (reference actune/kernels/wxa4_native.py) ---- */

/* Per-row dynamic INT4 activations, _quantize_rows_a4_kernel (wxa4_native.py:27-64):
 * scale = max(absmax, 1e-8) * fp32(1/7); codes clamp(rint(x / scale), -8, 7) with
 * the division correctly rounded; two codes per byte, even k in the low nibble;
 * packed is [M, (K+1)/2]. */
int oracle_quantize_rows_a4(const uint16_t* x, int64_t M, int64_t K, uint8_t* packed, float* scales) {
    if (M < 0 || K <= 0) return 1;
    const float recip = 1.0f / 7.0f;
    const int64_t KB = (K + 1) / 2;
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* row = x + m * K;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float v = fabsf(bf16_to_f32(row[k]));
            if (v > amax) amax = v;
        }
        const float scale = (amax > 1e-8f ? amax : 1e-8f) * recip;
        scales[m] = scale;
        for (int64_t j = 0; j < KB; ++j) {
            int nib[2] = {0, 0};
            for (int h = 0; h < 2; ++h) {
                const int64_t k = 2 * j + h;
                float q = k < K ? rintf(bf16_to_f32(row[k]) / scale) : 0.0f;
                if (q < -8.0f) q = -8.0f;
                if (q > 7.0f) q = 7.0f;
                nib[h] = ((int)q) & 15;
            }
            packed[m * KB + j] = (uint8_t)(nib[0] | (nib[1] << 4));
        }
    }
    return 0;
}

/* The native W{2,4}A4 epilogue (native_s4_extension_kernel.cu:226-234): exact int32
 * dot over all of K, then value = float(acc); value *= as[m] * ws[n] (the scale
 * product rounded first); value += bias[n] (fma_mode 1 fuses the multiply and add,
 * as nvcc contracts them; 0 rounds twice).  a is [M, K] int8 codes, codes [N, K]. */
int oracle_rowwise_native_linear(const int8_t* a, const float* as, const int8_t* codes, const float* ws,
                                 const float* bias, int64_t M, int64_t N, int64_t K, int fma_mode, float* out) {
    if (M < 0 || N < 0 || K <= 0) return 1;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            int64_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int64_t)a[m * K + k] * (int64_t)codes[n * K + k];
            const float f = (float)(int32_t)acc;
            const float s = as[m] * ws[n];
            float y;
            if (bias) {
                y = fma_mode ? fmaf(f, s, bias[n]) : f * s + bias[n];
            } else {
                y = f * s;
            }
            out[m * N + n] = y;
        }
    }
    return 0;
}

int oracle_abi_version(void) { return 1; }
