/*
 * actune_b200 benchmark-harness kernels (bf16 glue around the packed linears of
 * the Llama- and Gemma-shaped benchmark backbones).  Not part of the reference's
 * packed-integer path; they replace the stock elementwise torch ops the
 * reference's models run between projections (HF Llama/Gemma RMSNorm, rotary
 * embedding, gated MLP activation) with one launch each.
 * Same conventions as actune_b200.h: device pointers, caller-owned buffers,
 * asynchronous on `stream`, actune_status return codes.
 */
#ifndef ACTUNE_B200_HARNESS_H
#define ACTUNE_B200_HARNESS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Row-wise RMSNorm of x [T, D] bf16 (optionally after adding `residual`, whose
 * sum is written to residual_out).  gemma != 0 selects the Gemma weight
 * convention out = r * inv * (1 + w); otherwise out = w * bf16(r * inv). */
int actune_harness_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                           int64_t T, int64_t D, float eps, int gemma, void* stream);

/* In-place rotate-half rotary embedding of the q (Hq heads) and k (Hkv heads)
 * parts of a fused bf16 [T, (Hq + 2*Hkv) * Dh] projection; cos/sin fp32 [T, Dh/2]. */
int actune_harness_rope(void* qkv, const float* cos_t, const float* sin_t, int64_t T, int Hq, int Hkv, int Dh,
                        void* stream);

/* out [T, I] = act(gate) * up for gu [T, 2I] = [gate | up]; gelu != 0 uses
 * tanh-GELU (Gemma), else SiLU (Llama). */
int actune_harness_gated_act(const void* gu, void* out, int64_t T, int64_t I, int gelu, void* stream);

/* actune_harness_rmsnorm (vector path: D % 256 == 0, D <= 8192, 16-byte aligned
 * buffers) that also quantizes the bf16 output it stores into the group-64
 * activation format of actune_quantize_group64 (A bits): packed [T, D*A/8] u8, or
 * with codes8 one int8 code per element [T, D] (actune_quantize_group64_codes), and
 * scales [T, D/64] f32, bit-identical to quantizing `out` with that entry. */
int actune_harness_rmsnorm_q(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                             int64_t T, int64_t D, float eps, int gemma, int A, int codes8, uint8_t* packed,
                             float* scales, void* stream);

/* actune_harness_gated_act (I % 64 == 0, 16-byte aligned buffers) that also
 * quantizes its bf16 output: packed [T, I*A/8] u8 (or int8 codes [T, I] with
 * codes8), scales [T, I/64] f32. */
int actune_harness_gated_act_q(const void* gu, void* out, int64_t T, int64_t I, int gelu, int A, int codes8,
                               uint8_t* packed, float* scales, void* stream);

/* actune_harness_rope for one key/value head (Hkv = 1, Dh/2 a multiple of 8,
 * 16-byte aligned buffers) that also writes each token's rotated key and its value
 * into a key/value cache of rows [.., 2, Dh], Tc positions apart between sequences:
 * row b * seq + t of qkv goes to position offset + t of sequence b (T = B * seq
 * rows, offset + seq <= Tc). */
int actune_harness_rope_cache(void* qkv, const float* cos_t, const float* sin_t, int64_t T, int Hq, int Dh,
                              void* cache, int64_t seq, int64_t Tc, int64_t offset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ACTUNE_B200_HARNESS_H */
