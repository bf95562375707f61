// Internal launcher declarations shared by capi.cu and the kernel files.
#pragma once

#include "gemm_group64.cuh"
#include "gemm_wt.cuh"

namespace actune {

// Per-row dynamic quantizer of the tokenwise (bits 8: int8 codes [M, K]) and per-row
// A4 (bits 4: packed [M, K/2]) backends (K % 8 == 0, 16-byte aligned x).
cudaError_t launch_quantize_rows(const void* x, int dtype, int64_t M, int64_t K, int bits, uint8_t* codes,
                                 float* scales, cudaStream_t stream);
// codes8: one int8 code per element instead of packed A-bit codes.
cudaError_t launch_quantize_group64(const void* x, int dtype, int64_t groups, int A, bool codes8, uint8_t* packed,
                                    float* scales, int num_sms, cudaStream_t stream);
cudaError_t launch_weight_codes(const void* w, int dtype, int64_t N, int64_t K, int W, int A, const float* clip,
                                int8_t* codes, float* scale, cudaStream_t stream);
cudaError_t launch_r4_refine(const void* w, int dtype, int64_t N, int64_t K, const int8_t* q4, const float* scale4,
                             int8_t* residual, int8_t* q8, cudaStream_t stream);
// Weight-streaming kernels for M <= 32 (gemv_group64.cu).  With `ts` (M <= 16, packed
// rows a multiple of 128 bytes): 3-D maps over (128-byte block, row, block index) with
// boxes of {128, M, 8 * A} tokens and {128, 32, 8 * W} weight rows, and `ts` a 2-D fp32
// map over the activation scales with boxes of {16, M} (unused when p.dots is set).
// Without: 2-D maps with 128-byte-wide boxes of 16 * ceil(M / 16) token rows and 32
// weight rows.  Packed boxes use the 128-byte swizzle.
constexpr int kGemvStageK = 1024;
// Up to 4 tokens and 2- or 4-bit weights: stages of 2048 K (measured 4-16% faster at
// M = 1; slower at M = 8, where the chain work per stage doubles).
constexpr int kGemvStageKWide = 2048;
inline bool gemv_wide(int64_t M, int W, bool dots) { return M <= 4 && W <= 4 && !dots; }
// Tokenwise decode (M <= 16, K*W/8 and K multiples of 128 bytes): whole-stage maps as
// above, no scale map; p.act_scale holds one scale per token.
cudaError_t launch_gemv_tokenwise(int W, int A, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                                  int num_sms, cudaStream_t stream);
constexpr int kGemvRows = 32;
cudaError_t launch_gemv_group64(int W, int A, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap* ts,
                                const GemmParams& p, int num_sms, cudaStream_t stream);
// Four-group-stage tile GEMM (gemm_wide.cu): every W x A pair, weight tiles of bn = 32
// or 64 rows, gs = 4 groups per stage (other values are refused), group-64 outputs
// only.  The same maps as the tile GEMM (int8 rows: 128-byte SW128
// boxes; packed rows: unswizzled boxes of 16 * bits bytes).
cudaError_t launch_group64_wide(int W, int A, int bn, int gs, const CUtensorMap& ta, const CUtensorMap& tw,
                                const GemmParams& p, cudaStream_t stream);
// Whether AUTO runs the four-group-stage form for this pair and tile width: when its
// shared-memory ring holds at least four stages (int8 codes at 32 and 64 columns; at
// 32 columns also W4A8, W2A8, W8A2, W2A2).  Packed activation staging leaves the other
// forms two-stage rings, measured slower than the two-group-stage kernel.
bool group64_wide_preferred(int W, int A, int bn);
cudaError_t launch_pack_rows(const int8_t* q, int64_t total_bytes, int bits, uint8_t* packed, int num_sms,
                             cudaStream_t stream);

}  // namespace actune
