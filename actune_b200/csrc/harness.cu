// bf16 glue kernels for the Llama/Gemma-shaped benchmark backbones (sm_100a):
// fused residual-add + RMSNorm, rotary embedding on a fused QKV buffer, and
// SiLU(gate) * up.  They are not part of the packed-integer path; they keep the
// surrounding model from being launch-bound (one launch each instead of the
// several elementwise torch kernels the same math would take).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "actune_b200.h"
#include "actune_b200_harness.h"

namespace {

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }

// One CTA (256 threads) per row.  r = x (+ residual); out = w * bf16(r * rsqrt(mean(r^2) + eps))
// (the HF Llama RMSNorm order: normalise in fp32, round to the model dtype, then
// scale by the bf16 weight); residual_out = bf16(r).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ residual,
                                                      const __nv_bfloat16* __restrict__ weight,
                                                      __nv_bfloat16* __restrict__ out,
                                                      __nv_bfloat16* __restrict__ residual_out, int D, float eps,
                                                      int gemma) {
  extern __shared__ float row[];
  __shared__ float red[8];
  const int64_t t = blockIdx.x;
  const __nv_bfloat16* xr = x + t * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = bf2f(xr[i]);
    if (residual) {
      // The residual stream is kept in bf16, as the reference model does.
      v = bf2f(__float2bfloat16_rn(v + bf2f(residual[t * D + i])));
      residual_out[t * D + i] = __float2bfloat16_rn(v);
    }
    row[i] = v;
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float w = bf2f(weight[i]);
    if (gemma) {
      // Gemma: out = bf16(r * inv * (1 + w)) computed in fp32.
      out[t * D + i] = __float2bfloat16_rn(row[i] * inv * (1.f + w));
    } else {
      out[t * D + i] = __float2bfloat16_rn(w * bf2f(__float2bfloat16_rn(row[i] * inv)));
    }
  }
}

// Rotary embedding (rotate-half convention) applied in place to the q and k
// heads of a fused [T, (Hq + 2*Hkv) * Dh] buffer.  cos/sin: [T, Dh/2] fp32.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int T, int Hq, int Hkv, int Dh) {
  const int half = Dh / 2;
  const int heads = Hq + Hkv;  // q and k heads (v untouched)
  const int64_t total = (int64_t)T * heads * half;
  const int stride_row = (Hq + 2 * Hkv) * Dh;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int h = (int)((i / half) % heads);
    const int t = (int)(i / ((int64_t)half * heads));
    __nv_bfloat16* base = qkv + (int64_t)t * stride_row + h * Dh;
    const float c = cos_t[(int64_t)t * half + j], s = sin_t[(int64_t)t * half + j];
    const float a = bf2f(base[j]), b = bf2f(base[j + half]);
    base[j] = __float2bfloat16_rn(a * c - b * s);
    base[j + half] = __float2bfloat16_rn(b * c + a * s);
  }
}

// out[t, i] = act(gate[t, i]) * up[t, i] with gate/up the two halves of gu[t, :];
// act = SiLU (Llama) or tanh-GELU (Gemma).
__global__ void gated_act_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int T,
                                 int I, int gelu) {
  const int64_t total = (int64_t)T * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / I, c = i % I;
    const float g = bf2f(gu[t * 2 * I + c]), u = bf2f(gu[t * 2 * I + I + c]);
    float a;
    if (gelu) {
      const float k = 0.7978845608028654f;  // sqrt(2/pi)
      a = 0.5f * g * (1.f + tanhf(k * (g + 0.044715f * g * g * g)));
    } else {
      a = g / (1.f + __expf(-g));
    }
    // The model's activation output is bf16 before the product, as in the reference model.
    out[i] = __float2bfloat16_rn(bf2f(__float2bfloat16_rn(a)) * u);
  }
}

int grid_for(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" {

int actune_harness_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                           int64_t T, int64_t D, float eps, int gemma, void* stream) {
  if (T < 0 || D <= 0 || D > 16384 || x == nullptr || weight == nullptr || out == nullptr ||
      (residual != nullptr && residual_out == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  rmsnorm_kernel<<<(unsigned)T, 256, D * sizeof(float), reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(residual),
      reinterpret_cast<const __nv_bfloat16*>(weight), reinterpret_cast<__nv_bfloat16*>(out),
      reinterpret_cast<__nv_bfloat16*>(residual_out), (int)D, eps, gemma);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_rope(void* qkv, const float* cos_t, const float* sin_t, int64_t T, int Hq, int Hkv, int Dh,
                        void* stream) {
  if (T < 0 || Hq <= 0 || Hkv <= 0 || Dh <= 0 || Dh % 2 || qkv == nullptr || cos_t == nullptr || sin_t == nullptr)
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  const int64_t n = T * (Hq + Hkv) * (Dh / 2);
  rope_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv), cos_t, sin_t, (int)T, Hq, Hkv, Dh);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_gated_act(const void* gu, void* out, int64_t T, int64_t I, int gelu, void* stream) {
  if (T < 0 || I <= 0 || gu == nullptr || out == nullptr) return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  gated_act_kernel<<<grid_for(T * I), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(out), (int)T, (int)I, gelu);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

}  // extern "C"
