// bf16 glue kernels for the Llama/Gemma-shaped benchmark backbones (sm_100a):
// fused residual-add + RMSNorm, rotary embedding on a fused QKV buffer, and
// SiLU(gate) * up, optionally also quantizing their output to the group-64
// packed activation format the next projection reads.  They are not part of the
// packed-integer path; they keep the
// surrounding model from being launch-bound (one launch each instead of the
// several elementwise torch kernels the same math would take).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "actune_b200.h"
#include "actune_b200_harness.h"
#include "common.cuh"

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
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
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
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
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
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
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

// ---- vectorised forms (16-byte loads/stores); shapes must be multiples of 8 ----
__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
}
__device__ __forceinline__ float bf16_round(float v) { return bf2f(__float2bfloat16_rn(v)); }

// One CTA (256 threads) per row, CPT chunks of 8 elements per thread kept in
// registers: D <= 2048 * CPT, D % 8 == 0.  Same arithmetic as rmsnorm_kernel.
// QA > 0: the bf16 output is also quantized (group 64, QA bits) into qpacked /
// qscales, from the rounded values it stores (D % 256 == 0: whole warps per row);
// QOUT = QA packs the codes, QOUT = 8 stores one int8 code per element.
template <int CPT, int QA, int QOUT = QA>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ residual,
                                                          const __nv_bfloat16* __restrict__ weight,
                                                          __nv_bfloat16* __restrict__ out,
                                                          __nv_bfloat16* __restrict__ residual_out, int D, float eps,
                                                          int gemma, uint8_t* __restrict__ qpacked,
                                                          float* __restrict__ qscales) {
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
  __shared__ float red[8];
  const int64_t base = (int64_t)blockIdx.x * D;
  float v[CPT][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int i = (threadIdx.x + c * 256) * 8;
    if (i < D) {
      unpack8(__ldg(reinterpret_cast<const uint4*>(x + base + i)), v[c]);
      if (residual) {
        float r[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(residual + base + i)), r);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[c][k] = bf16_round(v[c][k] + r[k]);
        *reinterpret_cast<uint4*>(residual_out + base + i) = pack8(v[c]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[c][k] * v[c][k];
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)D + eps);
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int i = (threadIdx.x + c * 256) * 8;
    if (i < D) {
      float w[8], o[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(weight + i)), w);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = gemma ? v[c][k] * inv * (1.f + w[k]) : w[k] * bf16_round(v[c][k] * inv);
      const uint4 stored = pack8(o);
      *reinterpret_cast<uint4*>(out + base + i) = stored;
      if constexpr (QA > 0) {
        float q[8];
        unpack8(stored, q);
        uint32_t word[2];
        const float scale = actune::quantize_lane8<QA, QOUT>(q, word);
        actune::store_lane_codes<QOUT>(qpacked + (base + i) * QOUT / 8, word);
        if ((threadIdx.x & 7) == 0) qscales[(base + i) / 64] = scale;
      }
    }
  }
}

// Rotary embedding, one CTA per token; thread handles 8 consecutive rotation pairs
// of one head (half % 8 == 0).
// With `cache` (one key/value head): the token's rotated key and its value are also
// written to cache[b, offset + t, 0 / 1, :] for row b * seq + t.
__global__ void __launch_bounds__(256) rope_vec_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                                                       const float* __restrict__ sin_t, int Hq, int Hkv, int Dh,
                                                       __nv_bfloat16* __restrict__ cache, int seq, int Tc, int offset) {
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
  const int half = Dh / 2, per_head = half / 8, heads = Hq + Hkv;
  const int t = blockIdx.x;
  __nv_bfloat16* row = qkv + (int64_t)t * (Hq + 2 * Hkv) * Dh;
  const float* cr = cos_t + (int64_t)t * half;
  const float* sr = sin_t + (int64_t)t * half;
  for (int item = threadIdx.x; item < heads * per_head; item += blockDim.x) {
    const int h = item / per_head, j = (item % per_head) * 8;
    __nv_bfloat16* b = row + h * Dh;
    float a[8], bb[8], c[8], s[8];
    unpack8(*reinterpret_cast<const uint4*>(b + j), a);
    unpack8(*reinterpret_cast<const uint4*>(b + j + half), bb);
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(cr + j)), c1 = __ldg(reinterpret_cast<const float4*>(cr + j + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sr + j)), s1 = __ldg(reinterpret_cast<const float4*>(sr + j + 4));
    c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
    s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w; s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
    float o1[8], o2[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      o1[k] = a[k] * c[k] - bb[k] * s[k];
      o2[k] = bb[k] * c[k] + a[k] * s[k];
    }
    *reinterpret_cast<uint4*>(b + j) = pack8(o1);
    *reinterpret_cast<uint4*>(b + j + half) = pack8(o2);
  }
  if (cache != nullptr) {
    __syncthreads();  // the rotated key is complete
    const __nv_bfloat16* kv = row + Hq * Dh;  // key then value, Dh each
    __nv_bfloat16* dst = cache + ((int64_t)(t / seq) * Tc + offset + t % seq) * 2 * Dh;
    for (int c = threadIdx.x; c < 2 * Dh / 8; c += blockDim.x)
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(kv)[c];
  }
}

// Gated activation, 8 outputs per thread (I % 8 == 0).  QA > 0: the output is also
// quantized (group 64, QA bits; I % 64 == 0) from the rounded values it stores,
// packed (QOUT = QA) or one int8 code per element (QOUT = 8).  Warps step through
// the items together so that each 64-group's 8 lanes shuffle as one segment.
template <int QA, int QOUT = QA>
__global__ void __launch_bounds__(256) gated_act_vec_kernel(const __nv_bfloat16* __restrict__ gu,
                                                            __nv_bfloat16* __restrict__ out, int T, int I, int gelu,
                                                            uint8_t* __restrict__ qpacked,
                                                            float* __restrict__ qscales) {
  actune::griddep_enter();  // dependent launch: the inputs are the previous kernel's outputs
  const int per_row = I / 8;
  const int64_t total = (int64_t)T * per_row;
  const int lane = threadIdx.x & 31;
  for (int64_t wbase = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); wbase < total;
       wbase += (int64_t)gridDim.x * blockDim.x) {
    const int64_t item = wbase + lane;
    const bool live = item < total;
    uint4 stored = make_uint4(0, 0, 0, 0);
    if (live) {
      const int t = (int)(item / per_row), c = (int)(item % per_row) * 8;
      float g[8], u[8], o[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(gu + (int64_t)t * 2 * I + c)), g);
      unpack8(__ldg(reinterpret_cast<const uint4*>(gu + (int64_t)t * 2 * I + I + c)), u);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float a;
        if (gelu) {
          const float kk = 0.7978845608028654f;  // sqrt(2/pi)
          a = 0.5f * g[k] * (1.f + tanhf(kk * (g[k] + 0.044715f * g[k] * g[k] * g[k])));
        } else {
          a = g[k] / (1.f + __expf(-g[k]));
        }
        o[k] = bf16_round(a) * u[k];
      }
      stored = pack8(o);
      *reinterpret_cast<uint4*>(out + item * 8) = stored;
    }
    if constexpr (QA > 0) {
      // Groups never straddle live and dead items: total and wbase are multiples of 8.
      float q[8];
      unpack8(stored, q);
      uint32_t word[2];
      const float scale = actune::quantize_lane8<QA, QOUT>(q, word);
      if (live) {
        actune::store_lane_codes<QOUT>(qpacked + item * QOUT, word);
        if ((lane & 7) == 0) qscales[item / 8] = scale;
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int grid_for(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return (int)(b < 1 ? 1 : b);
}

template <int QA, int QOUT = QA>
cudaError_t launch_rmsnorm_q(const __nv_bfloat16* xb, const __nv_bfloat16* rb, const __nv_bfloat16* wb,
                             __nv_bfloat16* ob, __nv_bfloat16* rob, int64_t T, int64_t D, float eps, int gemma,
                             uint8_t* qp, float* qs, cudaStream_t cs) {
  if (D <= 2048)
    (void)actune::launch_pdl(rmsnorm_vec_kernel<1, QA, QOUT>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, qp, qs);
  else if (D <= 4096)
    (void)actune::launch_pdl(rmsnorm_vec_kernel<2, QA, QOUT>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, qp, qs);
  else
    (void)actune::launch_pdl(rmsnorm_vec_kernel<4, QA, QOUT>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, qp, qs);
  return cudaGetLastError();
}

}  // namespace

extern "C" {

int actune_harness_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                           int64_t T, int64_t D, float eps, int gemma, void* stream) {
  if (T < 0 || D <= 0 || D > 16384 || x == nullptr || weight == nullptr || out == nullptr ||
      (residual != nullptr && residual_out == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  const bool vec = D % 8 == 0 && D <= 8192 && aligned16(x) && aligned16(weight) && aligned16(out) &&
                   (residual == nullptr || (aligned16(residual) && aligned16(residual_out)));
  if (vec) {
    const auto cs = reinterpret_cast<cudaStream_t>(stream);
    const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
    const auto* rb = reinterpret_cast<const __nv_bfloat16*>(residual);
    const auto* wb = reinterpret_cast<const __nv_bfloat16*>(weight);
    auto* ob = reinterpret_cast<__nv_bfloat16*>(out);
    auto* rob = reinterpret_cast<__nv_bfloat16*>(residual_out);
    if (D <= 2048) (void)actune::launch_pdl(rmsnorm_vec_kernel<1, 0>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, nullptr, nullptr);
    else if (D <= 4096) (void)actune::launch_pdl(rmsnorm_vec_kernel<2, 0>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, nullptr, nullptr);
    else (void)actune::launch_pdl(rmsnorm_vec_kernel<4, 0>, dim3((unsigned)T), 256, 0, cs, xb, rb, wb, ob, rob, (int)D, eps, gemma, nullptr, nullptr);
    return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
  }
  (void)actune::launch_pdl(rmsnorm_kernel, dim3((unsigned)T), 256, D * sizeof(float), reinterpret_cast<cudaStream_t>(stream), 
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
  if ((Dh / 2) % 8 == 0 && aligned16(qkv) && aligned16(cos_t) && aligned16(sin_t)) {
    (void)actune::launch_pdl(rope_vec_kernel, dim3((unsigned)T), 256, 0, reinterpret_cast<cudaStream_t>(stream),
        reinterpret_cast<__nv_bfloat16*>(qkv), cos_t, sin_t, Hq, Hkv, Dh, nullptr, 1, 0, 0);
    return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
  }
  const int64_t n = T * (Hq + Hkv) * (Dh / 2);
  (void)actune::launch_pdl(rope_kernel, dim3(grid_for(n)), 256, 0, reinterpret_cast<cudaStream_t>(stream), 
      reinterpret_cast<__nv_bfloat16*>(qkv), cos_t, sin_t, (int)T, Hq, Hkv, Dh);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_rope_cache(void* qkv, const float* cos_t, const float* sin_t, int64_t T, int Hq, int Dh,
                              void* cache, int64_t seq, int64_t Tc, int64_t offset, void* stream) {
  if (T < 0 || Hq <= 0 || Dh <= 0 || (Dh / 2) % 8 || seq <= 0 || T % seq || offset < 0 || offset + seq > Tc ||
      qkv == nullptr || cos_t == nullptr || sin_t == nullptr || cache == nullptr)
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  if (!aligned16(qkv) || !aligned16(cos_t) || !aligned16(sin_t) || !aligned16(cache)) return ACTUNE_ERR_MISALIGNED;
  (void)actune::launch_pdl(rope_vec_kernel, dim3((unsigned)T), 256, 0, reinterpret_cast<cudaStream_t>(stream),
      reinterpret_cast<__nv_bfloat16*>(qkv), cos_t, sin_t, Hq, 1, Dh, reinterpret_cast<__nv_bfloat16*>(cache),
      (int)seq, (int)Tc, (int)offset);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_gated_act(const void* gu, void* out, int64_t T, int64_t I, int gelu, void* stream) {
  if (T < 0 || I <= 0 || gu == nullptr || out == nullptr) return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  if (I % 8 == 0 && aligned16(gu) && aligned16(out)) {
    (void)actune::launch_pdl(gated_act_vec_kernel<0>, dim3(grid_for(T * I / 8)), 256, 0, reinterpret_cast<cudaStream_t>(stream), 
        reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(out), (int)T, (int)I, gelu,
        nullptr, nullptr);
    return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
  }
  (void)actune::launch_pdl(gated_act_kernel, dim3(grid_for(T * I)), 256, 0, reinterpret_cast<cudaStream_t>(stream), 
      reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(out), (int)T, (int)I, gelu);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_rmsnorm_q(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                             int64_t T, int64_t D, float eps, int gemma, int A, int codes8, uint8_t* packed,
                             float* scales, void* stream) {
  if (T < 0 || D <= 0 || D > 8192 || D % 256 || x == nullptr || weight == nullptr || out == nullptr ||
      packed == nullptr || scales == nullptr || (residual != nullptr && residual_out == nullptr) ||
      (A != 2 && A != 4 && A != 8))
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || !aligned16(packed) || !aligned16(scales) ||
      (residual != nullptr && (!aligned16(residual) || !aligned16(residual_out))))
    return ACTUNE_ERR_MISALIGNED;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* rb = reinterpret_cast<const __nv_bfloat16*>(residual);
  const auto* wb = reinterpret_cast<const __nv_bfloat16*>(weight);
  auto* ob = reinterpret_cast<__nv_bfloat16*>(out);
  auto* rob = reinterpret_cast<__nv_bfloat16*>(residual_out);
  auto* cs = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = A == 8 ? launch_rmsnorm_q<8>(xb, rb, wb, ob, rob, T, D, eps, gemma, packed, scales, cs)
                : A == 4 ? (codes8 ? launch_rmsnorm_q<4, 8>(xb, rb, wb, ob, rob, T, D, eps, gemma, packed, scales, cs)
                                   : launch_rmsnorm_q<4>(xb, rb, wb, ob, rob, T, D, eps, gemma, packed, scales, cs))
                         : (codes8 ? launch_rmsnorm_q<2, 8>(xb, rb, wb, ob, rob, T, D, eps, gemma, packed, scales, cs)
                                   : launch_rmsnorm_q<2>(xb, rb, wb, ob, rob, T, D, eps, gemma, packed, scales, cs));
  return e == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

int actune_harness_gated_act_q(const void* gu, void* out, int64_t T, int64_t I, int gelu, int A, int codes8,
                               uint8_t* packed, float* scales, void* stream) {
  if (T < 0 || I <= 0 || I % 64 || gu == nullptr || out == nullptr || packed == nullptr || scales == nullptr ||
      (A != 2 && A != 4 && A != 8))
    return ACTUNE_ERR_INVALID_VALUE;
  if (T == 0) return ACTUNE_OK;
  if (!aligned16(gu) || !aligned16(out) || !aligned16(packed) || !aligned16(scales)) return ACTUNE_ERR_MISALIGNED;
  const auto* g = reinterpret_cast<const __nv_bfloat16*>(gu);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto* cs = reinterpret_cast<cudaStream_t>(stream);
  const int grid = grid_for(T * I / 8);
  if (A == 8) (void)actune::launch_pdl(gated_act_vec_kernel<8>, dim3(grid), 256, 0, cs, g, o, (int)T, (int)I, gelu, packed, scales);
  else if (A == 4 && codes8) (void)actune::launch_pdl(gated_act_vec_kernel<4, 8>, dim3(grid), 256, 0, cs, g, o, (int)T, (int)I, gelu, packed, scales);
  else if (A == 4) (void)actune::launch_pdl(gated_act_vec_kernel<4>, dim3(grid), 256, 0, cs, g, o, (int)T, (int)I, gelu, packed, scales);
  else if (codes8) (void)actune::launch_pdl(gated_act_vec_kernel<2, 8>, dim3(grid), 256, 0, cs, g, o, (int)T, (int)I, gelu, packed, scales);
  else (void)actune::launch_pdl(gated_act_vec_kernel<2>, dim3(grid), 256, 0, cs, g, o, (int)T, (int)I, gelu, packed, scales);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

}  // extern "C"
