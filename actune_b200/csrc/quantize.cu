// Activation quantizer/packer and install-time weight codebooks (sm_100a).
//
// quantize_group64_kernel restates actune/kernels/grouped.py:55-71 (per token,
// per 64-wide group along K):
//   scale = max(absmax, 1e-8) / (2^(A-1) - 1)        IEEE division
//   code  = clamp(rint(x / scale), -2^(A-1), 2^(A-1)-1)   IEEE division, RNE
//   byte j of the group = sum_i (code[j*P+i] & (2^A-1)) << (i*A),  P = 8/A
// One group is 64 elements = 8 lanes x 8 elements: each lane does one 16-byte
// (bf16/fp16) or 32-byte (fp32) coalesced load, the group's absmax is a 3-step
// xor-shuffle inside the 8-lane segment, and each lane stores its 8*A/8 packed
// bytes, so a warp moves 4 groups per step with fully coalesced traffic.
//
// weight_codes_kernel restates actune/kernels/quantizers.py:23-94 (one CTA per
// output row) and pack_rows_kernel restates grouped.py:108-111.
#include "common.cuh"
#include "kernels.cuh"

namespace actune {

__device__ int g_actune_error = 0;
__device__ int g_actune_error_site = 0;
__device__ unsigned long long g_actune_wait_limit_ns = kDefaultWaitLimitNs;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// OUT = A: packed A-bit codes [groups * 64 * A / 8]; OUT = 8: one int8 code per
// element (the same A-bit codes, for the W=8 / A=8 GEMM).
template <int A, typename T, int OUT = A>
__global__ void __launch_bounds__(256) quantize_group64_kernel(const T* __restrict__ x, uint8_t* __restrict__ packed,
                                                               float* __restrict__ scales, int64_t groups) {
  griddep_enter();  // dependent launch: x is the previous kernel's output
  const int lane = threadIdx.x & 31;
  const int seg = lane >> 3, l8 = lane & 7;
  const int64_t warp_global = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t warp_stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t base = warp_global * 4; base < groups; base += warp_stride * 4) {
    const int64_t g = base + seg;
    const bool live = g < groups;
    float v[8];
    if (live) {
      load8<T>(x + g * 64 + l8 * 8, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    uint32_t word[2];
    const float scale = quantize_lane8<A, OUT>(v, word);
    if (!live) continue;
    store_lane_codes<OUT>(packed + g * (64 * OUT / 8) + l8 * OUT, word);
    if (l8 == 0) scales[g] = scale;
  }
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// One CTA per output row n.  codes: int8 [N, K]; scale: f32 [N].
template <typename T>
__global__ void __launch_bounds__(256) weight_codes_kernel(const T* __restrict__ weight, int64_t K, int W, int A,
                                                           const float* __restrict__ clip, int8_t* __restrict__ codes,
                                                           float* __restrict__ scale_out) {
  __shared__ float red[8];
  const int64_t n = blockIdx.x;
  const T* row = weight + n * K;
  float amax = 0.f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f32(row[k])));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  float rowmax = fmaxf(red[0], 1e-8f);
  int8_t* q = codes + n * K;
  if (W == 8 && A != 4) {
    const float s = __fdiv_rn(rowmax, 127.0f);
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const float r = fminf(fmaxf(rintf(__fdiv_rn(to_f32(row[k]), s)), -128.f), 127.f);
      q[k] = (int8_t)(int)r;
    }
    if (threadIdx.x == 0) scale_out[n] = s;
    return;
  }
  if (clip != nullptr) rowmax = __fmul_rn(rowmax, clip[n]);
  const float s = (W == 2) ? rowmax : __fdiv_rn(rowmax, 7.0f);
  const float lo = (W == 2) ? -2.f : -8.f, hi = (W == 2) ? 1.f : 7.f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = to_f32(row[k]);
    const float quotient = __fdiv_rn(v, s);
    const float r4 = fminf(fmaxf(rintf(quotient), lo), hi);
    if (W == 8) {
      // Nested W8 for A4 (quantizers.py:42-57, 88-91): q8 = 16*q4 + r4'.
      const int q4 = (int)r4;
      const float resid = __fmul_rn(16.0f, __fsub_rn(quotient, r4));
      int r = (int)fminf(fmaxf(rintf(resid), -8.f), 7.f);
      const int rlo = max(-8, -128 - 16 * q4), rhi = min(7, 127 - 16 * q4);
      r = min(max(r, rlo), rhi);
      q[k] = (int8_t)(16 * q4 + r);
    } else {
      q[k] = (int8_t)(int)r4;
    }
  }
  if (threadIdx.x == 0) scale_out[n] = (W == 8) ? __fdiv_rn(s, 16.0f) : s;
}

// Nested W8 refinement for a given (q4, scale4) (quantizers.py:42-57):
//   resid = rint(16 * (v / s4 - q4)) clamped to [-8, 7] and to
//   [max(-8, -128 - 16*q4), min(7, 127 - 16*q4)];  q8 = 16*q4 + resid.
template <typename T>
__global__ void __launch_bounds__(256) r4_refine_kernel(const T* __restrict__ weight, int64_t K,
                                                        const int8_t* __restrict__ q4, const float* __restrict__ scale4,
                                                        int8_t* __restrict__ residual, int8_t* __restrict__ q8) {
  const int64_t n = blockIdx.x;
  const float s = scale4[n];
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    const int64_t i = n * K + k;
    const int q = q4[i];
    const float resid = __fmul_rn(16.0f, __fsub_rn(__fdiv_rn(to_f32(weight[i]), s), (float)q));
    int r = (int)fminf(fmaxf(rintf(resid), -8.f), 7.f);
    r = min(max(r, max(-8, -128 - 16 * q)), min(7, 127 - 16 * q));
    residual[i] = (int8_t)r;
    q8[i] = (int8_t)(16 * q + r);
  }
}

cudaError_t launch_r4_refine(const void* w, int dtype, int64_t N, int64_t K, const int8_t* q4, const float* scale4,
                             int8_t* residual, int8_t* q8, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  switch (dtype) {
    case kDtBF16:
      r4_refine_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(w), K, q4, scale4,
                                                        residual, q8);
      break;
    case kDtF16:
      r4_refine_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const __half*>(w), K, q4, scale4, residual,
                                                        q8);
      break;
    default:
      r4_refine_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const float*>(w), K, q4, scale4, residual,
                                                        q8);
      break;
  }
  return cudaGetLastError();
}

// One thread per packed byte: byte j of a row holds codes j*P .. j*P+P-1.
__global__ void __launch_bounds__(256) pack_rows_kernel(const int8_t* __restrict__ q, int64_t total_bytes, int bits,
                                                        uint8_t* __restrict__ packed) {
  const int per = 8 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < total_bytes;
       j += (int64_t)gridDim.x * blockDim.x) {
    uint32_t byte = 0;
    for (int i = 0; i < per; ++i) byte |= ((uint32_t)(uint8_t)q[j * per + i] & mask) << (i * bits);
    packed[j] = (uint8_t)byte;
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
template <typename T>
static cudaError_t launch_quantize_t(const T* x, int64_t groups, int A, bool codes8, uint8_t* packed, float* scales,
                                     int num_sms, cudaStream_t stream) {
  const int threads = 256;
  const int64_t warps_needed = (groups + 3) / 4;
  int64_t blocks = (warps_needed + 7) / 8;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (codes8 && A == 2)
    (void)launch_pdl(quantize_group64_kernel<2, T, 8>, dim3((unsigned)blocks), threads, 0, stream, x, packed, scales, groups);
  else if (codes8 && A == 4)
    (void)launch_pdl(quantize_group64_kernel<4, T, 8>, dim3((unsigned)blocks), threads, 0, stream, x, packed, scales, groups);
  else if (A == 2)
    (void)launch_pdl(quantize_group64_kernel<2, T>, dim3((unsigned)blocks), threads, 0, stream, x, packed, scales, groups);
  else if (A == 4)
    (void)launch_pdl(quantize_group64_kernel<4, T>, dim3((unsigned)blocks), threads, 0, stream, x, packed, scales, groups);
  else
    (void)launch_pdl(quantize_group64_kernel<8, T>, dim3((unsigned)blocks), threads, 0, stream, x, packed, scales, groups);
  return cudaGetLastError();
}

cudaError_t launch_quantize_group64(const void* x, int dtype, int64_t groups, int A, bool codes8, uint8_t* packed,
                                    float* scales, int num_sms, cudaStream_t stream) {
  if (groups == 0) return cudaSuccess;
  switch (dtype) {
    case kDtBF16:
      return launch_quantize_t(reinterpret_cast<const __nv_bfloat16*>(x), groups, A, codes8, packed, scales, num_sms,
                               stream);
    case kDtF16:
      return launch_quantize_t(reinterpret_cast<const __half*>(x), groups, A, codes8, packed, scales, num_sms, stream);
    default:
      return launch_quantize_t(reinterpret_cast<const float*>(x), groups, A, codes8, packed, scales, num_sms, stream);
  }
}

// Per-row dynamic activation quantizers of the tokenwise (A8) and per-row A4
// backends, restating actune/kernels/w4a8_triton.py:161-201 (BITS 8) and
// actune/kernels/wxa4_native.py:27-64 (BITS 4):
//   scale = max(row absmax, 1e-8) * fp32(1/P),  P = 2^(BITS-1) - 1
//   (a multiply by the binary32 reciprocal, which is what torch computes for a CUDA
//   tensor divided by a scalar and what the reference reproduces on purpose), then
//   code = clamp(rint(x / scale), -P-1, P) with IEEE division.
// BITS 8 stores int8 codes [M, K]; BITS 4 packs two codes per byte, even k in the
// low nibble (the group-64 row layout).  One CTA per row; each thread holds up to
// CPT chunks of 8 values in registers between the absmax and the quantizing pass
// (CPT == 0: K beyond the register cache, read twice).
template <typename T, int CPT, int BITS>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ x, uint8_t* __restrict__ codes,
                                                            float* __restrict__ scales, int64_t K) {
  constexpr float kPos = float((1 << (BITS - 1)) - 1);
  constexpr float kNeg = -float(1 << (BITS - 1));
  __shared__ float red[8];
  griddep_enter();  // dependent launch: x is the previous kernel's output
  const int64_t row = blockIdx.x;
  const T* xr = x + row * K;
  constexpr int C = CPT > 0 ? CPT : 1;
  float v[C][8];
  float amax = 0.f;
  if constexpr (CPT > 0) {
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int64_t i = ((int64_t)threadIdx.x + c * 256) * 8;
      if (i < K) {
        load8<T>(xr + i, v[c]);
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[c][k]));
      }
    }
  } else {
    for (int64_t i = (int64_t)threadIdx.x * 8; i < K; i += 256 * 8) {
      load8<T>(xr + i, v[0]);
#pragma unroll
      for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[0][k]));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float a = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) a = fmaxf(a, red[w]);
  const float recip = 1.0f / kPos;  // binary32 reciprocal, folded at compile time
  const float scale = fmaxf(a, 1e-8f) * recip;
  if (threadIdx.x == 0) scales[row] = scale;
  auto emit = [&](const float (&vv)[8], int64_t i) {
    uint32_t word[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float q = rintf(__fdiv_rn(vv[k], scale));
      q = fminf(fmaxf(q, kNeg), kPos);
      const uint32_t field = (uint32_t)((int)q) & ((1u << BITS) - 1);
      const int bit = k * BITS;
      word[bit >> 5] |= field << (bit & 31);
    }
    if constexpr (BITS == 8) {
      *reinterpret_cast<uint2*>(codes + row * K + i) = make_uint2(word[0], word[1]);
    } else {
      *reinterpret_cast<uint32_t*>(codes + (row * K + i) / 2) = word[0];
    }
  };
  if constexpr (CPT > 0) {
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int64_t i = ((int64_t)threadIdx.x + c * 256) * 8;
      if (i < K) emit(v[c], i);
    }
  } else {
    for (int64_t i = (int64_t)threadIdx.x * 8; i < K; i += 256 * 8) {
      load8<T>(xr + i, v[0]);
      emit(v[0], i);
    }
  }
}

template <typename T, int BITS>
static cudaError_t launch_rows_t(const T* x, int64_t M, int64_t K, uint8_t* codes, float* scales, cudaStream_t s) {
  const unsigned grid = (unsigned)M;
  if (K <= 2048) (void)launch_pdl(quantize_rows_kernel<T, 1, BITS>, dim3(grid), 256, 0, s, x, codes, scales, K);
  else if (K <= 4096) (void)launch_pdl(quantize_rows_kernel<T, 2, BITS>, dim3(grid), 256, 0, s, x, codes, scales, K);
  else if (K <= 8192) (void)launch_pdl(quantize_rows_kernel<T, 4, BITS>, dim3(grid), 256, 0, s, x, codes, scales, K);
  else (void)launch_pdl(quantize_rows_kernel<T, 0, BITS>, dim3(grid), 256, 0, s, x, codes, scales, K);
  return cudaGetLastError();
}

template <int BITS>
static cudaError_t launch_rows_bits(const void* x, int dtype, int64_t M, int64_t K, uint8_t* codes, float* scales,
                                    cudaStream_t stream) {
  switch (dtype) {
    case kDtBF16: return launch_rows_t<__nv_bfloat16, BITS>(reinterpret_cast<const __nv_bfloat16*>(x), M, K, codes, scales, stream);
    case kDtF16: return launch_rows_t<__half, BITS>(reinterpret_cast<const __half*>(x), M, K, codes, scales, stream);
    default: return launch_rows_t<float, BITS>(reinterpret_cast<const float*>(x), M, K, codes, scales, stream);
  }
}

cudaError_t launch_quantize_rows(const void* x, int dtype, int64_t M, int64_t K, int bits, uint8_t* codes,
                                 float* scales, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  return bits == 4 ? launch_rows_bits<4>(x, dtype, M, K, codes, scales, stream)
                   : launch_rows_bits<8>(x, dtype, M, K, codes, scales, stream);
}

cudaError_t launch_weight_codes(const void* w, int dtype, int64_t N, int64_t K, int W, int A, const float* clip,
                                int8_t* codes, float* scale, cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  switch (dtype) {
    case kDtBF16:
      weight_codes_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(w), K, W, A, clip,
                                                           codes, scale);
      break;
    case kDtF16:
      weight_codes_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const __half*>(w), K, W, A, clip, codes,
                                                           scale);
      break;
    default:
      weight_codes_kernel<<<(unsigned)N, 256, 0, stream>>>(reinterpret_cast<const float*>(w), K, W, A, clip, codes,
                                                           scale);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_pack_rows(const int8_t* q, int64_t total_bytes, int bits, uint8_t* packed, int num_sms,
                             cudaStream_t stream) {
  if (total_bytes == 0) return cudaSuccess;
  int64_t blocks = (total_bytes + 255) / 256;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  pack_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(q, total_bytes, bits, packed);
  return cudaGetLastError();
}

}  // namespace actune
