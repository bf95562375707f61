// Instantiations of the group-64 tcgen05 GEMM for W = 4 (all A, all tile widths).
#include "gemm_group64_persistent.cuh"

namespace actune {

template <int W, int A, int BN>
cudaError_t launch_group64_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                cudaStream_t stream, bool pdl) {
  using C = Group64Cfg<W, A, BN>;
  const bool dots = p.dots != nullptr;
  auto kernel = dots ? group64_gemm_kernel<W, A, BN, true> : group64_gemm_kernel<W, A, BN, false>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[2][64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dots][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dots][dev] = true;
  }
  const int n_end = p.n_end > 0 ? p.n_end : p.N;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (n_end - p.n_base + BN - 1) / BN);
  if (!pdl) {
    kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_act, tm_wgt, p);
}

// Two CTAs per SM (no debug-dots form: the one-CTA kernel exports dots).
template <int W, int A, int BN>
cudaError_t launch_group64_gemm_x2(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                   cudaStream_t stream) {
  using C = Group64Cfg<W, A, BN, 2>;
  if (p.dots != nullptr) return cudaErrorInvalidValue;
  auto kernel = group64_gemm_kernel<W, A, BN, false, false, 2>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const dim3 grid((p.M + C::BM - 1) / C::BM, (p.N + BN - 1) / BN);
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}

template <int W, int A, int BN>
cudaError_t launch_group64_tokenwise(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                     cudaStream_t stream, bool pdl) {
  using C = Group64Cfg<W, A, BN>;
  auto kernel = group64_gemm_kernel<W, A, BN, false, true>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int n_end = p.n_end > 0 ? p.n_end : p.N;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (n_end - p.n_base + BN - 1) / BN);
  if (!pdl) {
    kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_act, tm_wgt, p);
}

template cudaError_t launch_group64_tokenwise<4, 4, 32>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_group64_tokenwise<4, 4, 64>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_group64_tokenwise<4, 4, 128>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_group64_tokenwise<4, 8, 32>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_group64_tokenwise<4, 8, 64>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_group64_tokenwise<4, 8, 128>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t, bool);

template <int W, int A, int BN, bool TW>
cudaError_t launch_group64_persistent(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const CUtensorMap& tm_out,
                                      const GemmParams& p, int num_sms, cudaStream_t stream) {
  using C = PersistCfg<W, A, BN, TW>;
  auto kernel = group64_gemm_persistent_kernel<W, A, BN, TW>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int tiles = ((p.M + 127) / 128) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kernel<<<grid, Group64Cfg<W, A, BN>::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, tm_out, p);
  return cudaGetLastError();
}

#define ACTUNE_PERSIST(A, BN, TW)                                                                             \
  template cudaError_t launch_group64_persistent<4, A, BN, TW>(const CUtensorMap&, const CUtensorMap&,     \
                                                               const CUtensorMap&, const GemmParams&, int,   \
                                                               cudaStream_t);
ACTUNE_PERSIST(2, 64, false)
ACTUNE_PERSIST(2, 128, false)
ACTUNE_PERSIST(4, 64, false)
ACTUNE_PERSIST(4, 128, false)
ACTUNE_PERSIST(8, 64, false)
ACTUNE_PERSIST(8, 128, false)
ACTUNE_PERSIST(4, 64, true)
ACTUNE_PERSIST(4, 128, true)
ACTUNE_PERSIST(8, 64, true)
ACTUNE_PERSIST(8, 128, true)
#undef ACTUNE_PERSIST

#define ACTUNE_INST(A, BN)                                                                                  \
  template cudaError_t launch_group64_gemm<4, A, BN>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, \
                                                     cudaStream_t, bool);                                            \
  template cudaError_t launch_group64_gemm_x2<4, A, BN>(const CUtensorMap&, const CUtensorMap&,                   \
                                                        const GemmParams&, cudaStream_t);
ACTUNE_INST(2, 32)
ACTUNE_INST(2, 64)
ACTUNE_INST(2, 128)
ACTUNE_INST(4, 32)
ACTUNE_INST(4, 64)
ACTUNE_INST(4, 128)
ACTUNE_INST(8, 32)
ACTUNE_INST(8, 64)
ACTUNE_INST(8, 128)
#undef ACTUNE_INST

}  // namespace actune
