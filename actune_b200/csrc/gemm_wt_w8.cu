// Instantiations of the weights-in-TMEM group-64 GEMM for W = 8 (all A, all token tiles).
#include "gemm_wt.cuh"

namespace actune {

template <int W, int A, int BT>
cudaError_t launch_wt_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                           cudaStream_t stream) {
  using C = WtCfg<W, A, BT>;
  const bool dots = p.dots != nullptr;
  auto kernel = dots ? wt_gemm_kernel<W, A, BT, true> : wt_gemm_kernel<W, A, BT, false>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[2][64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dots][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dots][dev] = true;
  }
  const dim3 grid((p.M + BT - 1) / BT, (p.N + C::BM - 1) / C::BM);
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}

#define ACTUNE_INST(A, BT)                                                                                  \
  template cudaError_t launch_wt_gemm<8, A, BT>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, \
                                                cudaStream_t);
ACTUNE_INST(2, 16) ACTUNE_INST(2, 32) ACTUNE_INST(2, 64) ACTUNE_INST(2, 128)
ACTUNE_INST(4, 16) ACTUNE_INST(4, 32) ACTUNE_INST(4, 64) ACTUNE_INST(4, 128)
ACTUNE_INST(8, 16) ACTUNE_INST(8, 32) ACTUNE_INST(8, 64) ACTUNE_INST(8, 128)
#undef ACTUNE_INST

}  // namespace actune
