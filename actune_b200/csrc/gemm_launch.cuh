// Host launchers of the group-64 tcgen05 GEMM family (one-CTA, two-CTA, row-scaled
// and persistent forms).  Each gemm_w{2,4,8}.cu includes this file and instantiates
// the launchers for its weight width with ACTUNE_INSTANTIATE_GEMM(W), so the three
// widths compile in parallel from one definition.
#pragma once

#include "gemm_group64_persistent.cuh"

namespace actune {

template <int W, int A, int BN>
cudaError_t launch_group64_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                cudaStream_t stream, bool pdl) {
  using C = Group64Cfg<W, A, BN>;
  const bool dots = p.dots != nullptr;
  constexpr auto k_dots = group64_gemm_kernel<W, A, BN, true>;
  constexpr auto k_out = group64_gemm_kernel<W, A, BN, false>;
  const cudaError_t e = dots ? ensure_smem_limit<k_dots>(C::SMEM_BYTES) : ensure_smem_limit<k_out>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  auto kernel = dots ? k_dots : k_out;
  const int n_end = p.n_end > 0 ? p.n_end : p.N;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (n_end - p.n_base + BN - 1) / BN);
  if (pdl) return launch_pdl(kernel, grid, C::TILE_THREADS, C::SMEM_BYTES, stream, tm_act, tm_wgt, p);
  kernel<<<grid, C::TILE_THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}

// Two CTAs per SM (no debug-dots form: the one-CTA kernel exports dots).
template <int W, int A, int BN>
cudaError_t launch_group64_gemm_x2(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                   cudaStream_t stream) {
  using C = Group64Cfg<W, A, BN, 2>;
  if (p.dots != nullptr) return cudaErrorInvalidValue;
  constexpr auto kernel = group64_gemm_kernel<W, A, BN, false, false, 2>;
  const cudaError_t e = ensure_smem_limit<kernel>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (p.N + BN - 1) / BN);
  kernel<<<grid, C::TILE_THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}

template <int W, int A, int BN>
cudaError_t launch_group64_tokenwise(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                     cudaStream_t stream, bool pdl) {
  using C = Group64Cfg<W, A, BN>;
  constexpr auto kernel = group64_gemm_kernel<W, A, BN, false, true>;
  const cudaError_t e = ensure_smem_limit<kernel>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int n_end = p.n_end > 0 ? p.n_end : p.N;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (n_end - p.n_base + BN - 1) / BN);
  if (pdl) return launch_pdl(kernel, grid, C::TILE_THREADS, C::SMEM_BYTES, stream, tm_act, tm_wgt, p);
  kernel<<<grid, C::TILE_THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}

template <int W, int A, int BN, bool TW>
cudaError_t launch_group64_persistent(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const CUtensorMap& tm_out,
                                      const GemmParams& p, int num_sms, cudaStream_t stream) {
  using C = PersistCfg<W, A, BN, TW>;
  constexpr auto kernel = group64_gemm_persistent_kernel<W, A, BN, TW>;
  const cudaError_t e = ensure_smem_limit<kernel>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + 127) / 128) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kernel<<<grid, Group64Cfg<W, A, BN>::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, tm_out, p);
  return cudaGetLastError();
}

}  // namespace actune

// Every launcher of one weight width W: one-CTA and two-CTA tiles of 32/64/128
// weight rows for A in {2, 4, 8}; the row-scaled mode for A in {4, 8}; persistent
// tiles of 64/128 rows (group-64 for all A, row-scaled for A in {4, 8}).
#define ACTUNE_GEMM_INST_ONE(W, A, BN)                                                                     \
  template cudaError_t launch_group64_gemm<W, A, BN>(const CUtensorMap&, const CUtensorMap&,              \
                                                     const GemmParams&, cudaStream_t, bool);               \
  template cudaError_t launch_group64_gemm_x2<W, A, BN>(const CUtensorMap&, const CUtensorMap&,           \
                                                        const GemmParams&, cudaStream_t);
#define ACTUNE_GEMM_INST_ROWWISE(W, A, BN)                                                                 \
  template cudaError_t launch_group64_tokenwise<W, A, BN>(const CUtensorMap&, const CUtensorMap&,         \
                                                          const GemmParams&, cudaStream_t, bool);
#define ACTUNE_GEMM_INST_PERSIST(W, A, BN, TW)                                                             \
  template cudaError_t launch_group64_persistent<W, A, BN, TW>(const CUtensorMap&, const CUtensorMap&,    \
                                                               const CUtensorMap&, const GemmParams&, int, \
                                                               cudaStream_t);
#define ACTUNE_INSTANTIATE_GEMM(W)                                                                          \
  namespace actune {                                                                                        \
  ACTUNE_GEMM_INST_ONE(W, 2, 32) ACTUNE_GEMM_INST_ONE(W, 2, 64) ACTUNE_GEMM_INST_ONE(W, 2, 128)             \
  ACTUNE_GEMM_INST_ONE(W, 4, 32) ACTUNE_GEMM_INST_ONE(W, 4, 64) ACTUNE_GEMM_INST_ONE(W, 4, 128)             \
  ACTUNE_GEMM_INST_ONE(W, 8, 32) ACTUNE_GEMM_INST_ONE(W, 8, 64) ACTUNE_GEMM_INST_ONE(W, 8, 128)             \
  ACTUNE_GEMM_INST_ROWWISE(W, 4, 32) ACTUNE_GEMM_INST_ROWWISE(W, 4, 64) ACTUNE_GEMM_INST_ROWWISE(W, 4, 128) \
  ACTUNE_GEMM_INST_ROWWISE(W, 8, 32) ACTUNE_GEMM_INST_ROWWISE(W, 8, 64) ACTUNE_GEMM_INST_ROWWISE(W, 8, 128) \
  ACTUNE_GEMM_INST_PERSIST(W, 2, 64, false) ACTUNE_GEMM_INST_PERSIST(W, 2, 128, false)                      \
  ACTUNE_GEMM_INST_PERSIST(W, 4, 64, false) ACTUNE_GEMM_INST_PERSIST(W, 4, 128, false)                      \
  ACTUNE_GEMM_INST_PERSIST(W, 8, 64, false) ACTUNE_GEMM_INST_PERSIST(W, 8, 128, false)                      \
  ACTUNE_GEMM_INST_PERSIST(W, 4, 64, true) ACTUNE_GEMM_INST_PERSIST(W, 4, 128, true)                        \
  ACTUNE_GEMM_INST_PERSIST(W, 8, 64, true) ACTUNE_GEMM_INST_PERSIST(W, 8, 128, true)                        \
  }
