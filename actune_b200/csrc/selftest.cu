// Failure-detection self-test and the wait-limit control (declared in
// include/actune_b200.h).
//
// Every pipeline wait in this library is bounded (mbar_wait in common.cuh): when a
// barrier phase does not complete within g_actune_wait_limit_ns, the waiting thread
// records ACTUNE_DEV_TIMEOUT and the wait site in the device error word and the
// kernel runs to its end instead of hanging the GPU.  The self-test kernel below
// exercises exactly that path: it waits, with the same primitive the GEMM uses, on
// a barrier that nothing ever arrives on.  It holds no tensor memory and issues no
// bulk copies, so giving up leaves nothing in flight.
#include "actune_b200.h"
#include "kernels.cuh"

namespace actune {
namespace {

__global__ void wait_timeout_probe_kernel(int site) {
  __shared__ __align__(8) uint64_t never_completes;
  if (threadIdx.x == 0) {
    mbar_init(&never_completes, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // Phase 0 needs one arrival, and no thread arrives: the wait runs out.
  if (threadIdx.x == 0) (void)mbar_wait(&never_completes, 0, site);
}

}  // namespace
}  // namespace actune

using namespace actune;

extern "C" {

int actune_set_wait_limit_ns(uint64_t ns) {
  if (ns < 1000000ull || ns > 60000000000ull) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ACTUNE_ERR_CUDA;
  const unsigned long long v = ns;
  if (cudaMemcpyToSymbol(g_actune_wait_limit_ns, &v, sizeof(v)) != cudaSuccess) return ACTUNE_ERR_CUDA;
  return ACTUNE_OK;
}

int actune_wait_limit_ns(uint64_t* ns) {
  if (ns == nullptr) return ACTUNE_ERR_INVALID_VALUE;
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, g_actune_wait_limit_ns, sizeof(v)) != cudaSuccess) return ACTUNE_ERR_CUDA;
  *ns = v;
  return ACTUNE_OK;
}

int actune_selftest_wait_timeout(int site, void* stream) {
  if (site <= 0) return ACTUNE_ERR_INVALID_VALUE;
  int major = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return ACTUNE_ERR_CUDA;
  if (major != 10) return ACTUNE_ERR_DEVICE;
  wait_timeout_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(site);
  return cudaGetLastError() == cudaSuccess ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

}  // extern "C"
