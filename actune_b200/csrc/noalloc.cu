// Allocation-free variant of actune_grouped_linear (declared in include/actune_b200.h).
//
// Some callers cannot allocate device memory at the point where they run the
// linear: hosts whose device memory is owned and budgeted by another allocator
// (a serving runtime with a fixed memory pool, a framework that must account
// for every allocation), and control loops that must not allocate once they
// are running (allocation latency, fragmentation or an out-of-memory error in
// the middle of an episode).  For them this entry point keeps the activation
// scratch -- packed codes and group scales of one call -- in a fixed array in
// this library's device memory, so the caller passes only inputs and outputs.
#include "actune_b200.h"
#include "kernels.cuh"

// The scratch itself.  In host code `g_noalloc_scratch` is only a stand-in
// symbol, not a device address: the device address is looked up with
// cudaGetSymbolAddress below, with the device current.  Every device that loads
// this library holds these bytes until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[ACTUNE_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch on the current device.  Looked up on every
// call (a table lookup once the library's module is loaded on the device), so a
// context that was reset and re-created gets the array's new address instead of
// a stale one.  The first call on a device also loads the module there, which is
// why that first call must come before any stream capture.
int scratch_address(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return ACTUNE_ERR_CUDA;
  *out = p;
  return ACTUNE_OK;
}

}  // namespace

extern "C" int actune_grouped_linear_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* w,
                                             const float* w_scale, const void* bias, int bias_dtype, int64_t N,
                                             int W, int A, void* out, int out_dtype, int variant, void* stream) {
  if (M < 0 || K <= 0 || K % 64 || (A != 2 && A != 4 && A != 8)) return ACTUNE_ERR_INVALID_VALUE;
  // Requests whose packed activations and scales do not fit the fixed scratch
  // are refused before anything is launched.
  if (actune_grouped_linear_workspace_size(M, K, A) > (size_t)ACTUNE_NOALLOC_SCRATCH_BYTES) return ACTUNE_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != ACTUNE_OK) return rc;
  // Nothing in the scratch needs to start at zero: the quantizer writes every
  // packed byte and scale the GEMM of the same call reads (rows beyond M are
  // never read from memory; the GEMM's tensor map bounds them).
  return actune_grouped_linear(x, x_dtype, M, K, w, w_scale, bias, bias_dtype, N, W, A, out, out_dtype, scratch,
                               (size_t)ACTUNE_NOALLOC_SCRATCH_BYTES, variant, stream);
}
