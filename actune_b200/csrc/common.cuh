// Shared device helpers for the group-64 packed-integer path (sm_100a only).
//
// Everything that waits (mbarrier phases) waits with a time limit: after
// g_actune_wait_limit_ns without progress the waiting thread records an error code in
// g_actune_error and returns false, so a broken pipeline ends the kernel with
// an error status the host can read (actune_device_error) instead of hanging
// the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "actune_b200 kernels are written for sm_100a (Blackwell) only"
#endif

namespace actune {

// Raises `Kernel`'s dynamic shared-memory limit to `bytes` on the current device,
// once per device.  Safe for concurrent first calls from several host threads
// (std::call_once per device); devices beyond the first kMaxDevices ordinals are
// refused with cudaErrorInvalidDevice rather than left unconfigured.
constexpr int kMaxDevices = 64;
template <auto Kernel>
cudaError_t ensure_smem_limit(int bytes) {
  static std::once_flag once[kMaxDevices];
  static cudaError_t status[kMaxDevices];
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [&] {
    status[dev] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return status[dev];
}

// ---------------------------------------------------------------------------
// Device error word (first error wins).  Codes are the ACTUNE_DEV_* values in
// include/actune_b200.h; `g_actune_error_site` records which wait gave up.
// ---------------------------------------------------------------------------
extern __device__ int g_actune_error;
extern __device__ int g_actune_error_site;
// Time limit of every pipeline wait on this device (ns).  Legitimate waits are
// microseconds; the default is 2 s, and actune_set_wait_limit_ns changes it (the
// failure-detection self-test shortens it so that its deliberately abandoned wait
// ends quickly).
extern __device__ unsigned long long g_actune_wait_limit_ns;
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;

__device__ __forceinline__ void report_error(int code, int site) {
  if (atomicCAS(&g_actune_error, 0, code) == 0) atomicExch(&g_actune_error_site, site);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes (woken by the barrier) or about `hint_ns` elapse, instead of
// spinning and taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms per sleep; the 2 s limit is checked between sleeps

// Wait for the phase with the given parity to complete; false after the limit
// (g_actune_wait_limit_ns, checked every 16 sleeps).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait_sleep(addr, parity, kSuspendHintNs)) return true;
    if ((spin & 15) == 15) {
      const uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > g_actune_wait_limit_ns) {
        report_error(1 /* ACTUNE_DEV_TIMEOUT */, site);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this project)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Same with the destination and barrier given as shared-memory addresses.
// Prefetch a 2-D box into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared -> global tiled store, tracked in this thread's bulk async-group.  The
// tile is clipped to the tensor's bounds (rows past M, columns past N are not
// written); x is in elements of the map (bytes here) and never negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared memory read by this thread's earlier bulk stores may be rewritten.
__device__ __forceinline__ void bulk_wait_group_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// This thread's earlier bulk stores are complete.
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Programmatic dependent launch: allow a dependent launch to start / wait for the
// grids this one depends on (both return at once when there are none).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Every kernel on the hot path is launched with programmatic stream serialization:
// it may start while the kernel before it in the stream is still running (once all
// of that kernel's CTAs have started and signalled), does what does not depend on
// it (barrier set-up, tensor-memory allocation, descriptor prefetch, loads of the
// resident weights), then waits in griddep_wait() before it reads anything the
// previous kernel may have written or writes any global memory (an output buffer
// may reuse memory the previous kernel still reads).  After a kernel that never
// signals (a library kernel) the launch starts when that kernel completes.
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, int threads, int smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Prologue of a dependent-launched kernel that reads its inputs from the start:
// wait for the previous kernel, then let the next one start.
__device__ __forceinline__ void griddep_enter() {
  griddep_wait();
  griddep_launch_dependents();
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (cta_group::1)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 op issued so far by this thread completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mma_commit_u32(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Store one 32-bit value to 32 lanes x N columns (N = 8, 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_fill(uint32_t taddr, uint32_t v) {
  if constexpr (N == 32) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(v)
        : "memory");
  } else if constexpr (N == 16) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
                     taddr),
                 "r"(v)
                 : "memory");
  } else {
    static_assert(N == 8, "tmem_fill width");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
                 : "memory");
  }
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 4 columns of 32-bit -> 4 registers per thread.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// 32 lanes x 8 columns of 32-bit -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// 32 lanes x 16 columns of 32-bit -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 columns of 32-bit -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// UMMA shared-memory matrix descriptor for a K-major operand stored in the
// canonical 128-byte-swizzled layout (8-row x 128-byte atoms, atoms 1024 B
// apart): start address, LBO = 16 B (unused for swizzled K-major), SBO = 1024 B,
// descriptor version 1, layout type SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor: kind::i8, D = s32, A = B = s8, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4)                        // D format: S32
         | (1u << 7) | (1u << 10)         // A, B: signed 8-bit
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100): two lanes of IEEE binary32, RNE, one issue.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Exact int32 -> fp32 for |v| < 2^22: the bit pattern 0x4B400000 + v is the
// binary32 number 1.5*2^23 + v (ulp 1 in that binade); subtracting 1.5*2^23
// afterwards is exact.  Used by the decode and weights-in-TMEM kernels; the
// group-64 GEMM epilogue measured faster with the hardware conversion.
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagicValue = 12582912.0f;

// ---------------------------------------------------------------------------
// Sub-byte unpack.  A code c of `bits` bits is placed in the top bits of a
// byte: the int8 value is c * 2^(8-bits).  The extra power of two is removed
// exactly in the fp32 epilogue (scale * 2^-(shift)).
// ---------------------------------------------------------------------------
// 4 packed bytes (8 int4 codes, element 2j in the low nibble of byte j) -> 8 bytes.
__device__ __forceinline__ uint2 unpack_w4_word(uint32_t x) {
  const uint32_t lo = (x << 4) & 0xF0F0F0F0u;
  const uint32_t hi = x & 0xF0F0F0F0u;
  return make_uint2(__byte_perm(lo, hi, 0x5140), __byte_perm(lo, hi, 0x7362));
}

// Group-64 activation quantization of one lane's 8 consecutive values, the group
// spread over 8 consecutive lanes of the warp (lanes 8s .. 8s+7, in K order; all 32
// lanes must call it together).  Restates actune/kernels/grouped.py:55-71:
//   scale = max(absmax, 1e-8) / (2^(A-1) - 1)               IEEE division
//   code  = clamp(rint(x / scale), -2^(A-1), 2^(A-1) - 1)    IEEE division, RNE
// and packs the lane's 8 codes little-endian, code i at bit i*OUT of `word`: the
// A-bit packed layout (OUT = A) or one int8 per code (OUT = 8, the layout the
// W=8 / A=8 GEMM reads, whatever A).  Returns the group's scale (the same in all 8
// lanes).
template <int A, int OUT = A>
__device__ __forceinline__ float quantize_lane8(const float (&v)[8], uint32_t (&word)[2]) {
  constexpr float kPositive = float((1 << (A - 1)) - 1);
  constexpr float kLo = -float(1 << (A - 1));
  static_assert(OUT == A || OUT == 8, "codes are stored at A bits or as int8");
  constexpr int kMask = (1 << OUT) - 1;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), kPositive);
  word[0] = word[1] = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float q = rintf(__fdiv_rn(v[i], scale));
    q = fminf(fmaxf(q, kLo), kPositive);
    const uint32_t field = (uint32_t)((int)q) & kMask;
    const int bit = i * OUT;
    word[bit >> 5] |= field << (bit & 31);
  }
  return scale;
}

// Stores a lane's packed codes (8*A bits) at dst.
template <int A>
__device__ __forceinline__ void store_lane_codes(uint8_t* dst, const uint32_t (&word)[2]) {
  if constexpr (A == 8) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(word[0], word[1]);
  } else if constexpr (A == 4) {
    *reinterpret_cast<uint32_t*>(dst) = word[0];
  } else {
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)word[0];
  }
}

// 4 packed bytes (16 int2 codes, element 4j+i at bits 2i of byte j) -> 16 bytes.
__device__ __forceinline__ uint4 unpack_w2_word(uint32_t x) {
  const uint32_t t0 = (x << 6) & 0xC0C0C0C0u;
  const uint32_t t1 = (x << 4) & 0xC0C0C0C0u;
  const uint32_t t2 = (x << 2) & 0xC0C0C0C0u;
  const uint32_t t3 = x & 0xC0C0C0C0u;
  const uint32_t u0 = __byte_perm(t0, t1, 0x5140), u1 = __byte_perm(t0, t1, 0x7362);
  const uint32_t v0 = __byte_perm(t2, t3, 0x5140), v1 = __byte_perm(t2, t3, 0x7362);
  return make_uint4(__byte_perm(u0, v0, 0x5410), __byte_perm(u0, v0, 0x7632), __byte_perm(u1, v1, 0x5410),
                    __byte_perm(u1, v1, 0x7632));
}

}  // namespace actune

namespace actune {
// Named barrier among `count` threads (multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also returns the AND of `pred` over the `count` threads.
__device__ __forceinline__ bool named_barrier_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
}  // namespace actune
