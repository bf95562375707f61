// extern "C" boundary of libactune_b200.so (declared in include/actune_b200.h).
//
// Validation mirrors the reference's checks (actune/kernels/grouped_native.cu:92-105,
// grouped.py:117-119): bit widths in {2,4,8}, K a multiple of 64, matching
// shapes; violations return a status instead of throwing across the ABI.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "actune_b200.h"
#include "kernels.cuh"

namespace actune {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::atomic<int> state{0};  // 0 unknown, 1 ok, 2 unsupported
  int num_sms = 0;
};
DeviceInfo g_devices[kMaxDevices];
std::mutex g_init_mutex;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ACTUNE_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return ACTUNE_ERR_DEVICE;
  DeviceInfo& d = g_devices[dev];
  int st = d.state.load(std::memory_order_acquire);
  if (st == 0) {
    std::lock_guard<std::mutex> lock(g_init_mutex);
    st = d.state.load(std::memory_order_relaxed);
    if (st == 0) {
      int major = 0, minor = 0, sms = 0;
      if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return ACTUNE_ERR_CUDA;
      if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || fn == nullptr)
          return ACTUNE_ERR_CUDA;
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
      d.num_sms = sms;
      st = (major == 10 && minor == 0) ? 1 : 2;
      d.state.store(st, std::memory_order_release);
    }
  }
  if (st != 1) return ACTUNE_ERR_DEVICE;
  *dev_out = dev;
  return ACTUNE_OK;
}

// CUDA error behind the last ACTUNE_ERR_CUDA returned on this thread.
thread_local int g_last_cuda_error = 0;
int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return ACTUNE_OK;
  g_last_cuda_error = (int)e;
  return ACTUNE_ERR_CUDA;
}

bool valid_bits(int b) { return b == 2 || b == 4 || b == 8; }
bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
bool valid_float_dtype(int t) { return t == ACTUNE_DTYPE_F32 || t == ACTUNE_DTYPE_F16 || t == ACTUNE_DTYPE_BF16; }
size_t dtype_size(int t) { return t == ACTUNE_DTYPE_F32 ? 4 : 2; }

// 2D uint8 tensor map [rows, row_bytes] with a box of [box_rows, box_bytes]; the
// shared-memory swizzle span equals the box row width (32, 64 or 128 bytes) or none.
enum class Swz { None, B32, B64, B128 };
CUtensorMapSwizzle swizzle_mode(Swz z) {
  switch (z) {
    case Swz::B32: return CU_TENSOR_MAP_SWIZZLE_32B;
    case Swz::B64: return CU_TENSOR_MAP_SWIZZLE_64B;
    case Swz::B128: return CU_TENSOR_MAP_SWIZZLE_128B;
    default: return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}
int encode_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_bytes, int box_rows,
               Swz swz) {
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_mode(swz),
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

// Token tile of the weights-in-TMEM kernel: the smallest of 16/32/64/128 that
// holds M, else 128.
int pick_wt(int variant, int64_t M) {
  switch (variant) {
    case ACTUNE_VARIANT_WT16: return 16;
    case ACTUNE_VARIANT_WT32: return 32;
    case ACTUNE_VARIANT_WT64: return 64;
    case ACTUNE_VARIANT_WT128: return 128;
    default: break;
  }
  return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
}

bool is_wt_variant(int variant) { return variant >= ACTUNE_VARIANT_WT16 && variant <= ACTUNE_VARIANT_WT128; }
bool is_x2_variant(int variant) { return variant >= ACTUNE_VARIANT_BN32X2 && variant <= ACTUNE_VARIANT_BN128X2; }
bool is_persistent_variant(int variant) {
  return variant == ACTUNE_VARIANT_BN64P || variant == ACTUNE_VARIANT_BN128P;
}

// The persistent kernel stores 16-bit outputs with TMA: rows of N*2 bytes at a
// 16-byte aligned base and pitch.
bool persistent_ok(const void* out, int out_dtype, int64_t N) {
  return (out_dtype == kDtBF16 || out_dtype == kDtF16) && N % 8 == 0 && N >= 64 && aligned(out, 16);
}

// 3-D uint8 tensor map over a [rows, row_bytes] matrix (row_bytes a multiple of
// 128) seen as (128-byte block, row, block index): a box of {128, box_rows,
// box_blocks} lands as [block][row][128 B], 128-byte swizzled.
int encode_map_blocks(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_rows,
                      int box_blocks) {
  const cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(row_bytes / 128)};
  const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 128};
  const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, (cuuint32_t)box_blocks};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

// 2-D fp32 tensor map over a [rows, cols] row-major matrix (cols a multiple of 4),
// no swizzle; boxes of {box_cols, box_rows}.
int encode_map_f32(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * 4)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ACTUNE_OK : ACTUNE_ERR_CUDA;
}

bool use_gemv(int variant, int64_t M) {
  return variant == ACTUNE_VARIANT_GEMV || (variant == ACTUNE_VARIANT_AUTO && M <= 32);
}

int pick_bn(int variant, int64_t M, int64_t N, int num_sms) {
  switch (variant) {
    case ACTUNE_VARIANT_BN32: return 32;
    case ACTUNE_VARIANT_BN64: return 64;
    case ACTUNE_VARIANT_BN128: return 128;
    case ACTUNE_VARIANT_BN32X2: return 32;
    case ACTUNE_VARIANT_BN64X2: return 64;
    case ACTUNE_VARIANT_BN128X2: return 128;
    case ACTUNE_VARIANT_BN64P: return 64;
    case ACTUNE_VARIANT_BN128P: return 128;
    default: break;
  }
  // Minimise waves x per-tile time, modelled as (BN + 64) (a tile has a fixed
  // cost for its 128-row activation stream and epilogue besides its BN weight
  // rows); prefer wider tiles on ties.
  const int64_t mt = (M + 127) / 128;
  int best = 128;
  int64_t best_cost = INT64_MAX;
  for (int bn : {128, 64, 32}) {
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + num_sms - 1) / num_sms;
    const int64_t cost = waves * (bn + 64);
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <int W, int A>
cudaError_t dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p, cudaStream_t s,
                        bool pdl = false) {
  switch (bn) {
    case 32: return launch_group64_gemm<W, A, 32>(ta, tw, p, s, pdl);
    case 64: return launch_group64_gemm<W, A, 64>(ta, tw, p, s, pdl);
    default: return launch_group64_gemm<W, A, 128>(ta, tw, p, s, pdl);
  }
}

template <int W, int A>
cudaError_t dispatch_bn_x2(int bn, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                           cudaStream_t s) {
  switch (bn) {
    case 32: return launch_group64_gemm_x2<W, A, 32>(ta, tw, p, s);
    case 64: return launch_group64_gemm_x2<W, A, 64>(ta, tw, p, s);
    default: return launch_group64_gemm_x2<W, A, 128>(ta, tw, p, s);
  }
}

template <int W, int A>
cudaError_t dispatch_wt(int bt, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p, cudaStream_t s) {
  switch (bt) {
    case 16: return launch_wt_gemm<W, A, 16>(ta, tw, p, s);
    case 32: return launch_wt_gemm<W, A, 32>(ta, tw, p, s);
    case 64: return launch_wt_gemm<W, A, 64>(ta, tw, p, s);
    default: return launch_wt_gemm<W, A, 128>(ta, tw, p, s);
  }
}

cudaError_t dispatch_wt_gemm(int W, int A, int bt, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                             cudaStream_t s) {
#define ACTUNE_CASE(WW, AA) \
  if (W == WW && A == AA) return dispatch_wt<WW, AA>(bt, ta, tw, p, s);
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

template <int W, int A, bool TW>
cudaError_t dispatch_persistent_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to,
                                   const GemmParams& p, int num_sms, cudaStream_t s) {
  return bn == 64 ? launch_group64_persistent<W, A, 64, TW>(ta, tw, to, p, num_sms, s)
                  : launch_group64_persistent<W, A, 128, TW>(ta, tw, to, p, num_sms, s);
}

cudaError_t dispatch_persistent(int W, int A, bool tw_mode, int bn, const CUtensorMap& ta, const CUtensorMap& tw,
                                const CUtensorMap& to, const GemmParams& p, int num_sms, cudaStream_t s) {
#define ACTUNE_CASE(WW, AA)                                                                              \
  if (W == WW && A == AA && !tw_mode) return dispatch_persistent_bn<WW, AA, false>(bn, ta, tw, to, p, num_sms, s);
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
#define ACTUNE_CASE(WW, AA)                                                                             \
  if (W == WW && A == AA && tw_mode) return dispatch_persistent_bn<WW, AA, true>(bn, ta, tw, to, p, num_sms, s);
  ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

// Wave-tail split of an AUTO GEMM with 128-column tiles: when the tiles leave a
// partial last wave, the whole waves take the first *na128 * 128 columns and the rest
// runs as narrower tiles (the returned width, 32 or 64, whichever fits one wave) in a
// second launch that may start while the first drains.  0: no split.
int wave_tail_split(int64_t M, int64_t N, int sms, int64_t* na128) {
  const int64_t mt = (M + 127) / 128, tiles = mt * ((N + 127) / 128);
  const int64_t na = (tiles - tiles % sms) / mt;
  if (tiles <= sms || tiles % sms == 0 || na <= 0 || na * 128 >= N) return 0;
  const int64_t rest = N - na * 128;
  *na128 = na;
  if (mt * ((rest + 31) / 32) <= sms) return 32;
  if (mt * ((rest + 63) / 64) <= sms) return 64;
  return 0;
}

cudaError_t dispatch_gemm(int W, int A, int bn, bool x2, const CUtensorMap& ta, const CUtensorMap& tw,
                          const GemmParams& p, cudaStream_t s, bool pdl = false) {
#define ACTUNE_CASE(WW, AA) \
  if (W == WW && A == AA)   \
    return x2 ? dispatch_bn_x2<WW, AA>(bn, ta, tw, p, s) : dispatch_bn<WW, AA>(bn, ta, tw, p, s, pdl);
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

int check_gemm_shape(int64_t M, int64_t N, int64_t K, int W, int A) {
  if (!valid_bits(W) || !valid_bits(A)) return ACTUNE_ERR_INVALID_VALUE;
  if (K <= 0 || K % 64 || K > (int64_t(1) << 24)) return ACTUNE_ERR_INVALID_VALUE;
  if (M < 0 || N < 0 || M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31)) return ACTUNE_ERR_INVALID_VALUE;
  return ACTUNE_OK;
}

int run_gemm(const uint8_t* a, const float* a_scale, const uint8_t* w, const float* w_scale, const void* bias,
             int bias_dtype, void* out, int out_dtype, int32_t* dots, int64_t M, int64_t N, int64_t K, int W, int A,
             int variant, cudaStream_t stream) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0 || N == 0) return ACTUNE_OK;
  if (!aligned(a, 16) || !aligned(w, 16)) return ACTUNE_ERR_MISALIGNED;
  if (use_gemv(variant, M)) {
    if (M > 32) return ACTUNE_ERR_INVALID_VALUE;
    CUtensorMap ta, tw, ts;
    const int tok = M <= 16 ? 16 : 32;
    // The split-role kernel loads the stage's activation scales as a tile: 16-byte
    // scale rows at a 16-byte aligned base.  Packed rows of whole 128-byte blocks
    // load as one 3-D box per operand, other rows as one 2-D box per block.
    const bool whole = M <= 16 && (dots != nullptr || ((K / 64) % 4 == 0 && aligned(a_scale, 16)));
    const bool boxes2d = (K * A / 8) % 128 != 0 || (K * W / 8) % 128 != 0;
    if (whole) {
      const int sk = gemv_wide(M, W, dots != nullptr) ? kGemvStageKWide : kGemvStageK;
      if (boxes2d) {
        rc = encode_map(&ta, a, M, K * A / 8, 128, M > 8 ? 16 : 8, Swz::B128);
        if (rc != ACTUNE_OK) return rc;
        rc = encode_map(&tw, w, N, K * W / 8, 128, kGemvRows, Swz::B128);
      } else {
        rc = encode_map_blocks(&ta, a, M, K * A / 8, (int)M, sk * A / 8 / 128);
        if (rc != ACTUNE_OK) return rc;
        rc = encode_map_blocks(&tw, w, N, K * W / 8, kGemvRows, sk * W / 8 / 128);
      }
      if (rc != ACTUNE_OK) return rc;
      ts = ta;  // never read by the dots export
      if (dots == nullptr) rc = encode_map_f32(&ts, a_scale, M, K / 64, sk / 64, (int)M);
    } else {
      rc = encode_map(&ta, a, M, K * A / 8, 128, tok, Swz::B128);
      if (rc != ACTUNE_OK) return rc;
      rc = encode_map(&tw, w, N, K * W / 8, 128, kGemvRows, Swz::B128);
    }
    if (rc != ACTUNE_OK) return rc;
    GemmParams p{};
    p.act_scale = a_scale;
    p.w_scale = w_scale;
    p.bias = bias;
    p.out = out;
    p.dots = dots;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.G = (int)(K / 64);
    p.bias_dtype = bias == nullptr ? kDtNone : bias_dtype;
    p.out_dtype = out_dtype;
    p.out_vec_ok = 0;
    p.gemv_boxes2d = whole && boxes2d;
    return cuda_status(launch_gemv_group64(W, A, ta, tw, whole ? &ts : nullptr, p, g_devices[dev].num_sms, stream));
  }
  const bool wt = is_wt_variant(variant);
  const int bn = wt ? pick_wt(variant, M) : pick_bn(variant, M, N, g_devices[dev].num_sms);
  CUtensorMap ta, tw;
  // Token tile: int8 rows land in the SW128 operand layout; packed sub-byte rows are
  // staged unswizzled for the in-kernel expansion.  A single tile of few tokens loads
  // only its rows (rounded up to 8): the TMA unit spends time on every box row,
  // zero-filled ones included.  The persistent form keeps whole-tile boxes.
  const int a_rows = wt ? bn : (M <= 128 && !is_persistent_variant(variant) ? (int)((M + 7) / 8 * 8) : 128);
  rc = encode_map(&ta, a, M, K * A / 8, A == 8 ? 128 : 16 * A, a_rows, A == 8 ? Swz::B128 : Swz::None);
  if (rc != ACTUNE_OK) return rc;
  if (wt) {
    // Weight tile [128 rows x 16*W bytes] with the swizzle whose span is the row width,
    // read row-per-thread by the converters without bank conflicts.
    rc = encode_map(&tw, w, N, K * W / 8, 16 * W, 128, W == 8 ? Swz::B128 : (W == 4 ? Swz::B64 : Swz::B32));
  } else {
    rc = encode_map(&tw, w, N, K * W / 8, W == 8 ? 128 : 16 * W, bn, W == 8 ? Swz::B128 : Swz::None);
  }
  if (rc != ACTUNE_OK) return rc;
  GemmParams p{};
  p.act_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = out;
  p.dots = dots;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.G = (int)(K / 64);
  p.bias_dtype = bias == nullptr ? kDtNone : bias_dtype;
  p.out_dtype = out_dtype;
  p.out_vec_ok = (N % 8 == 0) && aligned(out, 16);
  p.a_box_rows = wt ? 0 : a_rows;
  if (!wt && dots == nullptr && is_persistent_variant(variant) && persistent_ok(out, out_dtype, N)) {
    CUtensorMap to;
    rc = encode_map(&to, out, M, N * 2, 128, 128, Swz::B128);
    if (rc != ACTUNE_OK) return rc;
    return cuda_status(dispatch_persistent(W, A, false, bn, ta, tw, to, p, g_devices[dev].num_sms, stream));
  }
  // AUTO with 128-column tiles whose last wave is partial: the whole waves as one
  // launch and the remaining columns as narrower tiles in a second launch that may
  // start while the first drains (programmatic dependent launch), so that the
  // partial wave is shorter.  Same arithmetic per element: bit-identical output.
  if (variant == ACTUNE_VARIANT_AUTO && !wt && dots == nullptr && bn == 128) {
    int64_t na = 0;
    const int bn_b = wave_tail_split(M, N, g_devices[dev].num_sms, &na);
    if (bn_b > 0) {
      CUtensorMap tw_b;
      rc = encode_map(&tw_b, w, N, K * W / 8, W == 8 ? 128 : 16 * W, bn_b, W == 8 ? Swz::B128 : Swz::None);
      if (rc != ACTUNE_OK) return rc;
      // The first launch starts after the previous kernel completes (normal stream
      // order), so the second, dependent on it, may read the same inputs at once.
      GemmParams pa = p, pb = p;
      pa.n_end = (int)(na * 128);
      pb.n_base = (int)(na * 128);
      cudaError_t e = dispatch_gemm(W, A, 128, false, ta, tw, pa, stream);
      // The narrow tail tiles run the four-group-stage form (a dependent launch like
      // the two-group one).
      if (e == cudaSuccess)
        e = group64_wide_preferred(W, A, bn_b) ? launch_group64_wide(W, A, bn_b, 4, ta, tw_b, pb, stream)
                                               : dispatch_gemm(W, A, bn_b, false, ta, tw_b, pb, stream, true);
      return cuda_status(e);
    }
  }
  // AUTO with a narrow weight tile (few token tiles, narrow outputs): the four-group-
  // stage kernel (same arithmetic, half the per-stage waits and commits per group).
  // The explicit BN32 / BN64 variants keep the two-group-stage kernel.
  if (variant == ACTUNE_VARIANT_AUTO && !wt && dots == nullptr && (bn == 32 || bn == 64) &&
      group64_wide_preferred(W, A, bn)) {
    p.pdl_wait = 1;
    return cuda_status(launch_group64_wide(W, A, bn, 4, ta, tw, p, stream));
  }
  // The debug dots export always runs the one-CTA-per-SM form.  The one-CTA form is a
  // dependent launch: it prefetches its first weight tiles while the previous kernel
  // finishes.
  const bool x2 = is_x2_variant(variant) && dots == nullptr;
  if (!wt && !x2) p.pdl_wait = 1;
  const cudaError_t e = wt ? dispatch_wt_gemm(W, A, bn, ta, tw, p, stream)
                           : dispatch_gemm(W, A, bn, x2, ta, tw, p, stream, !x2);
  return cuda_status(e);
}

// Row-scaled linear (the tokenwise A8 and per-row A4 backends): full-K int32 dots,
// one activation scale per token, `order` 0 = (acc*as)*ws, 1 = acc*(as*ws).
int run_rowwise(const uint8_t* a, int A, const float* a_scale, const uint8_t* w, int W, const float* w_scale,
                const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K, int order,
                int variant, cudaStream_t stream) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0 || N == 0) return ACTUNE_OK;
  if (!aligned(a, 16) || !aligned(w, 16)) return ACTUNE_ERR_MISALIGNED;
  GemmParams p{};
  p.act_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = out;
  p.dots = nullptr;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bias_dtype = bias == nullptr ? kDtNone : bias_dtype;
  p.out_dtype = out_dtype;
  p.rowwise_order = order;
  CUtensorMap ta, tw;
  if (variant == ACTUNE_VARIANT_AUTO && M <= 16) {
    // Decode sizes: the weight-streaming kernel in its row-scaled mode (3-D boxes for
    // rows of whole 128-byte blocks, else one 2-D box per block).
    const int sk = gemv_wide(M, W, false) ? kGemvStageKWide : kGemvStageK;
    p.gemv_boxes2d = (K * A / 8) % 128 != 0 || (K * W / 8) % 128 != 0;
    if (p.gemv_boxes2d) {
      rc = encode_map(&ta, a, M, K * A / 8, 128, M > 8 ? 16 : 8, Swz::B128);
      if (rc != ACTUNE_OK) return rc;
      rc = encode_map(&tw, w, N, K * W / 8, 128, kGemvRows, Swz::B128);
    } else {
      rc = encode_map_blocks(&ta, a, M, K * A / 8, (int)M, sk * A / 8 / 128);
      if (rc != ACTUNE_OK) return rc;
      rc = encode_map_blocks(&tw, w, N, K * W / 8, kGemvRows, sk * W / 8 / 128);
    }
    if (rc != ACTUNE_OK) return rc;
    p.G = (int)(K / 64);
    p.out_vec_ok = 0;
    return cuda_status(launch_gemv_tokenwise(W, A, ta, tw, p, g_devices[dev].num_sms, stream));
  }
  const int bn = pick_bn(variant, M, N, g_devices[dev].num_sms);
  rc = encode_map(&ta, a, M, K * A / 8, A == 8 ? 128 : 16 * A, 128, A == 8 ? Swz::B128 : Swz::None);
  if (rc != ACTUNE_OK) return rc;
  rc = encode_map(&tw, w, N, K * W / 8, W == 8 ? 128 : 16 * W, bn, W == 8 ? Swz::B128 : Swz::None);
  if (rc != ACTUNE_OK) return rc;
  p.G = (int)((K + 63) / 64);  // stages of 128 codes; the zero fill past K adds nothing
  p.out_vec_ok = (N % 8 == 0) && aligned(out, 16);
  if (is_persistent_variant(variant) && persistent_ok(out, out_dtype, N)) {
    CUtensorMap to;
    rc = encode_map(&to, out, M, N * 2, 128, 128, Swz::B128);
    if (rc != ACTUNE_OK) return rc;
    return cuda_status(dispatch_persistent(W, A, true, bn, ta, tw, to, p, g_devices[dev].num_sms, stream));
  }
  auto launch = [&](int bnx, const CUtensorMap& twx, const GemmParams& px, bool pdl) -> cudaError_t {
#define ACTUNE_TW(WW, AA)                                                                      \
  if (W == WW && A == AA)                                                                      \
    return bnx == 32   ? launch_group64_tokenwise<WW, AA, 32>(ta, twx, px, stream, pdl)        \
           : bnx == 64 ? launch_group64_tokenwise<WW, AA, 64>(ta, twx, px, stream, pdl)        \
                       : launch_group64_tokenwise<WW, AA, 128>(ta, twx, px, stream, pdl);
    ACTUNE_TW(2, 8) ACTUNE_TW(4, 8) ACTUNE_TW(8, 8) ACTUNE_TW(2, 4) ACTUNE_TW(4, 4) ACTUNE_TW(8, 4)
#undef ACTUNE_TW
    return cudaErrorInvalidValue;
  };
  if (variant == ACTUNE_VARIANT_AUTO && bn == 128) {
    // The wave-tail split of the group-64 GEMM (bit-identical outputs).
    int64_t na = 0;
    const int bn_b = wave_tail_split(M, N, g_devices[dev].num_sms, &na);
    if (bn_b > 0) {
      CUtensorMap tw_b;
      rc = encode_map(&tw_b, w, N, K * W / 8, W == 8 ? 128 : 16 * W, bn_b, W == 8 ? Swz::B128 : Swz::None);
      if (rc != ACTUNE_OK) return rc;
      GemmParams pa = p, pb = p;
      pa.n_end = (int)(na * 128);
      pb.n_base = (int)(na * 128);
      cudaError_t e = launch(128, tw, pa, false);
      if (e == cudaSuccess) e = launch(bn_b, tw_b, pb, true);
      return cuda_status(e);
    }
  }
  p.pdl_wait = 1;
  return cuda_status(launch(bn, tw, p, true));
}

}  // namespace
}  // namespace actune

using namespace actune;

extern "C" {

int actune_abi_version(void) { return ACTUNE_ABI_VERSION; }

int actune_last_cuda_error(void) { return g_last_cuda_error; }

const char* actune_status_string(int status) {
  switch (status) {
    case ACTUNE_OK: return "ok";
    case ACTUNE_ERR_INVALID_VALUE: return "invalid value (shape, bit width, dtype or null pointer)";
    case ACTUNE_ERR_MISALIGNED: return "misaligned pointer";
    case ACTUNE_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200-class) GPU";
    case ACTUNE_ERR_CUDA: return "CUDA runtime/driver call failed";
    case ACTUNE_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

namespace {
int quantize_group64(const void* x, int x_dtype, int64_t M, int64_t K, int A, bool codes8, uint8_t* packed,
                     float* scales, void* stream) {
  if (!valid_bits(A) || !valid_float_dtype(x_dtype) || M < 0 || K <= 0 || K % 64) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && (x == nullptr || packed == nullptr || scales == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0) return ACTUNE_OK;
  if (!aligned(x, 16) || !aligned(packed, 8) || !aligned(scales, 4)) return ACTUNE_ERR_MISALIGNED;
  const int dt = x_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (x_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  cudaError_t e = launch_quantize_group64(x, dt, M * (K / 64), A, codes8, packed, scales, g_devices[dev].num_sms,
                                          reinterpret_cast<cudaStream_t>(stream));
  return cuda_status(e);
}
}  // namespace

int actune_quantize_group64(const void* x, int x_dtype, int64_t M, int64_t K, int A, uint8_t* packed, float* scales,
                            void* stream) {
  return quantize_group64(x, x_dtype, M, K, A, false, packed, scales, stream);
}

int actune_quantize_group64_codes(const void* x, int x_dtype, int64_t M, int64_t K, int A, uint8_t* codes,
                                  float* scales, void* stream) {
  return quantize_group64(x, x_dtype, M, K, A, true, codes, scales, stream);
}

int actune_packed_linear(const uint8_t* a, const float* a_scale, const uint8_t* w, const float* w_scale,
                         const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                         int W, int A, int variant, void* stream) {
  int rc = check_gemm_shape(M, N, K, W, A);
  if (rc != ACTUNE_OK) return rc;
  if (!valid_float_dtype(out_dtype) || variant < 0 || variant > ACTUNE_VARIANT_BN128P) return ACTUNE_ERR_INVALID_VALUE;
  if (bias != nullptr && !valid_float_dtype(bias_dtype)) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && N > 0 && (a == nullptr || a_scale == nullptr || w == nullptr || w_scale == nullptr || out == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  if (!aligned(a_scale, 4) || !aligned(w_scale, 4) || !aligned(out, dtype_size(out_dtype)) ||
      (bias != nullptr && !aligned(bias, dtype_size(bias_dtype))))
    return ACTUNE_ERR_MISALIGNED;
  const int bdt = bias == nullptr ? kDtNone
                                  : (bias_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16
                                                                     : (bias_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32));
  const int odt = out_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (out_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  return run_gemm(a, a_scale, w, w_scale, bias, bdt, out, odt, nullptr, M, N, K, W, A, variant,
                  reinterpret_cast<cudaStream_t>(stream));
}

int actune_quantize_rows_a8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* codes, float* scales,
                            void* stream) {
  if (!valid_float_dtype(x_dtype) || M < 0 || K <= 0 || K % 8) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && (x == nullptr || codes == nullptr || scales == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0) return ACTUNE_OK;
  if (!aligned(x, 16) || !aligned(codes, 8) || !aligned(scales, 4)) return ACTUNE_ERR_MISALIGNED;
  const int dt = x_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (x_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  return cuda_status(launch_quantize_rows(x, dt, M, K, 8, reinterpret_cast<uint8_t*>(codes), scales,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

int actune_quantize_rows_a4(const void* x, int x_dtype, int64_t M, int64_t K, uint8_t* packed, float* scales,
                            void* stream) {
  if (!valid_float_dtype(x_dtype) || M < 0 || K <= 0 || K % 8) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && (x == nullptr || packed == nullptr || scales == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0) return ACTUNE_OK;
  if (!aligned(x, 16) || !aligned(packed, 4) || !aligned(scales, 4)) return ACTUNE_ERR_MISALIGNED;
  const int dt = x_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (x_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  return cuda_status(launch_quantize_rows(x, dt, M, K, 4, packed, scales, reinterpret_cast<cudaStream_t>(stream)));
}

int actune_tokenwise_linear(const int8_t* a, const float* a_scale, const uint8_t* w, const float* w_scale,
                            const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                            int W, int variant, void* stream) {
  if (!valid_bits(W) || K <= 0 || K % 64 || K > (int64_t(1) << 24) || M < 0 || N < 0 || M >= (int64_t(1) << 31) ||
      N >= (int64_t(1) << 31))
    return ACTUNE_ERR_INVALID_VALUE;
  if (!valid_float_dtype(out_dtype) || variant < 0 || (variant > ACTUNE_VARIANT_BN128 && !is_persistent_variant(variant)))
    return ACTUNE_ERR_INVALID_VALUE;
  if (bias != nullptr && !valid_float_dtype(bias_dtype)) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && N > 0 && (a == nullptr || a_scale == nullptr || w == nullptr || w_scale == nullptr || out == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  if (!aligned(a_scale, 4) || !aligned(w_scale, 4) || !aligned(out, dtype_size(out_dtype)) ||
      (bias != nullptr && !aligned(bias, dtype_size(bias_dtype))))
    return ACTUNE_ERR_MISALIGNED;
  const int bdt = bias == nullptr ? kDtNone
                                  : (bias_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16
                                                                     : (bias_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32));
  const int odt = out_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (out_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  return run_rowwise(reinterpret_cast<const uint8_t*>(a), 8, a_scale, w, W, w_scale, bias, bdt, out, odt, M, N, K, 0,
                     variant, reinterpret_cast<cudaStream_t>(stream));
}

int actune_rowwise_linear(const uint8_t* a, int A, const float* a_scale, const uint8_t* w, int W, const float* w_scale,
                          const void* bias, int bias_dtype, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                          int order, int variant, void* stream) {
  if (!valid_bits(W) || (A != 4 && A != 8) || (order != 0 && order != 1) || K <= 0 || K % 64 ||
      K > (int64_t(1) << 24) || M < 0 || N < 0 || M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31))
    return ACTUNE_ERR_INVALID_VALUE;
  if (!valid_float_dtype(out_dtype) || variant < 0 || (variant > ACTUNE_VARIANT_BN128 && !is_persistent_variant(variant)))
    return ACTUNE_ERR_INVALID_VALUE;
  if (bias != nullptr && !valid_float_dtype(bias_dtype)) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && N > 0 && (a == nullptr || a_scale == nullptr || w == nullptr || w_scale == nullptr || out == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  if (!aligned(a_scale, 4) || !aligned(w_scale, 4) || !aligned(out, dtype_size(out_dtype)) ||
      (bias != nullptr && !aligned(bias, dtype_size(bias_dtype))))
    return ACTUNE_ERR_MISALIGNED;
  const int bdt = bias == nullptr ? kDtNone
                                  : (bias_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16
                                                                     : (bias_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32));
  const int odt = out_dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (out_dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  return run_rowwise(a, A, a_scale, w, W, w_scale, bias, bdt, out, odt, M, N, K, order, variant,
                     reinterpret_cast<cudaStream_t>(stream));
}

int actune_packed_linear_dots(const uint8_t* a, const uint8_t* w, int32_t* dots, int64_t M, int64_t N, int64_t K,
                              int W, int A, int variant, void* stream) {
  int rc = check_gemm_shape(M, N, K, W, A);
  if (rc != ACTUNE_OK) return rc;
  if (variant < 0 || variant > ACTUNE_VARIANT_BN128P) return ACTUNE_ERR_INVALID_VALUE;
  if (M > 0 && N > 0 && (a == nullptr || w == nullptr || dots == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  if (!aligned(dots, 4)) return ACTUNE_ERR_MISALIGNED;
  return run_gemm(a, nullptr, w, nullptr, nullptr, kDtNone, nullptr, kDtF32, dots, M, N, K, W, A, variant,
                  reinterpret_cast<cudaStream_t>(stream));
}

int actune_weight_codes(const void* weight, int dtype, int64_t N, int64_t K, int W, int A, const float* clip,
                        int8_t* codes, float* scale, void* stream) {
  if (!valid_bits(W) || !valid_bits(A) || !valid_float_dtype(dtype) || N < 0 || K <= 0 || N >= (int64_t(1) << 31))
    return ACTUNE_ERR_INVALID_VALUE;
  if (N > 0 && (weight == nullptr || codes == nullptr || scale == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (!aligned(weight, dtype_size(dtype)) || !aligned(scale, 4) || (clip != nullptr && !aligned(clip, 4)))
    return ACTUNE_ERR_MISALIGNED;
  const int dt = dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  cudaError_t e = launch_weight_codes(weight, dt, N, K, W, A, clip, codes, scale, reinterpret_cast<cudaStream_t>(stream));
  return cuda_status(e);
}

int actune_r4_refine(const void* weight, int dtype, int64_t N, int64_t K, const int8_t* q4, const float* scale4,
                     int8_t* residual, int8_t* q8, void* stream) {
  if (!valid_float_dtype(dtype) || N < 0 || K <= 0 || N >= (int64_t(1) << 31)) return ACTUNE_ERR_INVALID_VALUE;
  if (N > 0 && (weight == nullptr || q4 == nullptr || scale4 == nullptr || residual == nullptr || q8 == nullptr))
    return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (!aligned(weight, dtype_size(dtype)) || !aligned(scale4, 4)) return ACTUNE_ERR_MISALIGNED;
  const int dt = dtype == ACTUNE_DTYPE_BF16 ? kDtBF16 : (dtype == ACTUNE_DTYPE_F16 ? kDtF16 : kDtF32);
  cudaError_t e = launch_r4_refine(weight, dt, N, K, q4, scale4, residual, q8, reinterpret_cast<cudaStream_t>(stream));
  return cuda_status(e);
}

int actune_pack_rows(const int8_t* codes, int64_t R, int64_t K, int bits, uint8_t* packed, void* stream) {
  if (!valid_bits(bits) || R < 0 || K <= 0 || K % (8 / bits)) return ACTUNE_ERR_INVALID_VALUE;
  if (R > 0 && (codes == nullptr || packed == nullptr)) return ACTUNE_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  cudaError_t e = launch_pack_rows(codes, R * (K * bits / 8), bits, packed, g_devices[dev].num_sms,
                                   reinterpret_cast<cudaStream_t>(stream));
  return cuda_status(e);
}

size_t actune_grouped_linear_workspace_size(int64_t M, int64_t K, int A) {
  if (M <= 0 || K <= 0 || !valid_bits(A)) return 0;
  const size_t packed = ((size_t)M * (size_t)K * (size_t)A / 8 + 255) / 256 * 256;
  const size_t scales = ((size_t)M * (size_t)(K / 64) * 4 + 255) / 256 * 256;
  return packed + scales;
}

int actune_grouped_linear(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* w, const float* w_scale,
                          const void* bias, int bias_dtype, int64_t N, int W, int A, void* out, int out_dtype,
                          void* workspace, size_t workspace_bytes, int variant, void* stream) {
  int rc = check_gemm_shape(M, N, K, W, A);
  if (rc != ACTUNE_OK) return rc;
  if (M == 0 || N == 0) {
    int dev = 0;
    return current_device(&dev);
  }
  const size_t need = actune_grouped_linear_workspace_size(M, K, A);
  if (workspace == nullptr || workspace_bytes < need) return ACTUNE_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return ACTUNE_ERR_MISALIGNED;
  uint8_t* packed = reinterpret_cast<uint8_t*>(workspace);
  float* scales = reinterpret_cast<float*>(packed + ((size_t)M * (size_t)K * (size_t)A / 8 + 255) / 256 * 256);
  rc = actune_quantize_group64(x, x_dtype, M, K, A, packed, scales, stream);
  if (rc != ACTUNE_OK) return rc;
  return actune_packed_linear(packed, scales, w, w_scale, bias, bias_dtype, out, out_dtype, M, N, K, W, A, variant,
                              stream);
}

int actune_device_error(int* code, int* site, int reset) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != ACTUNE_OK) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return ACTUNE_ERR_CUDA;
  int c = 0, s = 0;
  if (cudaMemcpyFromSymbol(&c, g_actune_error, sizeof(int)) != cudaSuccess ||
      cudaMemcpyFromSymbol(&s, g_actune_error_site, sizeof(int)) != cudaSuccess)
    return ACTUNE_ERR_CUDA;
  if (code) *code = c;
  if (site) *site = s;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_actune_error, &zero, sizeof(int)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_actune_error_site, &zero, sizeof(int)) != cudaSuccess)
      return ACTUNE_ERR_CUDA;
  }
  return ACTUNE_OK;
}

}  // extern "C"
