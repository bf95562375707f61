// Packed-integer group-64 linear on Blackwell tensor cores (sm_100a).
//
//   y[m, n] = ws[n] * sum_g ( float(dot_g(m, n)) * as[m, g] )  (+ bias[n])
//   dot_g(m, n) = sum_{k in group g} a[m, k] * w[n, k]          (exact int32)
//
// with the fp32 chain evaluated exactly as the reference's GPU kernels do
// (actune/kernels/grouped.py:80-94, actune/kernels/grouped_native.cu:70-85):
// acc = fma(float(dot_g), as[m, g], acc) for g = 0, 1, ... in order, then
// y = fma(acc, ws[n], bias[n]) (or acc * ws[n] without bias), rounded once to
// the output type.  Every W x A pair in {2,4,8}^2 runs on tcgen05 kind::i8.
//
// CTA tile: 128 token rows (TMEM lanes) x BN weight rows (TMEM columns); K is
// streamed in stages of 128 = two groups of 64.  Each stage's two groups go to
// a pair of TMEM int32 accumulator buffers (NPAIR pairs rotate), so the MMA
// issuer and the epilogue hand off once per stage.  Warp roles:
//   warp 0      TMA producer: packed activation and weight tiles -> smem ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (straight-line
//               4 MMAs per stage from precomputed descriptors)
//   warps 2-5   converters (sub-byte W or A only): codes -> int8 in the canonical
//               128B-swizzled K-major layout (code placed in the top bits of
//               the byte, i.e. scaled by 2^(8-bits); compensated exactly in fp32)
//   then 8      epilogue warps: tcgen05.ld of each group's int32 dots, exact
//               int->fp32 conversion, packed fp32x2 FMA into register
//               accumulators, final scale/bias/convert/store
#pragma once

#include <type_traits>

#include "common.cuh"

namespace actune {

enum : int { kDtNone = 0, kDtF32 = 1, kDtF16 = 2, kDtBF16 = 3 };

struct GemmParams {
  const float* act_scale;  // [M, G]
  const float* w_scale;    // [N]
  const void* bias;        // [N] (bias_dtype) or nullptr
  void* out;               // [M, N] (out_dtype)
  int32_t* dots;           // debug export [M, N, G] int32 (exact group dots) or nullptr
  int M, N, K, G;
  int bias_dtype;
  int out_dtype;
  int out_vec_ok;          // N % 8 == 0 and out 16-byte aligned
  int rowwise_order;       // row-scaled modes: 0 (acc*as)*ws, 1 acc*(as*ws) (the per-row A4 native order)
  int gemv_boxes2d;        // decode: packed rows not whole 128-byte blocks, one 2-D box per block
  int a_box_rows;          // GEMM: token box height of the activation map (0: a whole 128-row tile)
  int pdl_wait;            // dependent launch: wait for the previous kernel before reading its outputs
  int n_base, n_end;       // GEMM: output columns [n_base, n_end) of [0, N) (n_end 0: N)
};

// Wait-site identifiers recorded with a device timeout.
enum : int { kSiteProducer = 1, kSiteConverter, kSiteMmaFull, kSiteMmaAcc, kSiteMmaDone, kSiteEpilogue, kSiteDrain };

// OCC = CTAs resident per SM: 1, or 2 (half the TMEM columns, shared memory and
// registers each, so that one CTA's MMA runs while the other's epilogue drains).
template <int W, int A, int BN, int OCC = 1>
struct Group64Cfg {
  static_assert(W == 2 || W == 4 || W == 8, "W");
  static_assert(A == 2 || A == 4 || A == 8, "A");
  static_assert(BN == 32 || BN == 64 || BN == 128, "BN");
  static_assert(OCC == 1 || OCC == 2, "OCC");
  static constexpr int BM = 128;     // token rows per tile = TMEM lanes = MMA M
  static constexpr int KS = 128;     // K elements per pipeline stage (two groups)
  static constexpr int EPI_WG = 2;   // two epilogue warpgroups split the columns
  static constexpr int COLS = BN / EPI_WG;      // accumulator columns per epilogue thread
  // Accumulator buffer pairs (one pair per stage): 512 TMEM columns per CTA, or 256
  // at two CTAs per SM.
  static constexpr int NPAIR = OCC == 1 ? (BN == 32 ? 4 : 2) : (BN == 128 ? 1 : 2);
  static constexpr int TMEM_COLS = NPAIR * 2 * BN; // 256 or 512 (power of two)
  static constexpr bool CONVERT = (A < 8) || (W < 8);
  // Warps: producer, MMA issuer, CVT_WARPS converters, then 4 * EPI_WG epilogue warps.
  static constexpr int CVT_WARPS = CONVERT ? (OCC == 1 ? 4 : 2) : 0;
  static constexpr int EPI_WARP0 = 2 + CVT_WARPS;
  static constexpr int THREADS = 32 * EPI_WARP0 + 128 * EPI_WG;
  // The tile kernel adds a second MMA-issuing warp after the epilogue warps: the two
  // issue alternate stages, so that one thread's barrier waits and commits overlap
  // the other's MMAs (one issuing thread is held for each MMA's duration).
  static constexpr int MMA2_WARP = THREADS / 32;
  static constexpr int TILE_THREADS = THREADS + 32;
  // Per-stage shared-memory layout: [act int8 | wgt int8 | act packed | wgt packed].
  static constexpr int OP_A_BYTES = BM * KS;        // 16 KB, SW128 K-major
  static constexpr int OP_W_BYTES = BN * KS;
  static constexpr int STG_A_BYTES = A < 8 ? BM * KS * A / 8 : 0;
  static constexpr int STG_W_BYTES = W < 8 ? BN * KS * W / 8 : 0;
  static constexpr int STAGE_RAW = OP_A_BYTES + OP_W_BYTES + STG_A_BYTES + STG_W_BYTES;
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int STAGES_FIT = ((OCC == 1 ? 200 : 104) * 1024) / STAGE_BYTES;
  // A multiple of NPAIR, so that the accumulator pair of an unrolled ring slot is a
  // compile-time constant, and even (the MMA issuer's two descriptor sets).
  static constexpr int SLOT_MULT = NPAIR > 2 ? NPAIR : 2;
  static constexpr int STAGES = (STAGES_FIT > 8 ? 8 : STAGES_FIT) / SLOT_MULT * SLOT_MULT;
  // The final epilogue stages the fp32 tile [BM][BN + 4] through the ring.
  static constexpr int OUT_STAGE_BYTES = BM * (BN + 4) * 4;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES > OUT_STAGE_BYTES ? STAGES * STAGE_BYTES : OUT_STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + 1024;  // + alignment slack
  // int8 operand value = code * 2^(8-bits): the dot carries 2^SHIFT.
  static constexpr int SHIFT = (8 - A) + (8 - W);
  // Bytes one stage's two TMA loads deliver with a whole 128-row token box (OOB parts
  // of a box are zero-filled and count).
  static constexpr uint32_t TX_BYTES = BM * KS * A / 8 + BN * KS * W / 8;
  static_assert(STAGES >= 2, "stages");
};

// Unpack one stage of packed sub-byte codes (ROWS rows x 128 codes, row pitch
// 16*BITS bytes) into the SW128 K-major int8 operand (row pitch 128 bytes,
// 16-byte chunk c of row r stored at chunk c ^ (r mod 8)).  One item = 16
// packed bytes = 2 (BITS 4) or 4 (BITS 2) output chunks.  NT threads split the
// items; thread t handles items t, t + NT, ... which all share the same chunk
// index and row phase (r mod 8), so every address is a per-thread base plus a
// compile-time offset.
//
// Only rows below `rows_valid` are expanded: the operand rows past the last token
// keep whatever they held, which reaches only accumulator rows that are never stored
// (an MMA row depends on its own operand row alone).
template <int BITS, int ROWS, int NT_ALL>
__device__ __forceinline__ void unpack_stage(const uint8_t* __restrict__ stg, uint8_t* __restrict__ op, int tid,
                                             int rows_valid = ROWS) {
  constexpr int IPR = BITS;                   // items per row: 16*BITS packed bytes / 16
  constexpr int CHUNKS = 8 / IPR;             // output chunks per item
  constexpr int ITEMS = ROWS * IPR;
  constexpr int NT = NT_ALL < ITEMS ? NT_ALL : ITEMS;  // threads with work
  static_assert(ITEMS % NT == 0, "items must split evenly");
  if (tid >= NT) return;
  constexpr int ROW_STEP = NT / IPR;          // rows advanced per pass
  static_assert(ROW_STEP % 8 == 0, "row step must keep the swizzle phase");
  const int r0 = tid / IPR, i = tid % IPR;
  const int x = r0 & 7;
  const uint8_t* src = stg + tid * 16;
  uint8_t* row = op + (r0 >> 3) * 1024 + x * 128;
  const int c0 = i * CHUNKS;
  // Passes that hold a valid row (all of them for a full tile).
  const int passes = rows_valid >= ROWS ? ITEMS / NT : (rows_valid - r0 + ROW_STEP - 1) / ROW_STEP;
#pragma unroll
  for (int j = 0; j < ITEMS / NT; ++j) {
    if (j >= passes) break;
    const uint4 v = *reinterpret_cast<const uint4*>(src + j * NT * 16);
    uint8_t* dst = row + j * (ROW_STEP / 8) * 1024;
    if constexpr (BITS == 4) {
      const uint2 a = unpack_w4_word(v.x), b = unpack_w4_word(v.y);
      const uint2 c = unpack_w4_word(v.z), d = unpack_w4_word(v.w);
      *reinterpret_cast<uint4*>(dst + (((c0 + 0) ^ x) << 4)) = make_uint4(a.x, a.y, b.x, b.y);
      *reinterpret_cast<uint4*>(dst + (((c0 + 1) ^ x) << 4)) = make_uint4(c.x, c.y, d.x, d.y);
    } else {
      static_assert(BITS == 2, "BITS");
      *reinterpret_cast<uint4*>(dst + (((c0 + 0) ^ x) << 4)) = unpack_w2_word(v.x);
      *reinterpret_cast<uint4*>(dst + (((c0 + 1) ^ x) << 4)) = unpack_w2_word(v.y);
      *reinterpret_cast<uint4*>(dst + (((c0 + 2) ^ x) << 4)) = unpack_w2_word(v.z);
      *reinterpret_cast<uint4*>(dst + (((c0 + 3) ^ x) << 4)) = unpack_w2_word(v.w);
    }
  }
}

__device__ __forceinline__ float load_bias(const void* bias, int dtype, int n) {
  if (dtype == kDtF32) return __ldg(reinterpret_cast<const float*>(bias) + n);
  if (dtype == kDtBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  return __half2float(reinterpret_cast<const __half*>(bias)[n]);
}

__device__ __forceinline__ float finish(float acc, const GemmParams& p, int n) {
  const float ws = __ldg(p.w_scale + n);
  if (p.bias_dtype != kDtNone) return fmaf(acc, ws, load_bias(p.bias, p.bias_dtype, n));
  return acc * ws;
}

// Row-scaled epilogue in the per-row A4 native order (native_s4_extension_kernel.cu:
// 229-233): y = acc * (as[m] * ws[n]) (+ bias, fused).
__device__ __forceinline__ float finish_native(float acc, const GemmParams& p, int n, float as_m) {
  const float s = as_m * __ldg(p.w_scale + n);
  if (p.bias_dtype != kDtNone) return fmaf(acc, s, load_bias(p.bias, p.bias_dtype, n));
  return acc * s;
}

__device__ __forceinline__ void store_scalar(const GemmParams& p, int64_t idx, float y) {
  if (p.out_dtype == kDtBF16) reinterpret_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(y);
  else if (p.out_dtype == kDtF16) reinterpret_cast<__half*>(p.out)[idx] = __float2half_rn(y);
  else reinterpret_cast<float*>(p.out)[idx] = y;
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 32) {
    tmem_ld32(taddr, r);
  } else if constexpr (N == 16) {
    tmem_ld16(taddr, r);
  } else if constexpr (N == 8) {
    tmem_ld8(taddr, r);
  } else {
    static_assert(N == 4, "tmem_ld width");
    tmem_ld4(taddr, r);
  }
}

// acc[j] += float(d[2j..2j+1]) * s for H int32 dots (exact conversion, packed fp32x2 FMA).
template <int H>
__device__ __forceinline__ void accumulate(float2* acc, const uint32_t (&d)[H], float s) {
  // float(dot) exactly (|dot * 2^SHIFT| < 2^24): the hardware conversion measured
  // 4-7% faster here than the two-instruction bit-pattern form.
  const float2 s2 = make_float2(s, s);
#pragma unroll
  for (int j = 0; j < H / 2; ++j) {
    const float2 f = make_float2(__int2float_rn((int)d[2 * j]), __int2float_rn((int)d[2 * j + 1]));
    acc[j] = ffma2(f, s2, acc[j]);
  }
}

template <int H>
__device__ __forceinline__ void store_dots(const GemmParams& p, int m, int col, int g, const uint32_t (&d)[H],
                                           int shift) {
  if (m >= p.M || g >= p.G) return;
#pragma unroll
  for (int j = 0; j < H; ++j) {
    const int n = col + j;
    if (n < p.N) p.dots[((int64_t)m * p.N + n) * p.G + g] = static_cast<int32_t>(d[j]) >> shift;
  }
}

// TW (tokenwise backends): one full-K int32 accumulator per tile instead of one per
// 64-group; the epilogue reads it once, converts it exactly (round to nearest) and
// applies the per-token scale (p.act_scale[m]), then ws / bias as below.
template <int W, int A, int BN, bool DOTS, bool TW = false, int OCC = 1>
__global__ void __launch_bounds__(Group64Cfg<W, A, BN, OCC>::TILE_THREADS, OCC)
    group64_gemm_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_wgt,
                        const GemmParams p) {
  using C = Group64Cfg<W, A, BN, OCC>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_raw[C::STAGES];
  __shared__ __align__(8) uint64_t full_op[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t acc_full[C::NPAIR];
  __shared__ __align__(8) uint64_t acc_empty[C::NPAIR];
  __shared__ __align__(8) uint64_t mma_done[2];
  __shared__ uint32_t tmem_holder;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_iters = (G + 1) >> 1;
  const int m0 = blockIdx.x * C::BM;
  const int n0 = p.n_base + blockIdx.y * BN;
  // The next launch in the stream (made with programmatic stream serialization) may
  // start as soon as SMs come free: the rest of a wave-tail split, which reads the
  // same inputs, or a kernel that waits for this one before reading its output.
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&full_op[s], C::CVT_WARPS > 0 ? C::CVT_WARPS : 1);  // one arrival per converter warp
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < C::NPAIR; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * C::EPI_WG);
    }
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_act);
    prefetch_tensormap(&tm_wgt);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane 0 loads the activation tile and lane 1 the weight tile of a stage
    // with ONE bulk-tensor instruction: copies issued by successive
    // instructions of a thread are serviced one after another (about one L2
    // round trip each), while the lanes of one instruction proceed together.
    // The loop is unrolled over the ring and every operand of a copy sits in a
    // register of its own: an asynchronous copy reads its register operands some
    // time after issue, and rewriting one for the next copy stalls until it has.
    int issued = 0;
    // A token box may be lower than the tile (a single tile of few tokens): the
    // transaction count is the bytes the two boxes deliver.
    const uint32_t tx_bytes = (uint32_t)(p.a_box_rows > 0 ? p.a_box_rows : C::BM) * (C::KS * A / 8) +
                              (uint32_t)BN * (C::KS * W / 8);
    if (lane < 2) {
      const CUtensorMap* map = lane == 0 ? &tm_act : &tm_wgt;
      const int x_step = lane == 0 ? C::KS * A / 8 : C::KS * W / 8;
      const int y = lane == 0 ? m0 : n0;
      const uint32_t dst_off = lane == 0 ? (A < 8 ? C::OP_A_BYTES + C::OP_W_BYTES : 0)
                                         : (W < 8 ? C::OP_A_BYTES + C::OP_W_BYTES + C::STG_A_BYTES : C::OP_A_BYTES);
      constexpr int S = C::STAGES, HALF = C::STAGES / 2;
      uint32_t dst[S], bar[S];
      int xs[S];
#pragma unroll
      for (int j = 0; j < S; ++j) {
        dst[j] = smem_u32(smem + j * C::STAGE_BYTES + dst_off);
        bar[j] = smem_u32(&full_raw[j]);
        xs[j] = j * x_step;
      }
      // Dependent launch: the set-up above overlapped the previous kernel; the tiles
      // are requested once it has completed.  (Requesting the first weight tiles
      // before the wait measured slower: the extra path costs the ring loop more
      // than the early loads save.)
      if (p.pdl_wait) griddep_wait();
      uint32_t ph = 0;
      bool ok = true;
      for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          if (it0 + j >= n_iters) break;
          bool w_ok = true;
          if (lane == 0) {
            w_ok = mbar_wait(&empty_bar[j], ph ^ 1, kSiteProducer);
            if (w_ok) mbar_arrive_expect_tx(&full_raw[j], tx_bytes);
          }
          if (!__shfl_sync(0x3u, w_ok, 0)) { ok = false; break; }
          if (j + HALF < S) xs[j + HALF] = (it0 + j + HALF) * x_step;  // read HALF copies from now
          tma_load_2d_u32(dst[j], map, xs[j], y, bar[j]);
          ++issued;
          if (j >= HALF) xs[j - HALF] = (it0 + S + j - HALF) * x_step;  // its copy went HALF ago
        }
        ph ^= 1;
      }
    }
    // Never leave the CTA with bulk copies still landing in shared memory.
    if (lane == 0) {
      for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it)
        mbar_wait(&full_raw[it % C::STAGES], (it / C::STAGES) & 1, kSiteDrain);
    }
  } else if (warp == 1 || warp == C::MMA2_WARP) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues the even stages, the last warp the odd ones (warp 1 all of them in
    // the row-scaled mode, whose stages accumulate into one buffer, and with a single
    // accumulator pair): one issuing
    // thread is held for each MMA's duration, so one issuer's barrier waits and
    // commits overlap the other's MMAs.  With an even ring depth and an even number
    // of accumulator pairs, a ring slot and an accumulator pair always belong to the
    // same issuer, whose commits track its own MMAs.
    // Per stage: wait operands, wait the accumulator pair, 4 MMAs, 2 commits.  An MMA
    // reads its register operands when the tensor core takes it: each issuer keeps
    // the descriptors of its own ring slots in registers of their own (never
    // rewritten); the single row-scaled issuer alternates two sets, each rewritten
    // only after the other stage's MMAs have been issued.
    // Two issuers need an even number of accumulator pairs (else one issuer).
    constexpr bool TWO = !TW && C::NPAIR % 2 == 0;
    static_assert(C::STAGES % 2 == 0, "even ring depth");
    constexpr int S = C::STAGES;
    constexpr uint32_t idesc = idesc_i8(C::BM, BN);
    const uint64_t desc_a0 = smem_desc_sw128(smem_u32(smem));
    const uint64_t desc_w0 = smem_desc_sw128(smem_u32(smem) + C::OP_A_BYTES);
    constexpr uint64_t kStageStep = (uint64_t)(C::STAGE_BYTES >> 4);
    const int who = warp == 1 ? 0 : 1;
    auto issue = [&](auto parity_tag) {
      constexpr int PAR = decltype(parity_tag)::value;
      uint32_t dacc[C::NPAIR][2], bacc[C::NPAIR], bempty[S];
#pragma unroll
      for (int pr = 0; pr < C::NPAIR; ++pr) {
        dacc[pr][0] = tmem_base + pr * (2 * BN);
        dacc[pr][1] = tmem_base + pr * (2 * BN) + BN;
        bacc[pr] = smem_u32(&acc_full[pr]);
      }
#pragma unroll
      for (int j = 0; j < S; ++j) bempty[j] = smem_u32(&empty_bar[j]);
      uint32_t ph = 0;
      bool ok = true;
      if constexpr (!TWO) {
        uint64_t da[2][4], dw[2][4];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            da[q][k] = desc_a0 + kStageStep * q + 2 * k;
            dw[q][k] = desc_w0 + kStageStep * q + 2 * k;
          }
        for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
          for (int j = 0; j < S; ++j) {
            const int it = it0 + j;
            if (it >= n_iters) break;
            const int q = j & 1, pr = j % C::NPAIR;
            uint64_t* ready = C::CONVERT ? &full_op[j] : &full_raw[j];
            if (!mbar_wait(ready, ph, kSiteMmaFull) ||
                (!TW && !mbar_wait(&acc_empty[pr], ((it / C::NPAIR) & 1) ^ 1, kSiteMmaAcc))) {
              ok = false;
              break;
            }
            tc_fence_after();
            if constexpr (TW) {
              // Every K slice of every stage into one accumulator.
              mma_i8(dacc[0][0], da[q][0], dw[q][0], idesc, it > 0 ? 1u : 0u);
              mma_i8(dacc[0][0], da[q][1], dw[q][1], idesc, 1u);
              mma_i8(dacc[0][0], da[q][2], dw[q][2], idesc, 1u);
              mma_i8(dacc[0][0], da[q][3], dw[q][3], idesc, 1u);
              if (it == n_iters - 1) mma_commit_u32(bacc[0]);
            } else {
              mma_i8(dacc[pr][0], da[q][0], dw[q][0], idesc, 0u);
              mma_i8(dacc[pr][0], da[q][1], dw[q][1], idesc, 1u);
              mma_i8(dacc[pr][1], da[q][2], dw[q][2], idesc, 0u);
              mma_i8(dacc[pr][1], da[q][3], dw[q][3], idesc, 1u);
              mma_commit_u32(bacc[pr]);
            }
            mma_commit_u32(bempty[j]);
            const int jn = (j + 1) % S;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              da[q ^ 1][k] = desc_a0 + kStageStep * jn + 2 * k;
              dw[q ^ 1][k] = desc_w0 + kStageStep * jn + 2 * k;
            }
          }
          ph ^= 1;
        }
      } else {
        constexpr int NS = S / 2;  // ring slots PAR, PAR + 2, ...
        uint64_t da[NS][4], dw[NS][4];
#pragma unroll
        for (int u = 0; u < NS; ++u)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            da[u][k] = desc_a0 + kStageStep * (PAR + 2 * u) + 2 * k;
            dw[u][k] = desc_w0 + kStageStep * (PAR + 2 * u) + 2 * k;
          }
        for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
          for (int j = PAR; j < S; j += 2) {
            const int it = it0 + j;
            if (it >= n_iters) break;
            const int pr = j % C::NPAIR, u = j / 2;
            uint64_t* ready = C::CONVERT ? &full_op[j] : &full_raw[j];
            if (!mbar_wait(ready, ph, kSiteMmaFull) ||
                !mbar_wait(&acc_empty[pr], ((it / C::NPAIR) & 1) ^ 1, kSiteMmaAcc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // Always both groups: past the end of K (odd G) the tiles are the
            // TMA's zero fill, the dots are 0 and the epilogue gives them scale 0.
            mma_i8(dacc[pr][0], da[u][0], dw[u][0], idesc, 0u);  // group 2it:   K bytes 0..31
            mma_i8(dacc[pr][0], da[u][1], dw[u][1], idesc, 1u);  //              K bytes 32..63
            mma_i8(dacc[pr][1], da[u][2], dw[u][2], idesc, 0u);  // group 2it+1: K bytes 64..95
            mma_i8(dacc[pr][1], da[u][3], dw[u][3], idesc, 1u);  //              K bytes 96..127
            mma_commit_u32(bacc[pr]);
            mma_commit_u32(bempty[j]);
          }
          ph ^= 1;
        }
      }
    };
    if (lane == 0) {
      if (who == 0) issue(std::integral_constant<int, 0>{});
      else if constexpr (TWO) issue(std::integral_constant<int, 1>{});
      mma_commit(&mma_done[who]);
      mbar_wait(&mma_done[who], 0, kSiteMmaDone);
    }
  } else if (warp < C::EPI_WARP0) {
    // ------------------------------------------------------------ converters
    if constexpr (C::CONVERT) {
      const int ctid = threadIdx.x - 64;
      constexpr int NT = 32 * C::CVT_WARPS;
      const int a_rows_valid = min(C::BM, p.M - m0);
      for (int it = 0; it < n_iters; ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(&full_raw[s], (it / C::STAGES) & 1, kSiteConverter)) break;
        uint8_t* st = smem + s * C::STAGE_BYTES;
        if constexpr (A < 8) unpack_stage<A, C::BM, NT>(st + C::OP_A_BYTES + C::OP_W_BYTES, st, ctid, a_rows_valid);
        if constexpr (W < 8)
          unpack_stage<W, BN, NT>(st + C::OP_A_BYTES + C::OP_W_BYTES + C::STG_A_BYTES, st + C::OP_A_BYTES, ctid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_op[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each thread owns one token row (TMEM lane) and COLS columns, read from
    // TMEM in halves of H columns.  Within a stage each half-load overlaps the
    // accumulation of the previous half, and the first half of the next stage
    // is loaded before the last half of this one is accumulated.  Activation
    // scales are fetched two stages ahead into static register slots.
    // Dependent launch: while the previous kernel finishes, pull this tile's first
    // weight boxes into L2 (they never depend on it), so that the producer's first
    // copies after the wait hit L2.  Activation scales and the output may belong to
    // the previous kernel: wait for it before touching them.
    if (p.pdl_wait) {
      if (warp == C::EPI_WARP0 && lane == 0) {
        const int pre = min(C::STAGES, n_iters);
        for (int j = 0; j < pre; ++j) tma_prefetch_l2_2d(&tm_wgt, j * (C::KS * W / 8), n0);
      }
      griddep_wait();
    }
    const int ew = warp - C::EPI_WARP0;
    const int q = warp & 3;      // TMEM lane quarter this warp may access
    const int e = ew >> 2;       // column slice
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const bool warp_live = (m0 + q * 32) < p.M;  // any valid token row in this warp
    const int col0 = n0 + e * C::COLS;
    // TMEM is read in P parts of H columns per group: for 128-column tiles eight parts
    // when converter warps share the register file, four otherwise; narrower tiles
    // read a group in one or two parts (measured best; the part size moves the GEMM
    // by a few percent at most).
    constexpr int P = C::CVT_WARPS > 0 ? (C::COLS >= 64 ? 8 : C::COLS >= 32 ? 2 : 1) : (C::COLS >= 64 ? 4 : C::COLS >= 32 ? 2 : 1);
    constexpr int H = C::COLS / P;
    const float shift_scale = 1.0f / float(1 << C::SHIFT);
    const bool load_scales = !DOTS && warp_live && m < p.M;
    const float* as_row = p.act_scale + (int64_t)(m < p.M ? m : 0) * G;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + e * C::COLS;
    float2 acc[C::COLS / 2];
#pragma unroll
    for (int j = 0; j < C::COLS / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    auto scale_at = [&](int g) -> float { return (load_scales && g < G) ? __ldg(as_row + g) : 0.f; };
    uint32_t ra[H], rb[H];
    bool ok = true;
    if constexpr (TW) {
      // One wait for the whole-K accumulator, then y = float(acc) * 2^-SHIFT (exact:
      // a power of two) * as[m], stored in the accumulator registers for the final
      // ws / bias step below.
      ok = mbar_wait(&acc_full[0], 0, kSiteEpilogue);
      if (ok) {
        tc_fence_after();
        // Order 1 applies as[m] with ws in the final store.
        const float as_m = p.rowwise_order ? 1.f : ((m < p.M) ? __ldg(p.act_scale + m) : 0.f);
#pragma unroll
        for (int part = 0; part < C::COLS / H; ++part) {
          tmem_ld<H>(lane_base + part * H, ra);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < H / 2; ++j) {
            const float f0 = __int2float_rn((int)ra[2 * j]) * shift_scale;
            const float f1 = __int2float_rn((int)ra[2 * j + 1]) * shift_scale;
            acc[part * (H / 2) + j] = make_float2(f0 * as_m, f1 * as_m);
          }
        }
      }
    } else if (!warp_live) {
      // No valid token row in this warp: only keep the accumulator handshake.
      for (int it = 0; it < n_iters; ++it) {
        const int pr = it % C::NPAIR;
        if (!mbar_wait(&acc_full[pr], (it / C::NPAIR) & 1, kSiteEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[pr]);
      }
    } else if constexpr (!DOTS && C::COLS <= 32) {
      // Narrow tiles (at most 32 columns per thread): the TMEM loads of NB whole
      // stages are issued back to back and waited for once, their accumulator pairs
      // released, then accumulated, so that a stage costs a fraction of one TMEM load
      // latency instead of one latency per part; with NPAIR >= 2 * NB the MMA fills
      // the next batch's pairs meanwhile.  Scales are fetched two batches ahead.
      constexpr int NB = (C::COLS <= 16 && C::NPAIR >= 4) ? 2 : 1;
      uint32_t r[NB][2][C::COLS];
      float sc[NB][2], sn[NB][2], sn2[NB][2];
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          sc[b][h] = scale_at(2 * b + h);
          sn[b][h] = scale_at(2 * (NB + b) + h);
        }
      for (int it = 0; it < n_iters && ok; it += NB) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
          for (int h = 0; h < 2; ++h) sn2[b][h] = scale_at(2 * (it + 2 * NB + b) + h);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const int s = it + b;
          if (s < n_iters) {
            const int pr = s % C::NPAIR;
            if (!mbar_wait(&acc_full[pr], (s / C::NPAIR) & 1, kSiteEpilogue)) {
              ok = false;
              break;
            }
            tc_fence_after();
            tmem_ld<C::COLS>(lane_base + pr * (2 * BN), r[b][0]);
            tmem_ld<C::COLS>(lane_base + pr * (2 * BN) + BN, r[b][1]);
          }
        }
        if (!ok) break;
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int b = 0; b < NB; ++b)
            if (it + b < n_iters) mbar_arrive(&acc_empty[(it + b) % C::NPAIR]);
        }
        // Past the end of K (odd G) the second group's dots are 0 and so is its scale.
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (it + b < n_iters) {
            accumulate<C::COLS>(acc, r[b][0], sc[b][0] * shift_scale);
            accumulate<C::COLS>(acc, r[b][1], sc[b][1] * shift_scale);
          }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            sc[b][h] = sn[b][h];
            sn[b][h] = sn2[b][h];
          }
      }
    } else {
      ok = mbar_wait(&acc_full[0], 0, kSiteEpilogue);
      if (ok) {
        tc_fence_after();
        tmem_ld<H>(lane_base, ra);
        tmem_wait_ld();
      }
      // One stage: ra already holds part 0 of group 2it.  The 2 * P parts of the
      // stage's two groups are read in order into ra / rb alternately, each load
      // overlapping the accumulation of the part before it; the accumulator pair
      // is released as soon as its last part is in registers, and part 0 of the
      // next stage is loaded before that last part is accumulated.
      auto stage = [&](int it, float s0raw, float s1raw) {
        const int pr = it % C::NPAIR;
        const uint32_t base = lane_base + pr * (2 * BN);
        const int g0 = 2 * it;
        // Past the end of K (odd G) the second group's dots are 0 and s1 is 0
        // (scale_at), so acc += 0 * 0 leaves every accumulator unchanged (an
        // accumulator is never -0: it starts at +0 and the scales are > 0).
        const float s0 = s0raw * shift_scale, s1 = s1raw * shift_scale;
        auto part_step = [&](int idx, uint32_t(&cur)[H], uint32_t(&nxt)[H]) {
          const int grp = idx / P, part = idx % P;
          if (idx + 1 < 2 * P) {
            tmem_ld<H>(base + ((idx + 1) / P) * BN + ((idx + 1) % P) * H, nxt);
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[pr]);
            if (it + 1 < n_iters) {
              const int pn = (it + 1) % C::NPAIR;
              if (!mbar_wait(&acc_full[pn], ((it + 1) / C::NPAIR) & 1, kSiteEpilogue)) {
                ok = false;
              } else {
                tc_fence_after();
                tmem_ld<H>(lane_base + pn * (2 * BN), nxt);
              }
            }
          }
          if constexpr (DOTS) store_dots<H>(p, m, col0 + part * H, g0 + grp, cur, C::SHIFT);
          else accumulate<H>(acc + part * (H / 2), cur, grp ? s1 : s0);
          tmem_wait_ld();
        };
#pragma unroll
        for (int idx = 0; idx < 2 * P; idx += 2) {
          part_step(idx, ra, rb);
          part_step(idx + 1, rb, ra);
        }
      };
      // Scale slots: x for even stages, y for odd stages (fetched two stages ahead).
      float x0 = scale_at(0), x1 = scale_at(1), y0 = scale_at(2), y1 = scale_at(3);
      for (int it = 0; it < n_iters && ok; it += 2) {
        const float a0 = x0, a1 = x1;
        x0 = scale_at(2 * it + 4);
        x1 = scale_at(2 * it + 5);
        stage(it, a0, a1);
        if (it + 1 < n_iters && ok) {
          const float b0 = y0, b1 = y1;
          y0 = scale_at(2 * it + 6);
          y1 = scale_at(2 * it + 7);
          stage(it + 1, b0, b1);
        }
      }
    }

    // Final epilogue: stage fp32 accumulators through the (now idle) pipeline
    // shared memory, then every epilogue thread applies ws/bias to 8
    // consecutive columns of one row and writes them with one coalesced store.
    if constexpr (!DOTS) {
      constexpr int LD = BN + 4;  // padded row pitch (floats)
      float* stage_buf = reinterpret_cast<float*>(smem);
      if (ok) {
#pragma unroll
        for (int j = 0; j < C::COLS / 2; ++j)
          *reinterpret_cast<float2*>(stage_buf + row * LD + e * C::COLS + 2 * j) = acc[j];
      }
      named_barrier_sync(1, 128 * C::EPI_WG);
      if (ok) {
        const int et = threadIdx.x - 32 * C::EPI_WARP0;
        const int rows_here = min(C::BM, p.M - m0);
        for (int chunk = et; chunk < rows_here * (BN / 8); chunk += 128 * C::EPI_WG) {
          const int r = chunk / (BN / 8), c8 = (chunk % (BN / 8)) * 8;
          const int n = n0 + c8;
          if (n >= p.N) continue;
          const float4 lo = *reinterpret_cast<const float4*>(stage_buf + r * LD + c8);
          const float4 hi = *reinterpret_cast<const float4*>(stage_buf + r * LD + c8 + 4);
          const float a8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
          const int64_t orow = (int64_t)(m0 + r) * p.N;
          const bool native = TW && p.rowwise_order;
          const float as_r = native ? __ldg(p.act_scale + m0 + r) : 0.f;
          auto fin = [&](float a, int nn) { return native ? finish_native(a, p, nn, as_r) : finish(a, p, nn); };
          if (p.out_vec_ok && n + 8 <= p.N && p.out_dtype != kDtF32) {
            float y[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) y[t] = fin(a8[t], n + t);
            uint4 v;
            if (p.out_dtype == kDtBF16) {
              __nv_bfloat162 h0 = __floats2bfloat162_rn(y[0], y[1]), h1 = __floats2bfloat162_rn(y[2], y[3]);
              __nv_bfloat162 h2 = __floats2bfloat162_rn(y[4], y[5]), h3 = __floats2bfloat162_rn(y[6], y[7]);
              v = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                             *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
            } else {
              __half2 h0 = __floats2half2_rn(y[0], y[1]), h1 = __floats2half2_rn(y[2], y[3]);
              __half2 h2 = __floats2half2_rn(y[4], y[5]), h3 = __floats2half2_rn(y[6], y[7]);
              v = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                             *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
            }
            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + orow + n) = v;
          } else {
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (n + t < p.N) store_scalar(p, orow + n + t, fin(a8[t], n + t));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  // Launched early after another part of the same GEMM: finish only after it, so that
  // the stream's next operation sees both (returns at once without such a launch).
  if (threadIdx.x == 0) griddep_wait();
}

// Host-side launch (defined per W in gemm_w*.cu).  `pdl`: launch with programmatic
// stream serialization (the previous kernel in the stream must be the launch of
// another column range of the same GEMM).
template <int W, int A, int BN>
cudaError_t launch_group64_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                cudaStream_t stream, bool pdl = false);
// The same GEMM at two CTAs per SM (Group64Cfg OCC = 2).
template <int W, int A, int BN>
cudaError_t launch_group64_gemm_x2(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                   cudaStream_t stream);
// Persistent form (gemm_group64_persistent.cuh): bf16 / f16 output through a TMA
// store map `tm_out` (uint8 view of [M, N*2] bytes, box 128 B x 128 rows, 128B
// swizzle); BN 64 or 128; TW selects the row-scaled mode.
template <int W, int A, int BN, bool TW>
cudaError_t launch_group64_persistent(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const CUtensorMap& tm_out,
                                      const GemmParams& p, int num_sms, cudaStream_t stream);
// Row-scaled mode (per-token act_scale [M]; A = 8 tokenwise, A = 4 per-row A4).
template <int W, int A, int BN>
cudaError_t launch_group64_tokenwise(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                                     cudaStream_t stream, bool pdl = false);

}  // namespace actune
