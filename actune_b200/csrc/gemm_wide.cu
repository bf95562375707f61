// Group-64 tile GEMM with four-group stages for narrow weight tiles (32 or 64 rows),
// which AUTO picks for few token tiles and narrow outputs, for every W x A pair:
// int8 codes (W = A = 8, the decoded-code path) load straight into the operand
// layout, packed sub-byte codes through a staging area that four converter warps
// expand to int8 (code in the top bits of the byte, as in gemm_group64.cuh).
//
// Same arithmetic as group64_gemm_kernel (gemm_group64.cuh): exact int32 dots per
// 64-group on tcgen05 kind::i8, then acc = fma(float(dot_g), as[m, g], acc) for
// g = 0, 1, ... in order and y = fma(acc, ws[n], bias[n]) (or acc * ws[n]), rounded
// once (actune/kernels/grouped.py:80-94, actune/kernels/grouped_native.cu:70-85).
//
// Why a separate kernel: with few token tiles the K loop of one CTA is the whole
// critical path, and per stage it pays a fixed cost besides its MMAs -- the operand
// and accumulator waits, one commit for the accumulators and one for the ring slot,
// each holding the issuing thread about as long as an MMA.  A stage of 256 K (four
// groups, 8 MMAs) pays that cost once per four groups instead of once per two.
//
// Layout: a stage holds each operand as K/128 column blocks of 128-byte rows in the
// canonical 128-byte-swizzled K-major layout (token blocks 128 rows, of which a single
// tile's token box fills the first M rounded up to 8; weight blocks BN rows), and
// packed sub-byte codes in a staging area after them.  Tensor memory holds NSET sets
// of GS accumulators of BN int32 columns.  Roles: warp 0 producer
// (lanes 0..KB-1 the token blocks, lanes KB..2KB-1 the weight blocks of a stage, one
// instruction), warp 1 and the last warp MMA issuers (even and odd stages: one issuing
// thread is held for each MMA's duration, so one issuer's waits and commits overlap the
// other's MMAs), with sub-byte operands four converter warps, then eight epilogue warps
// (one token row and BN/2 columns per thread).  Every wait is bounded (common.cuh:
// mbar_wait records ACTUNE_DEV_TIMEOUT and returns false).
#include "kernels.cuh"

namespace actune {

template <int W, int A, int BN, int GS>
struct WideCfg {
  static_assert(W == 2 || W == 4 || W == 8, "W");
  static_assert(A == 2 || A == 4 || A == 8, "A");
  static_assert(BN == 32 || BN == 64, "narrow weight tiles");
  static_assert(GS == 4 || GS == 8, "groups per stage");
  static constexpr int BM = 128;                  // MMA M = TMEM lanes
  static constexpr int KS = 64 * GS;              // K codes (bytes) per stage
  static constexpr int KB = KS / 128;             // 128-byte column blocks per operand row
  static constexpr int EPI_WG = 2;
  static constexpr int COLS = BN / EPI_WG;        // accumulator columns per epilogue thread
  static constexpr int SET_COLS = GS * BN;        // tensor-memory columns of one stage
  static constexpr int NSET = 512 / SET_COLS;
  static_assert(NSET >= 2 && NSET % 2 == 0, "an even number of accumulator sets (two issuers)");
  static constexpr int A_BLK_BYTES = BM * 128;
  static constexpr int W_BLK_BYTES = BN * 128;
  static constexpr int OP_A_BYTES = KB * A_BLK_BYTES;
  static constexpr int OP_W_BYTES = KB * W_BLK_BYTES;
  // Packed sub-byte codes of a 128-K block: rows of 16 * bits bytes, unswizzled.
  static constexpr bool CONVERT = (A < 8) || (W < 8);
  static constexpr int STG_A_BLK = A < 8 ? BM * 16 * A : 0;
  static constexpr int STG_W_BLK = W < 8 ? BN * 16 * W : 0;
  static constexpr int STG_A_OFF = OP_A_BYTES + OP_W_BYTES;
  static constexpr int STG_W_OFF = STG_A_OFF + KB * STG_A_BLK;
  static constexpr int STAGE_RAW = STG_W_OFF + KB * STG_W_BLK;
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int STAGES_FIT = (200 * 1024) / STAGE_BYTES;
  // Even: each issuer owns every second ring slot (its descriptors stay in registers).
  static constexpr int STAGES = (STAGES_FIT > 8 ? 8 : STAGES_FIT) / 2 * 2;
  static_assert(STAGES >= 2, "ring depth");
  // int8 operand value = code * 2^(8 - bits): a dot carries 2^SHIFT.
  static constexpr int SHIFT = (8 - A) + (8 - W);
  static constexpr int OUT_STAGE_BYTES = BM * (BN + 4) * 4;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES > OUT_STAGE_BYTES ? STAGES * STAGE_BYTES : OUT_STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + 1024;
  static constexpr int CVT_WARPS = CONVERT ? 4 : 0;
  static constexpr int EPI_WARP0 = 2 + CVT_WARPS;
  static constexpr int EPI_WARPS = 4 * EPI_WG;
  static constexpr int MMA2_WARP = EPI_WARP0 + EPI_WARPS;
  static constexpr int THREADS = 32 * (MMA2_WARP + 1);
  // Groups read per tensor-memory wait: as many as 64 dot registers per thread hold.
  static constexpr int HG = COLS * GS <= 64 ? GS : 64 / COLS;
  static_assert(GS % HG == 0, "whole waits per stage");
};

template <int W, int A, int BN, int GS>
__global__ void __launch_bounds__(WideCfg<W, A, BN, GS>::THREADS, 1)
    group64_wide_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_wgt,
                        const GemmParams p) {
  using C = WideCfg<W, A, BN, GS>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];  // the stage's copies landed
  __shared__ __align__(8) uint64_t full_op[C::STAGES];   // converter warps done (sub-byte operands)
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t acc_full[C::NSET];
  __shared__ __align__(8) uint64_t acc_empty[C::NSET];
  __shared__ __align__(8) uint64_t mma_done[2];
  __shared__ uint32_t tmem_holder;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_iters = (G + GS - 1) / GS;
  const int m0 = blockIdx.x * C::BM;
  const int n0 = p.n_base + blockIdx.y * BN;
  // The next kernel in the stream may start as SMs come free; it waits for this one
  // before reading what this one writes.
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&full_op[s], C::CVT_WARPS > 0 ? C::CVT_WARPS : 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < C::NSET; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::EPI_WARPS);
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
    tmem_alloc(&tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One bulk-tensor instruction per stage: lane b < KB copies token block b, lane
    // KB + b weight block b.  Every operand of a copy sits in a register of its own
    // (a copy reads its register operands some time after issue).
    // Packed operands: a 128-K block is a box of 16 * bits bytes per row into the
    // staging area; int8 codes: 128 bytes per row straight into the operand block.
    int issued = 0;
    const uint32_t tx_bytes = (uint32_t)C::KB * (uint32_t)(p.a_box_rows * 16 * A + BN * 16 * W);
    if (lane < 2 * C::KB) {
      const bool is_a = lane < C::KB;
      const int blk = is_a ? lane : lane - C::KB;
      const CUtensorMap* map = is_a ? &tm_act : &tm_wgt;
      const int y = is_a ? m0 : n0;
      const int bits = is_a ? A : W;
      const uint32_t dst_off = is_a ? (A < 8 ? C::STG_A_OFF + blk * C::STG_A_BLK : blk * C::A_BLK_BYTES)
                                    : (W < 8 ? C::STG_W_OFF + blk * C::STG_W_BLK : C::OP_A_BYTES + blk * C::W_BLK_BYTES);
      const int x_step = C::KS * bits / 8, x_blk = blk * 16 * bits;
      constexpr int S = C::STAGES, HALF = C::STAGES / 2;
      uint32_t dst[S], bar[S];
      int xs[S];
#pragma unroll
      for (int j = 0; j < S; ++j) {
        dst[j] = smem_u32(smem + j * C::STAGE_BYTES + dst_off);
        bar[j] = smem_u32(&full_bar[j]);
        xs[j] = j * x_step + x_blk;
      }
      // Dependent launch: the tiles are requested once the previous kernel completed.
      if (p.pdl_wait) griddep_wait();
      const uint32_t mask = (1u << (2 * C::KB)) - 1u;
      uint32_t ph = 0;
      bool ok = true;
      for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          if (it0 + j >= n_iters) break;
          bool w_ok = true;
          if (lane == 0) {
            w_ok = mbar_wait(&empty_bar[j], ph ^ 1, kSiteProducer);
            if (w_ok) mbar_arrive_expect_tx(&full_bar[j], tx_bytes);
          }
          if (!__shfl_sync(mask, w_ok, 0)) {
            ok = false;
            break;
          }
          if (j + HALF < S) xs[j + HALF] = (it0 + j + HALF) * x_step + x_blk;
          tma_load_2d_u32(dst[j], map, xs[j], y, bar[j]);
          ++issued;
          if (j >= HALF) xs[j - HALF] = (it0 + S + j - HALF) * x_step + x_blk;
        }
        ph ^= 1;
      }
    }
    // Never leave the CTA with bulk copies still landing in shared memory.
    if (lane == 0) {
      for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it)
        mbar_wait(&full_bar[it % C::STAGES], (it / C::STAGES) & 1, kSiteDrain);
    }
  } else if (warp == 1 || warp == C::MMA2_WARP) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues the even stages, the last warp the odd ones.  Per stage: wait for
    // the operands and for the stage's accumulator set, 2 MMAs per group, one commit
    // to the set, one to the ring slot.  Descriptors of the issuer's own slots stay in
    // registers of their own (an MMA reads them when the tensor core takes it).
    const int who = warp == 1 ? 0 : 1;
    if (lane == 0) {
      constexpr int S = C::STAGES, NS = S / 2, KSTEPS = 2 * GS;
      constexpr uint32_t idesc = idesc_i8(C::BM, BN);
      const uint64_t desc_a0 = smem_desc_sw128(smem_u32(smem));
      const uint64_t desc_w0 = smem_desc_sw128(smem_u32(smem) + C::OP_A_BYTES);
      uint64_t da[NS][KSTEPS], dw[NS][KSTEPS];
#pragma unroll
      for (int u = 0; u < NS; ++u)
#pragma unroll
        for (int c = 0; c < KSTEPS; ++c) {
          // k-step c: 32 bytes at column block c / 4, offset (c % 4) * 32 within it.
          const uint64_t slot = (uint64_t)(((who + 2 * u) * C::STAGE_BYTES) >> 4);
          da[u][c] = desc_a0 + slot + (uint64_t)(((c / 4) * C::A_BLK_BYTES) >> 4) + 2 * (c % 4);
          dw[u][c] = desc_w0 + slot + (uint64_t)(((c / 4) * C::W_BLK_BYTES) >> 4) + 2 * (c % 4);
        }
      uint32_t ph = 0;
      bool ok = true;
      auto run = [&](auto parity_tag) {
        constexpr int PAR = decltype(parity_tag)::value;
        for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
          for (int j = PAR; j < S; j += 2) {
            const int it = it0 + j;
            if (it >= n_iters) break;
            const int set = it % C::NSET, u = j / 2;
            if (!mbar_wait(C::CONVERT ? &full_op[j] : &full_bar[j], ph, kSiteMmaFull) ||
                !mbar_wait(&acc_empty[set], ((it / C::NSET) & 1) ^ 1, kSiteMmaAcc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d0 = tmem_base + set * C::SET_COLS;
            // Past the end of K the operand blocks are the TMA's zero fill: those dots
            // are 0 and the epilogue gives them scale 0.
#pragma unroll
            for (int q = 0; q < GS; ++q) {
              mma_i8(d0 + q * BN, da[u][2 * q], dw[u][2 * q], idesc, 0u);
              mma_i8(d0 + q * BN, da[u][2 * q + 1], dw[u][2 * q + 1], idesc, 1u);
            }
            mma_commit(&acc_full[set]);
            mma_commit(&empty_bar[j]);
          }
          ph ^= 1;
        }
      };
      if (who == 0) run(std::integral_constant<int, 0>{});
      else run(std::integral_constant<int, 1>{});
      mma_commit(&mma_done[who]);
      mbar_wait(&mma_done[who], 0, kSiteMmaDone);
    }
  } else if (warp < C::EPI_WARP0) {
    // ------------------------------------------------------------ converters
    // Sub-byte codes of each 128-K block -> int8 in the canonical SW128 K-major layout
    // (token rows past the last token are left as they are: they reach only
    // accumulator rows that are never stored).
    if constexpr (C::CONVERT) {
      const int ctid = threadIdx.x - 64;
      constexpr int NT = 32 * C::CVT_WARPS;
      const int a_rows_valid = min(C::BM, p.M - m0);
      for (int it = 0; it < n_iters; ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(&full_bar[s], (it / C::STAGES) & 1, kSiteConverter)) break;
        uint8_t* st = smem + s * C::STAGE_BYTES;
#pragma unroll
        for (int b = 0; b < C::KB; ++b) {
          if constexpr (A < 8)
            unpack_stage<A, C::BM, NT>(st + C::STG_A_OFF + b * C::STG_A_BLK, st + b * C::A_BLK_BYTES, ctid,
                                       a_rows_valid);
          if constexpr (W < 8)
            unpack_stage<W, BN, NT>(st + C::STG_W_OFF + b * C::STG_W_BLK, st + C::OP_A_BYTES + b * C::W_BLK_BYTES,
                                    ctid);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_op[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Dependent launch: while the previous kernel finishes, pull this tile's first
    // weight blocks into L2 (they never depend on it); activation scales and the output
    // may belong to the previous kernel, so wait for it before touching them.
    if (p.pdl_wait) {
      if (warp == C::EPI_WARP0 && lane == 0) {
        const int pre = min(C::STAGES, n_iters);
        for (int j = 0; j < pre; ++j)
          for (int b = 0; b < C::KB; ++b) tma_prefetch_l2_2d(&tm_wgt, j * (C::KS * W / 8) + b * 16 * W, n0);
      }
      griddep_wait();
    }
    const int ew = warp - C::EPI_WARP0;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int e = ew >> 2;   // column slice
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const bool warp_live = (m0 + q * 32) < p.M;
    const bool load_scales = warp_live && m < p.M;
    const float* as_row = p.act_scale + (int64_t)(m < p.M ? m : 0) * G;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + e * C::COLS;
    float2 acc[C::COLS / 2];
#pragma unroll
    for (int j = 0; j < C::COLS / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    // Scales carry 2^-SHIFT (exact: a power of two) for the top-bit placement of
    // sub-byte codes; 1 for int8 codes.
    const float shift_scale = 1.0f / float(1 << C::SHIFT);
    auto scale_at = [&](int g) -> float {
      return (load_scales && g < G) ? __ldg(as_row + g) * shift_scale : 0.f;
    };
    bool ok = true;
    if (!warp_live) {
      // No valid token row in this warp: only keep the accumulator handshake.
      for (int it = 0; it < n_iters; ++it) {
        const int set = it % C::NSET;
        if (!mbar_wait(&acc_full[set], (it / C::NSET) & 1, kSiteEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[set]);
      }
    } else {
      float sc[GS], sn[GS];
#pragma unroll
      for (int h = 0; h < GS; ++h) sc[h] = scale_at(h);
      uint32_t r[C::HG][C::COLS];
      for (int it = 0; it < n_iters; ++it) {
#pragma unroll
        for (int h = 0; h < GS; ++h) sn[h] = scale_at((it + 1) * GS + h);
        const int set = it % C::NSET;
        if (!mbar_wait(&acc_full[set], (it / C::NSET) & 1, kSiteEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = lane_base + set * C::SET_COLS;
        // Groups past the end of K have dot 0 and scale 0: acc += 0 * 0 leaves every
        // accumulator unchanged (an accumulator is never -0).
#pragma unroll
        for (int half = 0; half < GS / C::HG; ++half) {
#pragma unroll
          for (int h = 0; h < C::HG; ++h) tmem_ld<C::COLS>(base + (half * C::HG + h) * BN, r[h]);
          tmem_wait_ld();
          if (half == GS / C::HG - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[set]);
          }
#pragma unroll
          for (int h = 0; h < C::HG; ++h) accumulate<C::COLS>(acc, r[h], sc[half * C::HG + h]);
        }
#pragma unroll
        for (int h = 0; h < GS; ++h) sc[h] = sn[h];
      }
    }

    // Final epilogue: stage the fp32 accumulators through the (now idle) ring, then
    // every epilogue thread applies ws / bias to 8 consecutive columns of one row and
    // writes them with one coalesced store.
    constexpr int LD = BN + 4;
    float* stage_buf = reinterpret_cast<float*>(smem);
    if (ok) {
#pragma unroll
      for (int j = 0; j < C::COLS / 2; ++j)
        *reinterpret_cast<float2*>(stage_buf + row * LD + e * C::COLS + 2 * j) = acc[j];
    }
    named_barrier_sync(1, 32 * C::EPI_WARPS);
    if (ok) {
      const int et = threadIdx.x - 32 * C::EPI_WARP0;
      const int rows_here = min(C::BM, p.M - m0);
      for (int chunk = et; chunk < rows_here * (BN / 8); chunk += 32 * C::EPI_WARPS) {
        const int rr = chunk / (BN / 8), c8 = (chunk % (BN / 8)) * 8;
        const int n = n0 + c8;
        if (n >= p.N) continue;
        const float4 lo = *reinterpret_cast<const float4*>(stage_buf + rr * LD + c8);
        const float4 hi = *reinterpret_cast<const float4*>(stage_buf + rr * LD + c8 + 4);
        const float a8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        const int64_t orow = (int64_t)(m0 + rr) * p.N;
        if (p.out_vec_ok && n + 8 <= p.N && p.out_dtype != kDtF32) {
          float yv[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) yv[t] = finish(a8[t], p, n + t);
          uint4 v;
          if (p.out_dtype == kDtBF16) {
            __nv_bfloat162 h0 = __floats2bfloat162_rn(yv[0], yv[1]), h1 = __floats2bfloat162_rn(yv[2], yv[3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(yv[4], yv[5]), h3 = __floats2bfloat162_rn(yv[6], yv[7]);
            v = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                           *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
          } else {
            __half2 h0 = __floats2half2_rn(yv[0], yv[1]), h1 = __floats2half2_rn(yv[2], yv[3]);
            __half2 h2 = __floats2half2_rn(yv[4], yv[5]), h3 = __floats2half2_rn(yv[6], yv[7]);
            v = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                           *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
          }
          *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + orow + n) = v;
        } else {
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (n + t < p.N) store_scalar(p, orow + n + t, finish(a8[t], p, n + t));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0) griddep_wait();
}

template <int W, int A, int BN, int GS>
static cudaError_t launch_wide_t(const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                                 cudaStream_t stream) {
  using C = WideCfg<W, A, BN, GS>;
  constexpr auto kernel = group64_wide_kernel<W, A, BN, GS>;
  const cudaError_t e = ensure_smem_limit<kernel>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int n_end = p.n_end > 0 ? p.n_end : p.N;
  const dim3 grid((p.M + C::BM - 1) / C::BM, (n_end - p.n_base + BN - 1) / BN);
  return launch_pdl(kernel, grid, C::THREADS, C::SMEM_BYTES, stream, ta, tw, p);
}

template <int W, int A>
static cudaError_t launch_wide_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                                  cudaStream_t stream) {
  if (bn == 32) return launch_wide_t<W, A, 32, 4>(ta, tw, p, stream);
  if (bn == 64) return launch_wide_t<W, A, 64, 4>(ta, tw, p, stream);
  return cudaErrorInvalidValue;
}

template <int W, int A>
static bool wide_deep_ring(int bn) {
  return bn == 32 ? WideCfg<W, A, 32, 4>::STAGES >= 4 : bn == 64 ? WideCfg<W, A, 64, 4>::STAGES >= 4 : false;
}

bool group64_wide_preferred(int W, int A, int bn) {
#define ACTUNE_CASE(WW, AA) \
  if (W == WW && A == AA) return wide_deep_ring<WW, AA>(bn);
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return false;
}

cudaError_t launch_group64_wide(int W, int A, int bn, int gs, const CUtensorMap& ta, const CUtensorMap& tw,
                                const GemmParams& p, cudaStream_t stream) {
  if (p.dots != nullptr || gs != 4) return cudaErrorInvalidValue;
#define ACTUNE_CASE(WW, AA) \
  if (W == WW && A == AA) return launch_wide_bn<WW, AA>(bn, ta, tw, p, stream);
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

}  // namespace actune
