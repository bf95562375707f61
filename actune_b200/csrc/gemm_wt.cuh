// Packed-integer group-64 linear, weights-in-tensor-memory form (sm_100a).
//
//   y[m, n] = ws[n] * sum_g ( float(dot_g(m, n)) * as[m, g] )  (+ bias[n])
//   dot_g(m, n) = sum_{k in group g} a[m, k] * w[n, k]          (exact int32)
//
// with the fp32 chain of the reference's GPU kernels (actune/kernels/grouped.py:80-94,
// actune/kernels/grouped_native.cu:70-85): acc = fma(float(dot_g), as[m, g], acc) for
// g = 0, 1, ... in order, then y = fma(acc, ws[n], bias[n]) (acc * ws[n] without bias),
// rounded once to the output type.
//
// Orientation: the MMA computes D[n, m] = W[n, :] . X[m, :] with the weight tile as the
// M = 128 operand held in TENSOR MEMORY and the token tile (BT rows) as the N operand in
// shared memory.  Sub-byte weight codes are expanded to int8 by converter threads
// straight from registers into TMEM (tcgen05.st), so the expanded weights never take a
// shared-memory round trip; the only shared-memory traffic of the weight stream is the
// packed tile written by TMA and read once by the converters.  Shared memory is the
// scarce resource next to the tensor core: a 128 x 128 x 32 int8 MMA reading both
// operands from it uses 128 B/clk, which starves ordinary loads and stores.
//
// Warp roles (one CTA per SM):
//   warp 0        TMA producer: token tile (int8, or packed for A < 8) and packed
//                 weight tile of each 128-wide K stage -> shared-memory ring
//   warp 1        TMEM owner + single-thread tcgen05.mma issuer
//   warps 2-5     converters, one per TMEM lane quarter: thread = weight row; packed
//                 row -> int8 codes in registers -> tcgen05.st into the TMEM A ring;
//                 also expand sub-byte activations (A < 8) into the shared-memory B
//                 operand and stage the stage's activation scales transposed
//   warps 6..     epilogue: per 64-wide group, tcgen05.ld of the int32 dots (lane =
//                 weight row, column = token), exact int->fp32, packed fp32x2 FMA with
//                 the per-token scales; final ws/bias/convert through shared memory
#pragma once

#include "common.cuh"
#include "gemm_group64.cuh"  // GemmParams, dtype ids, load_bias/store helpers

namespace actune {

template <int W, int A, int BT>
struct WtCfg {
  static_assert(W == 2 || W == 4 || W == 8, "W");
  static_assert(A == 2 || A == 4 || A == 8, "A");
  static_assert(BT == 16 || BT == 32 || BT == 64 || BT == 128, "BT");
  static constexpr int BM = 128;                 // weight rows per tile (MMA M, TMEM lanes)
  static constexpr int KS = 128;                 // K per stage = two groups of 64
  static constexpr int EPI_WG = BT >= 64 ? 2 : 1;
  static constexpr int COLS = BT / EPI_WG;       // token columns per epilogue thread
  static constexpr int H = COLS >= 64 ? 32 : COLS / 2;  // columns per tcgen05.ld
  static constexpr int NCH = COLS / H;           // chunks per group (2)
  static constexpr int CONV_WARPS = 4;
  static constexpr int EPI_WARP0 = 2 + CONV_WARPS;
  static constexpr int THREADS = 32 * (EPI_WARP0 + 4 * EPI_WG);
  // Shared memory per stage: [B operand int8 SW128 | B staging (A < 8) | packed weights].
  static constexpr int OPB_BYTES = BT * KS;
  static constexpr int STGB_BYTES = A < 8 ? BT * KS * A / 8 : 0;
  static constexpr int WP_BYTES = BM * KS * W / 8;
  static constexpr int WP_OFF = (OPB_BYTES + STGB_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGE_BYTES = (WP_OFF + WP_BYTES + 1023) / 1024 * 1024;
  static constexpr int SC_SLOTS = 8;             // activation-scale ring (2 groups x BT floats each)
  static constexpr int SC_BYTES = SC_SLOTS * 2 * BT * 4;
  static constexpr int STAGES_FIT = (200 * 1024 - SC_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int OUT_STAGE_BYTES = BT * BM * 4;  // final fp32-or-narrower staging
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES > OUT_STAGE_BYTES ? STAGES * STAGE_BYTES : OUT_STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + SC_BYTES + 1024;
  // TMEM: NB group accumulators of BT columns, then SA weight stages of 32 columns (128 B of K per row).
  // The TMEM weight ring has one 32-column slot per shared-memory stage, so the
  // stage's "MMA done" barrier also frees its TMEM slot.
  static constexpr int NB = 2;
  static constexpr int SA = STAGES;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t TX_BYTES = BT * KS * A / 8 + BM * KS * W / 8;
  static constexpr int SHIFT = (8 - A) + (8 - W);
  static_assert(STAGES >= 2 && SA >= 2, "pipeline depth");
  static_assert(NB * BT + SA * 32 <= TMEM_COLS, "tmem budget");
};

// Expand sub-byte codes of one packed row chunk (16 bytes) to int8 in the top bits.
__device__ __forceinline__ void expand_w4(const uint4 v, uint32_t* o) {
  const uint2 a = unpack_w4_word(v.x), b = unpack_w4_word(v.y), c = unpack_w4_word(v.z), d = unpack_w4_word(v.w);
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y; o[4] = c.x; o[5] = c.y; o[6] = d.x; o[7] = d.y;
}
__device__ __forceinline__ void expand_w2(const uint4 v, uint32_t* o) {
  const uint4 a = unpack_w2_word(v.x), b = unpack_w2_word(v.y), c = unpack_w2_word(v.z), d = unpack_w2_word(v.w);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  o[8] = c.x; o[9] = c.y; o[10] = c.z; o[11] = c.w; o[12] = d.x; o[13] = d.y; o[14] = d.z; o[15] = d.w;
}

// One weight row of a stage (128 codes) from the TMA-swizzled packed tile -> 32 words of
// int8 codes in K order.  The TMA tile is [128 rows x 16*W bytes] written with the
// swizzle that matches its row width (SW128 / SW64 / SW32), which XORs the 16-byte chunk
// index with bits 7.. of the byte offset; reading chunk c of all 32 rows of a warp then
// touches every bank group exactly as often as the 512 bytes require.
template <int W>
__device__ __forceinline__ void load_weight_row(const uint8_t* tile, int r, uint32_t (&o)[32]) {
  constexpr int RB = 16 * W;  // packed bytes per row
  const uint8_t* row = tile + r * RB;
  if constexpr (W == 8) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4));
      o[4 * c] = v.x; o[4 * c + 1] = v.y; o[4 * c + 2] = v.z; o[4 * c + 3] = v.w;
    }
  } else if constexpr (W == 4) {
    const int x = (r >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c) expand_w4(*reinterpret_cast<const uint4*>(row + ((c ^ x) << 4)), o + 8 * c);
  } else {
    const int x = (r >> 2) & 1;
#pragma unroll
    for (int c = 0; c < 2; ++c) expand_w2(*reinterpret_cast<const uint4*>(row + ((c ^ x) << 4)), o + 16 * c);
  }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, int8 x int8 -> int32, issued by one thread.
__device__ __forceinline__ void mma_i8_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Sub-byte activation staging (ROWS rows x 16*BITS bytes, no swizzle) -> SW128 int8
// operand (row pitch 128 bytes, chunk c of row r at chunk c ^ (r & 7)).
template <int BITS, int ROWS, int NT>
__device__ __forceinline__ void expand_act_stage(const uint8_t* __restrict__ stg, uint8_t* __restrict__ op, int tid) {
  constexpr int IPR = BITS;  // 16-byte items per row
  constexpr int ITEMS = ROWS * IPR;
#pragma unroll 2
  for (int item = tid; item < ITEMS; item += NT) {
    const int r = item / IPR, i = item % IPR;
    const uint4 v = *reinterpret_cast<const uint4*>(stg + item * 16);
    uint8_t* row = op + (r >> 3) * 1024 + (r & 7) * 128;
    const int x = r & 7;
    if constexpr (BITS == 4) {
      uint32_t o[8];
      expand_w4(v, o);
      *reinterpret_cast<uint4*>(row + (((2 * i) ^ x) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(row + (((2 * i + 1) ^ x) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
      uint32_t o[16];
      expand_w2(v, o);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(row + (((4 * i + q) ^ x) << 4)) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
    }
  }
}

enum : int { kWtSiteProducer = 11, kWtSiteConvFull, kWtSiteConvTmem, kWtSiteConvScale, kWtSiteMmaConv, kWtSiteMmaAcc,
             kWtSiteMmaDone, kWtSiteEpiScale, kWtSiteEpiAcc, kWtSiteDrain };

template <int W, int A, int BT, bool DOTS>
__global__ void __launch_bounds__(WtCfg<W, A, BT>::THREADS, 1)
    wt_gemm_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_wgt,
                   const GemmParams p) {
  using C = WtCfg<W, A, BT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];    // TMA landed (tx)
  __shared__ __align__(8) uint64_t conv_bar[C::STAGES];    // converters done with stage (4 warps)
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];   // MMA done with stage: smem + TMEM slot (commit)
  __shared__ __align__(8) uint64_t d_full[C::NB];          // group accumulator ready (commit)
  __shared__ __align__(8) uint64_t d_empty[C::NB];         // epilogue drained accumulator (epilogue warps)
  __shared__ __align__(8) uint64_t sc_full[C::SC_SLOTS];   // stage scales written (4 converter warps)
  __shared__ __align__(8) uint64_t sc_empty[C::SC_SLOTS];  // stage scales consumed (epilogue warps)
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_holder;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sc_ring = reinterpret_cast<float*>(smem + C::RING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_iters = (G + 1) >> 1;
  const int m0 = blockIdx.x * BT;   // token tile
  const int n0 = blockIdx.y * C::BM;  // weight-row tile
  constexpr int EPI_WARPS = 4 * C::EPI_WG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&conv_bar[s], C::CONV_WARPS);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < C::NB; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_empty[b], EPI_WARPS);
    }
    for (int s = 0; s < C::SC_SLOTS; ++s) {
      mbar_init(&sc_full[s], C::CONV_WARPS);
      mbar_init(&sc_empty[s], EPI_WARPS);
    }
    mbar_init(&mma_done, 1);
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
  const uint32_t tmem_a = tmem_base + C::NB * BT;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    // Lane 0 loads the token tile and lane 1 the weight tile of a stage in ONE
    // bulk-tensor instruction.  The loop is unrolled over the ring and every
    // operand of a copy (destination, barrier, coordinate) sits in a register of
    // its own: an asynchronous copy reads its register operands some time after
    // issue, and rewriting one of them for the next copy stalls until it has.  A
    // slot's coordinate is refreshed half a ring away from the copy that reads it.
    int issued = 0;
    if (lane < 2) {
      const CUtensorMap* map = lane == 0 ? &tm_act : &tm_wgt;
      const int x_step = lane == 0 ? C::KS * A / 8 : C::KS * W / 8;
      const int y = lane == 0 ? m0 : n0;
      const uint32_t dst_off = lane == 0 ? (A < 8 ? C::OPB_BYTES : 0) : C::WP_OFF;
      constexpr int S = C::STAGES, HALF = C::STAGES / 2;
      uint32_t dst[S], bar[S];
      int xs[S];
#pragma unroll
      for (int j = 0; j < S; ++j) {
        dst[j] = smem_u32(smem + j * C::STAGE_BYTES + dst_off);
        bar[j] = smem_u32(&full_bar[j]);
        xs[j] = j * x_step;
      }
      uint32_t ph = 0;
      bool ok = true;
      for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          if (it0 + j >= n_iters) break;
          bool w_ok = true;
          if (lane == 0) {
            w_ok = mbar_wait(&empty_bar[j], ph ^ 1, kWtSiteProducer);
            if (w_ok) mbar_arrive_expect_tx(&full_bar[j], C::TX_BYTES);
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
        mbar_wait(&full_bar[it % C::STAGES], (it / C::STAGES) & 1, kWtSiteDrain);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // Unrolled over the ring; every MMA of a ring cycle has its own precomputed
    // operand registers (see the producer), so issue runs at the tensor core's pace.
    if (lane == 0) {
      constexpr int S = C::STAGES;
      constexpr uint32_t idesc = idesc_i8(C::BM, BT);
      const uint64_t desc_b0 = smem_desc_sw128(smem_u32(smem));
      uint64_t db[S][4];
      uint32_t ta[S][4], bfull[S], bconv[S], bempty[S];
#pragma unroll
      for (int j = 0; j < S; ++j) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          db[j][k] = desc_b0 + (uint64_t)((j * C::STAGE_BYTES) >> 4) + 2 * k;  // +32 B of K per step
          ta[j][k] = tmem_a + j * 32 + 8 * k;                                   // +32 B of K = 8 columns
        }
        bfull[j] = smem_u32(&full_bar[j]);
        bconv[j] = smem_u32(&conv_bar[j]);
        bempty[j] = smem_u32(&empty_bar[j]);
      }
      const uint32_t d0 = tmem_base, d1 = tmem_base + BT;
      const uint32_t bdf0 = smem_u32(&d_full[0]), bdf1 = smem_u32(&d_full[1]);
      uint32_t ph = 0;
      bool ok = true;
      for (int it0 = 0; it0 < n_iters && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          if (it0 + j >= n_iters) break;
          // Two groups per stage, NB = 2: group 0 -> buffer 0, group 1 -> buffer 1,
          // each buffer's phase flips once per stage.
          const uint32_t phb = (it0 + j) & 1;
          ok = mbar_wait(&full_bar[j], ph, kWtSiteMmaConv) && mbar_wait(&conv_bar[j], ph, kWtSiteMmaConv) &&
               mbar_wait(&d_empty[0], phb ^ 1, kWtSiteMmaAcc);
          if (!ok) break;
          tc_fence_after();
          // Past the end of K (odd G) both tiles are the TMA's zero fill: dots 0, scale 0.
          mma_i8_tmem_a(d0, ta[j][0], db[j][0], idesc, 0u);
          mma_i8_tmem_a(d0, ta[j][1], db[j][1], idesc, 1u);
          mma_commit_u32(bdf0);
          if (!mbar_wait(&d_empty[1], phb ^ 1, kWtSiteMmaAcc)) { ok = false; break; }
          tc_fence_after();
          mma_i8_tmem_a(d1, ta[j][2], db[j][2], idesc, 0u);
          mma_i8_tmem_a(d1, ta[j][3], db[j][3], idesc, 1u);
          mma_commit_u32(bdf1);
          mma_commit_u32(bempty[j]);
        }
        ph ^= 1;
      }
      (void)bfull;
      (void)bconv;
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0, kWtSiteMmaDone);
    }
  } else if (warp < C::EPI_WARP0) {
    // ---------------------------------------------------------------- converters
    const int q = warp & 3;                 // TMEM lane quarter this warp may write
    const int r = q * 32 + lane;            // weight row within the tile
    const int ct = (warp - 2) * 32 + lane;  // converter thread id 0..127
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float shift_scale = 1.0f / float(1 << C::SHIFT);
    // Activation scales of this thread's tokens (ct, ct + 128 when BT > 128 -- not used).
    const int tok = ct;
    const bool tok_live = tok < BT && (m0 + tok) < p.M;
    const float* as_row = p.act_scale + (int64_t)(tok_live ? m0 + tok : 0) * G;
    auto scale_at = [&](int g) -> float {
      return (!DOTS && tok_live && g < G) ? __ldg(as_row + g) * shift_scale : 0.f;
    };
    int s = 0, sc = 0;
    uint32_t ph = 0, phc = 0;
    float nx0 = scale_at(0), nx1 = scale_at(1);
    for (int it = 0; it < n_iters; ++it) {
      const float c0 = nx0, c1 = nx1;
      nx0 = scale_at(2 * it + 2);
      nx1 = scale_at(2 * it + 3);
      if (!mbar_wait(&full_bar[s], ph, kWtSiteConvFull)) break;
      uint8_t* st = smem + s * C::STAGE_BYTES;
      uint32_t o[32];
      load_weight_row<W>(st + C::WP_OFF, r, o);
      if constexpr (A < 8) {
        expand_act_stage<A, BT, 128>(st + C::OPB_BYTES, st, ct);
        fence_proxy_async_smem();
      }
      // full[s] implies the producer saw empty[s]: the MMAs that last read this
      // TMEM slot (stage it - STAGES) have completed.
      tc_fence_after();
      tmem_st32(tmem_a + lane_off + s * 32, o);
      tmem_wait_st();
      if (!mbar_wait(&sc_empty[sc], phc ^ 1, kWtSiteConvScale)) break;
      if (tok < BT) {
        float* slot = sc_ring + sc * 2 * BT;
        slot[tok] = c0;
        slot[BT + tok] = c1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sc_full[sc]);
        mbar_arrive(&conv_bar[s]);
      }
      if (++s == C::STAGES) { s = 0; ph ^= 1; }
      if (++sc == C::SC_SLOTS) { sc = 0; phc ^= 1; }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp - C::EPI_WARP0;
    const int q = warp & 3;           // TMEM lane quarter
    const int e = ew >> 2;            // token-column slice
    const int r = q * 32 + lane;      // weight row within the tile
    const int n = n0 + r;
    const int col0 = e * C::COLS;     // first token column of this thread
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + col0;
    constexpr int H = C::H;
    float2 acc[C::COLS / 2];
#pragma unroll
    for (int j = 0; j < C::COLS / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    const float2 magic = make_float2(-kMagicValue, -kMagicValue);
    bool ok = true;
    int b = 0, sc = 0;
    uint32_t phb = 0, phc = 0;
    for (int it = 0; it < n_iters && ok; ++it) {
      if (!mbar_wait(&sc_full[sc], phc, kWtSiteEpiScale)) { ok = false; break; }
      const float* slot = sc_ring + sc * 2 * BT + col0;
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int g = 2 * it + grp;
        if (!mbar_wait(&d_full[b], phb, kWtSiteEpiAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t base = lane_base + b * BT;
        const float* sg = slot + grp * BT;
        uint32_t ra[H], rb[H];
        tmem_ld<H>(base, ra);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) {
          uint32_t (&cur)[H] = (c & 1) ? rb : ra;
          uint32_t (&nxt)[H] = (c & 1) ? ra : rb;
          if (c + 1 < C::NCH) tmem_ld<H>(base + (c + 1) * H, nxt);
          if constexpr (DOTS) {
            if (n < p.N && g < G) {
#pragma unroll
              for (int j = 0; j < H; ++j) {
                const int m = m0 + col0 + c * H + j;
                if (m < p.M) p.dots[((int64_t)m * p.N + n) * G + g] = static_cast<int32_t>(cur[j]) >> C::SHIFT;
              }
            }
          } else {
#pragma unroll
            for (int j4 = 0; j4 < H / 4; ++j4) {
              const float4 s4 = *reinterpret_cast<const float4*>(sg + c * H + 4 * j4);
              float2 f0 = make_float2(__uint_as_float(cur[4 * j4] + kMagicBits), __uint_as_float(cur[4 * j4 + 1] + kMagicBits));
              float2 f1 = make_float2(__uint_as_float(cur[4 * j4 + 2] + kMagicBits), __uint_as_float(cur[4 * j4 + 3] + kMagicBits));
              f0 = fadd2(f0, magic);
              f1 = fadd2(f1, magic);
              acc[(c * H) / 2 + 2 * j4] = ffma2(f0, make_float2(s4.x, s4.y), acc[(c * H) / 2 + 2 * j4]);
              acc[(c * H) / 2 + 2 * j4 + 1] = ffma2(f1, make_float2(s4.z, s4.w), acc[(c * H) / 2 + 2 * j4 + 1]);
            }
          }
          if (c + 1 < C::NCH) tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[b]);
        if (++b == C::NB) { b = 0; phb ^= 1; }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[sc]);
      if (++sc == C::SC_SLOTS) { sc = 0; phc ^= 1; }
    }

    // Final epilogue: y = fma(acc, ws, bias) per (token, weight row), staged through
    // the idle ring as [token][row] so each output row segment is written with 16-byte
    // stores.  Every stage has been consumed by the MMA (its last accumulator is in),
    // so no bulk copy is landing in the ring any more.
    if constexpr (!DOTS) {
      const bool row_live = n < p.N;
      float ws = 0.f, bias = 0.f;
      if (row_live) {
        ws = __ldg(p.w_scale + n);
        if (p.bias_dtype != kDtNone) bias = load_bias(p.bias, p.bias_dtype, n);
      }
      const bool has_bias = p.bias_dtype != kDtNone;
      const int osz = p.out_dtype == kDtF32 ? 4 : 2;
      uint8_t* ostage = smem;
      named_barrier_sync(1, 32 * EPI_WARPS);
      if (ok) {
#pragma unroll
        for (int j = 0; j < C::COLS / 2; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float a = h ? acc[j].y : acc[j].x;
            const float y = has_bias ? fmaf(a, ws, bias) : a * ws;
            const int t = col0 + 2 * j + h;
            uint8_t* dst = ostage + ((size_t)t * C::BM + r) * osz;
            if (p.out_dtype == kDtBF16) *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16_rn(y);
            else if (p.out_dtype == kDtF16) *reinterpret_cast<__half*>(dst) = __float2half_rn(y);
            else *reinterpret_cast<float*>(dst) = y;
          }
        }
      }
      named_barrier_sync(1, 32 * EPI_WARPS);
      if (ok) {
        const int et = threadIdx.x - 32 * C::EPI_WARP0;
        const int rows_here = min(BT, p.M - m0);
        const int cols_here = min(C::BM, p.N - n0);
        const int row_bytes = C::BM * osz;
        const int chunks = row_bytes / 16;  // 16-byte pieces of a staged token row
        const bool vec = p.out_vec_ok && cols_here == C::BM;
        for (int idx = et; idx < rows_here * chunks; idx += 32 * EPI_WARPS) {
          const int t = idx / chunks, c = idx % chunks;
          const uint8_t* src = ostage + (size_t)t * row_bytes + c * 16;
          uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) + ((int64_t)(m0 + t) * p.N + n0) * osz + c * 16;
          if (vec) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
            for (int bb = 0; bb < 16; bb += osz) {
              const int col = (c * 16 + bb) / osz;
              if (col < cols_here) {
                if (osz == 4) *reinterpret_cast<float*>(dst + bb) = *reinterpret_cast<const float*>(src + bb);
                else *reinterpret_cast<uint16_t*>(dst + bb) = *reinterpret_cast<const uint16_t*>(src + bb);
              }
            }
          }
        }
      }
      (void)row_live;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Host-side launch (instantiated per W in gemm_wt_w*.cu with ACTUNE_INSTANTIATE_WT(W)).
template <int W, int A, int BT>
cudaError_t launch_wt_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                           cudaStream_t stream);

#ifdef ACTUNE_WT_LAUNCH_DEFINITIONS
template <int W, int A, int BT>
cudaError_t launch_wt_gemm(const CUtensorMap& tm_act, const CUtensorMap& tm_wgt, const GemmParams& p,
                           cudaStream_t stream) {
  using C = WtCfg<W, A, BT>;
  const bool dots = p.dots != nullptr;
  constexpr auto k_dots = wt_gemm_kernel<W, A, BT, true>;
  constexpr auto k_out = wt_gemm_kernel<W, A, BT, false>;
  const cudaError_t e = dots ? ensure_smem_limit<k_dots>(C::SMEM_BYTES) : ensure_smem_limit<k_out>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  auto kernel = dots ? k_dots : k_out;
  const dim3 grid((p.M + BT - 1) / BT, (p.N + C::BM - 1) / C::BM);
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tm_act, tm_wgt, p);
  return cudaGetLastError();
}
#endif

}  // namespace actune

// All token tiles (16, 32, 64, 128) for A in {2, 4, 8} at weight width W.
#define ACTUNE_WT_INST(W, A, BT) \
  template cudaError_t launch_wt_gemm<W, A, BT>(const CUtensorMap&, const CUtensorMap&, const GemmParams&, cudaStream_t);
#define ACTUNE_INSTANTIATE_WT(W)                                                                             \
  namespace actune {                                                                                         \
  ACTUNE_WT_INST(W, 2, 16) ACTUNE_WT_INST(W, 2, 32) ACTUNE_WT_INST(W, 2, 64) ACTUNE_WT_INST(W, 2, 128)       \
  ACTUNE_WT_INST(W, 4, 16) ACTUNE_WT_INST(W, 4, 32) ACTUNE_WT_INST(W, 4, 64) ACTUNE_WT_INST(W, 4, 128)       \
  ACTUNE_WT_INST(W, 8, 16) ACTUNE_WT_INST(W, 8, 32) ACTUNE_WT_INST(W, 8, 64) ACTUNE_WT_INST(W, 8, 128)       \
  }
