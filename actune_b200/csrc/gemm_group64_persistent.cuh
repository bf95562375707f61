// Persistent form of group64_gemm_kernel (explicit variants BN64P / BN128P).
//
// Same arithmetic, roles and stage pipeline as gemm_group64.cuh, but one CTA per
// SM walks the tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... (token tile
// fastest), so that the ring, the TMEM accumulators and the barriers run on
// across tile boundaries: the producer fetches the next tile's first stages and
// the MMA issuer starts it while the epilogue warps finish the previous tile,
// instead of every tile paying the pipeline fill, the teardown and a new CTA.
// The final store goes through a staging tile in shared memory (128B-swizzled,
// conflict-free from the row-per-thread registers) and one TMA store per 64
// columns, issued by one epilogue thread and completed in the background while
// the next tile accumulates.  Output: bf16 or f16, N % 8 == 0, 16-byte aligned.
//
// Row-scaled mode (TW, the tokenwise and per-row A4 backends): one full-K
// accumulator per tile, two of them alternating between tiles.
#pragma once

#include "gemm_group64.cuh"

namespace actune {

template <int W, int A, int BN, bool TW>
struct PersistCfg {
  using B = Group64Cfg<W, A, BN>;
  static_assert(BN == 64 || BN == 128, "persistent tiles are 64 or 128 weight rows");
  static constexpr int OUT_BOX_COLS = 64;                   // 128 bytes of 16-bit outputs
  static constexpr int BOXES = BN / OUT_BOX_COLS;
  static constexpr int OUT_BYTES = B::BM * BN * 2;          // staging tile [box][row][128 B]
  static constexpr int SLOT_MULT = B::NPAIR > 2 ? B::NPAIR : 2;
  static constexpr int RING_FIT = (224 * 1024 - OUT_BYTES) / B::STAGE_BYTES;
  static constexpr int STAGES = (RING_FIT > 8 ? 8 : RING_FIT) / SLOT_MULT * SLOT_MULT;
  static constexpr int SMEM_BYTES = STAGES * B::STAGE_BYTES + OUT_BYTES + 1024;
  static constexpr int NACC = TW ? 2 : B::NPAIR;            // accumulator buffers (barrier pairs)
  static constexpr int TMEM_COLS = TW ? 2 * BN : B::TMEM_COLS;
  static_assert(STAGES >= 2, "stages");
};

template <int W, int A, int BN, bool TW>
__global__ void __launch_bounds__(Group64Cfg<W, A, BN>::THREADS, 1)
    group64_gemm_persistent_kernel(const __grid_constant__ CUtensorMap tm_act,
                                   const __grid_constant__ CUtensorMap tm_wgt,
                                   const __grid_constant__ CUtensorMap tm_out, const GemmParams p) {
  using B = Group64Cfg<W, A, BN>;
  using C = PersistCfg<W, A, BN, TW>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_raw[S];
  __shared__ __align__(8) uint64_t full_op[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full[C::NACC];
  __shared__ __align__(8) uint64_t acc_empty[C::NACC];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_holder;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_stage = smem + S * B::STAGE_BYTES;  // 1024-aligned: STAGE_BYTES is a multiple of 1024
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_iters = (G + 1) >> 1;
  const int m_tiles = (p.M + B::BM - 1) / B::BM;
  const int tiles = m_tiles * ((p.N + BN - 1) / BN);
  const int my_tiles = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * n_iters;
  auto tile_m0 = [&](int lt) { return (((int)blockIdx.x + lt * (int)gridDim.x) % m_tiles) * B::BM; };
  auto tile_n0 = [&](int lt) { return (((int)blockIdx.x + lt * (int)gridDim.x) / m_tiles) * BN; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&full_op[s], B::CVT_WARPS > 0 ? B::CVT_WARPS : 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * B::EPI_WG);
    }
    mbar_init(&mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_act);
    prefetch_tensormap(&tm_wgt);
    prefetch_tensormap(&tm_out);
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
    // As in the one-tile kernel: lanes 0 and 1 issue a stage's token and weight
    // boxes in one instruction, the ring loop is unrolled and each slot's copy
    // operands are rewritten only half a ring after their copy was issued.
    int issued = 0;
    if (lane < 2) {
      const CUtensorMap* map = lane == 0 ? &tm_act : &tm_wgt;
      const int x_step = lane == 0 ? B::KS * A / 8 : B::KS * W / 8;
      const uint32_t dst_off = lane == 0 ? (A < 8 ? B::OP_A_BYTES + B::OP_W_BYTES : 0)
                                         : (W < 8 ? B::OP_A_BYTES + B::OP_W_BYTES + B::STG_A_BYTES : B::OP_A_BYTES);
      constexpr int HALF = S / 2;
      // Stage `it` of the walk: k-stage it % n_iters of local tile it / n_iters.  The
      // coordinates are advanced one stage at a time (no division per stage; one
      // per tile boundary) by a cursor that runs HALF stages ahead of the issue.
      int c_kst = 0, c_lt = 0, c_y = lane == 0 ? tile_m0(0) : tile_n0(0);
      auto advance = [&]() {
        if (++c_kst == n_iters) {
          c_kst = 0;
          ++c_lt;
          c_y = lane == 0 ? tile_m0(c_lt) : tile_n0(c_lt);
        }
      };
      uint32_t dst[S], bar[S];
      int xs[S], ys[S];
#pragma unroll
      for (int j = 0; j < S; ++j) {
        dst[j] = smem_u32(smem + j * B::STAGE_BYTES + dst_off);
        bar[j] = smem_u32(&full_raw[j]);
        xs[j] = c_kst * x_step;
        ys[j] = c_y;
        advance();
      }
      // The cursor now stands at stage S; it must stand at stage HALF (the stage
      // whose coordinates the first iteration rewrites).
      c_kst = 0;
      c_lt = 0;
      c_y = lane == 0 ? tile_m0(0) : tile_n0(0);
#pragma unroll 1
      for (int h = 0; h < HALF; ++h) advance();
      uint32_t ph = 0;
      bool ok = true;
      for (int it0 = 0; it0 < total && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          if (it0 + j >= total) break;
          bool w_ok = true;
          if (lane == 0) {
            w_ok = mbar_wait(&empty_bar[j], ph ^ 1, kSiteProducer);
            if (w_ok) mbar_arrive_expect_tx(&full_raw[j], B::TX_BYTES);
          }
          if (!__shfl_sync(0x3u, w_ok, 0)) {
            ok = false;
            break;
          }
          // Slot (j + HALF) % S takes stage it0 + j + HALF (the cursor): before this
          // copy when that slot comes later in the ring, after it when it came earlier.
          if (j + HALF < S) {
            xs[j + HALF] = c_kst * x_step;
            ys[j + HALF] = c_y;
          }
          tma_load_2d_u32(dst[j], map, xs[j], ys[j], bar[j]);
          ++issued;
          if (j >= HALF) {
            xs[j - HALF] = c_kst * x_step;
            ys[j - HALF] = c_y;
          }
          advance();
        }
        ph ^= 1;
      }
    }
    // Never leave the CTA with bulk copies still landing in shared memory.
    if (lane == 0) {
      for (int it = issued > S ? issued - S : 0; it < issued; ++it)
        mbar_wait(&full_raw[it % S], (it / S) & 1, kSiteDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(B::BM, BN);
      const uint64_t desc_a0 = smem_desc_sw128(smem_u32(smem));
      const uint64_t desc_w0 = smem_desc_sw128(smem_u32(smem) + B::OP_A_BYTES);
      constexpr uint64_t kStageStep = (uint64_t)(B::STAGE_BYTES >> 4);
      uint64_t da[2][4], dw[2][4];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          da[q][k] = desc_a0 + kStageStep * q + 2 * k;
          dw[q][k] = desc_w0 + kStageStep * q + 2 * k;
        }
      uint32_t ph = 0;
      bool ok = true;
      int kst = 0, lt = 0;  // k-stage and local tile of stage `it` (row-scaled mode)
      for (int it0 = 0; it0 < total && ok; it0 += S) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int it = it0 + j;
          if (it >= total) break;
          const int q = j & 1;
          uint64_t* ready = B::CONVERT ? &full_op[j] : &full_raw[j];
          if (!mbar_wait(ready, ph, kSiteMmaFull)) {
            ok = false;
            break;
          }
          if constexpr (TW) {
            // Tile accumulators alternate; the first stage of a tile waits until the
            // epilogue has read the tile two back from the same buffer.
            const int tb = lt & 1;
            if (kst == 0 && !mbar_wait(&acc_empty[tb], ((lt >> 1) & 1) ^ 1, kSiteMmaAcc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + tb * BN;
            mma_i8(d, da[q][0], dw[q][0], idesc, kst > 0 ? 1u : 0u);
            mma_i8(d, da[q][1], dw[q][1], idesc, 1u);
            mma_i8(d, da[q][2], dw[q][2], idesc, 1u);
            mma_i8(d, da[q][3], dw[q][3], idesc, 1u);
            if (kst == n_iters - 1) mma_commit(&acc_full[tb]);
            if (++kst == n_iters) {
              kst = 0;
              ++lt;
            }
          } else {
            // The accumulator pair runs on across tiles (S is a multiple of NPAIR).
            const int pr = j % B::NPAIR;
            if (!mbar_wait(&acc_empty[pr], ((it / B::NPAIR) & 1) ^ 1, kSiteMmaAcc)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d0 = tmem_base + pr * (2 * BN), d1 = d0 + BN;
            mma_i8(d0, da[q][0], dw[q][0], idesc, 0u);
            mma_i8(d0, da[q][1], dw[q][1], idesc, 1u);
            mma_i8(d1, da[q][2], dw[q][2], idesc, 0u);
            mma_i8(d1, da[q][3], dw[q][3], idesc, 1u);
            mma_commit(&acc_full[pr]);
          }
          mma_commit(&empty_bar[j]);
          const int jn = (j + 1) % S;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            da[q ^ 1][k] = desc_a0 + kStageStep * jn + 2 * k;
            dw[q ^ 1][k] = desc_w0 + kStageStep * jn + 2 * k;
          }
        }
        ph ^= 1;
      }
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0, kSiteMmaDone);
    }
  } else if (warp < B::EPI_WARP0) {
    // ------------------------------------------------------------ converters
    if constexpr (B::CONVERT) {
      const int ctid = threadIdx.x - 64;
      constexpr int NT = 32 * B::CVT_WARPS;
      for (int it = 0; it < total; ++it) {
        const int s = it % S;
        if (!mbar_wait(&full_raw[s], (it / S) & 1, kSiteConverter)) break;
        uint8_t* st = smem + s * B::STAGE_BYTES;
        if constexpr (A < 8) unpack_stage<A, B::BM, NT>(st + B::OP_A_BYTES + B::OP_W_BYTES, st, ctid);
        if constexpr (W < 8)
          unpack_stage<W, BN, NT>(st + B::OP_A_BYTES + B::OP_W_BYTES + B::STG_A_BYTES, st + B::OP_A_BYTES, ctid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_op[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - B::EPI_WARP0;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int e = ew >> 2;   // column slice
    const int row = q * 32 + lane;
    const bool issuer = ew == 0 && lane == 0;
    constexpr int COLS = B::COLS;
    constexpr int P = B::CVT_WARPS > 0 ? (COLS >= 64 ? 8 : COLS >= 16 ? 4 : 2) : (COLS >= 16 ? 4 : 2);
    constexpr int H = COLS / P;
    const float shift_scale = 1.0f / float(1 << B::SHIFT);
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + e * COLS;
    uint32_t ra[H], rb[H];
    float2 acc[COLS / 2];
    bool ok = true;
    for (int lt = 0; lt < my_tiles && ok; ++lt) {
      const int m0 = tile_m0(lt), n0 = tile_n0(lt);
      const int m = m0 + row;
      const bool warp_live = (m0 + q * 32) < p.M;
      const int gs = lt * n_iters;  // global stage index of this tile's first stage
#pragma unroll
      for (int j = 0; j < COLS / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      float as_native = 1.f;  // order 1 of the row-scaled mode: as[m] joins ws in the store
      if constexpr (TW) {
        const int tb = lt & 1;
        ok = mbar_wait(&acc_full[tb], (lt >> 1) & 1, kSiteEpilogue);
        if (ok) {
          tc_fence_after();
          const float as_m = m < p.M ? __ldg(p.act_scale + m) : 0.f;
          const float as_acc = p.rowwise_order ? 1.f : as_m;
          as_native = as_m;
#pragma unroll
          for (int part = 0; part < COLS / H; ++part) {
            tmem_ld<H>(lane_base + tb * BN + part * H, ra);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < H / 2; ++j) {
              const float f0 = __int2float_rn((int)ra[2 * j]) * shift_scale;
              const float f1 = __int2float_rn((int)ra[2 * j + 1]) * shift_scale;
              acc[part * (H / 2) + j] = make_float2(f0 * as_acc, f1 * as_acc);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[tb]);
        }
      } else if (!warp_live) {
        // No valid token row in this warp: only keep the accumulator handshake.
        for (int it = 0; it < n_iters; ++it) {
          const int g_it = gs + it, pr = g_it % B::NPAIR;
          if (!mbar_wait(&acc_full[pr], (g_it / B::NPAIR) & 1, kSiteEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[pr]);
        }
      } else {
        const float* as_row = p.act_scale + (int64_t)(m < p.M ? m : 0) * G;
        const bool load_scales = m < p.M;
        auto scale_at = [&](int g) -> float { return (load_scales && g < G) ? __ldg(as_row + g) : 0.f; };
        {
          const int pr0 = gs % B::NPAIR;
          ok = mbar_wait(&acc_full[pr0], (gs / B::NPAIR) & 1, kSiteEpilogue);
          if (ok) {
            tc_fence_after();
            tmem_ld<H>(lane_base + pr0 * (2 * BN), ra);
            tmem_wait_ld();
          }
        }
        // One stage, as in the one-tile kernel: ra holds part 0 of group 2it; the
        // parts are read into ra / rb alternately, each load overlapping the
        // accumulation of the part before it; part 0 of the next stage of this
        // tile is loaded before the last part is accumulated.
        auto stage = [&](int it, float s0raw, float s1raw) {
          const int g_it = gs + it, pr = g_it % B::NPAIR;
          const uint32_t base = lane_base + pr * (2 * BN);
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
                const int pn = (g_it + 1) % B::NPAIR;
                if (!mbar_wait(&acc_full[pn], ((g_it + 1) / B::NPAIR) & 1, kSiteEpilogue)) {
                  ok = false;
                } else {
                  tc_fence_after();
                  tmem_ld<H>(lane_base + pn * (2 * BN), nxt);
                }
              }
            }
            accumulate<H>(acc + part * (H / 2), cur, grp ? s1 : s0);
            tmem_wait_ld();
          };
#pragma unroll
          for (int idx = 0; idx < 2 * P; idx += 2) {
            part_step(idx, ra, rb);
            part_step(idx + 1, rb, ra);
          }
        };
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

      // Final store of the tile: ws / bias in registers, 16-bit values into the
      // swizzled staging tile, one TMA store per 64 columns.  The staging tile is
      // rewritten only after the previous tile's stores have read it.
      // The AND makes `ok` uniform over the epilogue warps, so that all of them take
      // the same barriers and leave the tile loop together after a timed-out wait.
      if (issuer) bulk_wait_group_read_all();
      ok = named_barrier_and(1, 128 * B::EPI_WG, ok);
      if (ok) {
        const bool native = TW && p.rowwise_order;
        const bool bf16 = p.out_dtype == kDtBF16;
#pragma unroll
        for (int c8 = 0; c8 < COLS / 8; ++c8) {
          const int c = e * COLS + c8 * 8;  // column within the tile
          const int n = n0 + c;
          float y[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float2 v2 = acc[c8 * 4 + t / 2];
            const float a = (t & 1) ? v2.y : v2.x;
            y[t] = n + t < p.N ? (native ? finish_native(a, p, n + t, as_native) : finish(a, p, n + t)) : 0.f;
          }
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (bf16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * t], y[2 * t + 1]);
              w[t] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(y[2 * t], y[2 * t + 1]);
              w[t] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          const int box = c / C::OUT_BOX_COLS, chunk = (c % C::OUT_BOX_COLS) / 8;
          uint8_t* dst = out_stage + box * (B::BM * 128) + row * 128 + ((chunk ^ (row & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      named_barrier_sync(1, 128 * B::EPI_WG);
      if (issuer && ok) {
#pragma unroll
        for (int b = 0; b < C::BOXES; ++b)
          if (n0 + b * C::OUT_BOX_COLS < p.N)  // a box wholly past N is not issued
            tma_store_2d(&tm_out, smem_u32(out_stage + b * (B::BM * 128)), (n0 + b * C::OUT_BOX_COLS) * 2, m0);
        bulk_commit_group();
      }
    }
    if (issuer) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace actune
