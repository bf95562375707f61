// Weight-streaming group-64 linear for few tokens (M <= 32): the decode / denoise
// shape, where the work is bound by reading the packed weights from HBM.
//
//   y[m, n] = ws[n] * sum_g ( float(dot_g(m, n)) * as[m, g] )  (+ bias[n])
//
// with the same exact int32 group dots and the same fp32 chain as the tile kernels
// (actune/kernels/grouped.py:80-94, actune/kernels/grouped_native.cu:70-85):
// acc = fma(float(dot_g), as[m, g], acc) for g = 0, 1, ... then fma(acc, ws, bias).
//
// A 128-row tensor-core tile would waste most of its work on 16 tokens and the
// single-thread tcgen05 issue would bound it, so this kernel uses the warp-level
// integer MMA (m16n8k32, s8 x s8 -> s32): each warp owns 8 weight rows and all
// (up to 32) tokens and walks K group by group; a CTA of 4 warps covers 32 rows, so
// N / 32 CTAs stream disjoint weight rows with no reduction across CTAs.
//
// Operands reach shared memory by TMA in 1024-wide K stages through a 3-4 deep ring
// (96-192 KB in flight per CTA, enough to cover HBM latency), as 128-byte-wide boxes
// with the 128-byte swizzle: a stage is [128 B block][row][128 B], 16-byte chunk c of
// row r stored at chunk c ^ (r mod 8), so the lanes of a warp -- 8 rows x 4 lanes,
// each reading its 16 consecutive codes of a 64-wide group -- spread over all banks.
// K is permuted the same way for both operands inside each group (lane t takes codes
// 16t..16t+15), which leaves every dot unchanged.  Sub-byte codes go to the top bits
// of int8 (code * 2^(8-bits)); the power of two is removed exactly from the
// activation scale.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace actune {

template <int W, int A, int MT>
struct GemvCfg {
  static constexpr int ROWS = 32;                 // weight rows per CTA (4 warps x 8)
  static constexpr int TOK = 16 * MT;             // token rows staged per CTA
  static constexpr int KSTG = 1024;               // K per stage (16 groups)
  static constexpr int GPS = KSTG / 64;           // groups per stage
  static constexpr int A_BLK = KSTG * A / 8 / 128;  // 128-byte blocks per token row per stage (= boxes)
  static constexpr int W_BLK = KSTG * W / 8 / 128;  // 128-byte blocks per weight row per stage
  static constexpr int A_BYTES = A_BLK * TOK * 128;
  static constexpr int W_BYTES = W_BLK * ROWS * 128;
  static_assert(A_BLK + W_BLK <= 32, "one box per producer lane");
  static constexpr int STAGE_BYTES = (A_BYTES + W_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGES_FIT = (200 * 1024) / STAGE_BYTES;  // 3 for W8A8 with 32 tokens, else 4
  static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
  static_assert(STAGES >= 2, "ring depth");
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  static constexpr int SHIFT = (8 - A) + (8 - W);
  static constexpr int THREADS = 128;
};

__device__ __forceinline__ void mma_s8_16832(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Sixteen codes at `addr` (2 * BITS packed bytes) as four int8x4 words in K order,
// sub-byte codes placed in the top bits of each int8.
template <int BITS>
__device__ __forceinline__ uint4 load_codes16_at(const uint8_t* addr) {
  if constexpr (BITS == 8) {
    return *reinterpret_cast<const uint4*>(addr);
  } else if constexpr (BITS == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(addr);
    const uint2 lo = unpack_w4_word(v.x), hi = unpack_w4_word(v.y);
    return make_uint4(lo.x, lo.y, hi.x, hi.y);
  } else {
    return unpack_w2_word(*reinterpret_cast<const uint32_t*>(addr));
  }
}

// Sixteen codes (lane t's part of 64-wide group g) of row r of a staged operand as
// four int8x4 words in K order.  `rows` is the row count of one box; the stage holds
// [block][row][128 B] with the 128-byte swizzle.
template <int BITS>
__device__ __forceinline__ uint4 load_codes16(const uint8_t* tile, int rows, int r, int g, int t) {
  const int off = g * 8 * BITS + t * 2 * BITS;  // byte offset of the lane's codes within the stage row
  const int blk = off >> 7, c = (off >> 4) & 7, sub = off & 15;
  return load_codes16_at<BITS>(tile + (blk * rows + r) * 128 + ((c ^ (r & 7)) << 4) + sub);
}

// Exact int32 -> fp32 for |v| < 2^22 at full rate (see kMagicBits).
__device__ __forceinline__ float exact_float(int32_t v) {
  return __uint_as_float((uint32_t)v + kMagicBits) - kMagicValue;
}

enum : int { kGvSiteProducer = 31, kGvSiteFull, kGvSiteDrain };

template <int W, int A, int MT, bool DOTS>
__global__ void __launch_bounds__(128) gemv_group64_kernel(const __grid_constant__ CUtensorMap tm_act,
                                                            const __grid_constant__ CUtensorMap tm_wgt,
                                                            const GemmParams p) {
  using C = GemvCfg<W, A, MT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  // Activation scales of a stage, [group][token], times 2^-SHIFT; double-buffered
  // and filled one stage ahead so no group waits on a global load.
  __shared__ float sc_smem[2][C::GPS][C::TOK];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t = lane & 3;
  const int G = p.G;
  const int n_stages = (G + C::GPS - 1) / C::GPS;
  const int n0 = blockIdx.x * C::ROWS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 4);
    }
    fence_barrier_init();
  }
  // Dependent launch: everything below reads the previous kernel's outputs.
  griddep_enter();
  __syncthreads();

  // Producer: lanes 0 .. A_BLK-1 of warp 0 load the token boxes of a stage and the
  // next W_BLK lanes its weight boxes, all in one instruction, S stages ahead.
  constexpr int NBOX = C::A_BLK + C::W_BLK;
  constexpr uint32_t PMASK = (NBOX >= 32) ? 0xffffffffu : ((1u << NBOX) - 1u);
  auto issue = [&](int st) {
    const int s = st % C::STAGES;
    if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], C::A_BYTES + C::W_BYTES);
    __syncwarp(PMASK);
    uint8_t* base = smem + s * C::STAGE_BYTES;
    if (lane < C::A_BLK)
      tma_load_2d(base + lane * C::TOK * 128, &tm_act, (st * C::A_BLK + lane) * 128, 0, &full_bar[s]);
    else
      tma_load_2d(base + C::A_BYTES + (lane - C::A_BLK) * C::ROWS * 128, &tm_wgt,
                  (st * C::W_BLK + lane - C::A_BLK) * 128, n0, &full_bar[s]);
  };
  int issued = 0;
  if (warp == 0 && lane < NBOX) {
    if (lane < 2) prefetch_tensormap(lane == 0 ? &tm_act : &tm_wgt);
    for (int st = 0; st < n_stages && st < C::STAGES; ++st) {
      issue(st);
      ++issued;
    }
  }

  const int row = warp * 8 + gid;  // weight row (within the CTA) this lane's B operand comes from
  const float shift_scale = 1.0f / float(1 << C::SHIFT);
  // Accumulators: tile mt, {token gid, rows 2t, 2t+1}, {token gid + 8, rows 2t, 2t+1}.
  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
  // Cooperative scale staging: thread i covers entries i, i + 128, ... of the
  // [GPS][TOK] block of a stage.
  constexpr int SC_PER_THREAD = (C::GPS * C::TOK + 127) / 128;
  auto load_scales = [&](int st, float (&v)[SC_PER_THREAD]) {
#pragma unroll
    for (int j = 0; j < SC_PER_THREAD; ++j) {
      const int e = threadIdx.x + 128 * j;
      const int gl = e / C::TOK, m = e % C::TOK;
      const int g = st * C::GPS + gl;
      v[j] = (!DOTS && e < C::GPS * C::TOK && m < p.M && g < G) ? __ldg(p.act_scale + (int64_t)m * G + g) * shift_scale
                                                                 : 0.f;
    }
  };
  auto store_scales = [&](int buf, const float (&v)[SC_PER_THREAD]) {
#pragma unroll
    for (int j = 0; j < SC_PER_THREAD; ++j) {
      const int e = threadIdx.x + 128 * j;
      if (e < C::GPS * C::TOK) (&sc_smem[buf][0][0])[e] = v[j];
    }
  };
  float sc_next[SC_PER_THREAD];
  load_scales(0, sc_next);
  store_scales(0, sc_next);
  if (n_stages > 1) load_scales(1, sc_next);
  __syncthreads();

  bool ok = true;
  for (int st = 0; st < n_stages; ++st) {
    const int s = st % C::STAGES;
    // A failed wait only marks the CTA for exit; every thread still reaches the
    // end-of-stage barrier below, so the exit is CTA-uniform and no barrier waits
    // for a warp that has left.
    if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[s], (st / C::STAGES) & 1, kGvSiteFull))) ok = false;
    const uint8_t* a_tile = smem + s * C::STAGE_BYTES;
    const uint8_t* w_tile = a_tile + C::A_BYTES;
    // All 16 groups of a stage, unrolled: the shared-memory offsets become
    // constants and independent groups overlap.  Groups past the end of K are the
    // TMA's zero fill with scale 0 (acc += 0 * 0 leaves every accumulator as it is;
    // an accumulator is never -0), so only the dots export has to skip them.
#pragma unroll
    for (int gl = 0; gl < C::GPS; ++gl) {
      const int g = st * C::GPS + gl;
      if (!ok) break;
      float sc[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) sc[mt][h] = sc_smem[st & 1][gl][mt * 16 + h * 8 + gid];
      const uint4 wq = load_codes16<W>(w_tile, C::ROWS, row, gl, t);
      int32_t d[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 a_lo = load_codes16<A>(a_tile, C::TOK, mt * 16 + gid, gl, t);
        const uint4 a_hi = load_codes16<A>(a_tile, C::TOK, mt * 16 + gid + 8, gl, t);
        d[mt][0] = d[mt][1] = d[mt][2] = d[mt][3] = 0;
        // K permutation inside the group: MMA chunk 0 takes codes 16t+0..7, chunk 1
        // codes 16t+8..15 of this lane (both operands identically).
        const uint32_t a0[4] = {a_lo.x, a_hi.x, a_lo.y, a_hi.y};
        mma_s8_16832(d[mt], a0, wq.x, wq.y);
        const uint32_t a1[4] = {a_lo.z, a_hi.z, a_lo.w, a_hi.w};
        mma_s8_16832(d[mt], a1, wq.z, wq.w);
      }
      if constexpr (DOTS) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = mt * 16 + (i >> 1) * 8 + gid;
            const int n = n0 + warp * 8 + 2 * t + (i & 1);
            if (m < p.M && n < p.N && g < G) p.dots[((int64_t)m * p.N + n) * G + g] = d[mt][i] >> C::SHIFT;
          }
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            acc[mt][i] = fmaf(__int2float_rn(d[mt][i]), sc[mt][i >> 1], acc[mt][i]);
      }
    }
    // Publish the next stage's scales (its buffer was last read in stage st - 1,
    // before the previous barrier) and fetch the ones after it.
    if (st + 1 < n_stages) store_scales((st + 1) & 1, sc_next);
    if (st + 2 < n_stages) load_scales(st + 2, sc_next);
    // Release the stage; warp 0's producer lanes refill it once all 4 warps are done.
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
    if (ok && warp == 0 && lane < NBOX && st + C::STAGES < n_stages) {
      bool w_ok = true;
      if (lane == 0) w_ok = mbar_wait(&empty_bar[s], (st / C::STAGES) & 1, kGvSiteProducer);
      if (__shfl_sync(PMASK, w_ok, 0)) {
        issue(st + C::STAGES);
        ++issued;
      } else {
        ok = false;
      }
    }
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
  }
  // Never leave the CTA with bulk copies still landing in shared memory.
  // (Only the last STAGES issued copies can still be pending; an older barrier
  // phase cannot be waited for any more once its slot has been reused.)
  if (warp == 0 && lane == 0) {
    for (int st = issued > C::STAGES ? issued - C::STAGES : 0; st < issued; ++st)
      mbar_wait(&full_bar[st % C::STAGES], (st / C::STAGES) & 1, kGvSiteDrain);
  }

  if constexpr (!DOTS) {
    if (ok) {
#pragma unroll
      for (int i2 = 0; i2 < 2; ++i2) {
        const int n = n0 + warp * 8 + 2 * t + i2;
        if (n >= p.N) continue;
        const float ws = __ldg(p.w_scale + n);
        const bool has_bias = p.bias_dtype != kDtNone;
        const float bias = has_bias ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int m = mt * 16 + h * 8 + gid;
            if (m >= p.M) continue;
            const float a = acc[mt][h * 2 + i2];
            store_scalar(p, (int64_t)m * p.N + n, has_bias ? fmaf(a, ws, bias) : a * ws);
          }
      }
    }
  }
}

// Byte offset, within a stage tile of box_rows-high 128-byte lines laid out
// [block][row] with the 128-byte swizzle, of lane t's 16 codes of group gl in row r.
template <int BITS>
__device__ __forceinline__ uint32_t swizzled_offset(int gl, int t, int r, int box_rows) {
  const int off = gl * 8 * BITS + t * 2 * BITS;
  const int blk = off >> 7, c = (off >> 4) & 7, sub = off & 15;
  const int line = blk * box_rows + r;
  return (uint32_t)(line * 128 + ((c ^ (line & 7)) << 4) + sub);
}

// ---------------------------------------------------------------------------
// Up to 16 tokens, packed rows a multiple of 128 bytes: separate producer, dot and
// chain roles, persistent over row blocks.
//
// A CTA streams 32-row weight blocks (blockIdx.x, blockIdx.x + gridDim.x, ...)
// through one TMA ring.  A stage is K=1024 and three boxes: the weight tile and the
// token tile as 3-D boxes over (128-byte block, row, block index) views, landing as
// [block][row][128 B] with the 128-byte swizzle, and the stage's activation scales
// [M][16] fp32.  The TMA unit spends a roughly fixed time per box, so a few large
// boxes keep the ring full where many small ones starve it; token boxes are exactly
// M rows high because zero-filled box rows cost as much as loaded ones.
// One producer warp only issues copies.  16 dot warps = 2 row groups (16 weight
// rows, two 8-row MMA column blocks sharing each token fragment) x 8 K-lanes
// (K-lane q taking groups 2q, 2q+1 of every stage) turn a stage into exact fp32
// dots and write them to a ring of dot buffers in shared memory; they never wait
// for the fp32 chain except for a free dot buffer.  4 chain warps (one per 8 weight
// rows) fold the dots into the chain in K order, fma(dot, scale, acc) group by
// group, reading the scales from the stage slot, and write the outputs at the end
// of a row block.  With at most 8 tokens only the real half of each dot fragment
// is stored and read, and fragment rows past the last token are neither loaded,
// stored nor read back (at M = 1 a stage's shared-memory traffic drops from ~162 KB
// to ~78 KB; measured 1-5 % faster, so shared-memory bandwidth is not what sets
// the pace of the dot warps).
// A stage slot is free once the 16 dot warps and the 4 chain warps released it.
template <int W, int A, bool HI, bool WIDE = false>
struct Gemv4Cfg {
  static_assert(!WIDE || (!HI && W <= 4), "wide stages: at most 8 tokens, 2- or 4-bit weights");
  static constexpr int ROWS = 32, TOK = HI ? 16 : 8, KSTG = WIDE ? kGemvStageKWide : kGemvStageK;
  static constexpr int GPS = KSTG / 64, QL = 8, GPQ = GPS / QL;
  static constexpr int DOT_WARPS = 16, CHAIN_WARPS = 4, PRODUCER = DOT_WARPS + CHAIN_WARPS;
  static constexpr int THREADS = 32 * (PRODUCER + 1);
  static constexpr int A_BLK = KSTG * A / 8 / 128;
  static constexpr int W_BLK = KSTG * W / 8 / 128;
  static constexpr int W_BYTES = W_BLK * ROWS * 128;  // multiple of 4096
  static constexpr int A_BYTES = A_BLK * TOK * 128;   // multiple of 1024
  static constexpr int SC_BYTES = TOK * GPS * 4;
  static constexpr int STAGE_BYTES = (W_BYTES + A_BYTES + SC_BYTES + 1023) / 1024 * 1024;
  // Dot buffers: [8-row block (4)][group of the stage][lane] of the lane's d0..d3
  // (float4), or d0, d1 only (float2) when there are at most 8 tokens; plus a copy
  // of the stage's activation scales per 16-row group.
  static constexpr int DOT_LANE_BYTES = HI ? 16 : 8;
  static constexpr int DOT_BYTES = 4 * GPS * 32 * DOT_LANE_BYTES;
  static constexpr int DSC_BYTES = 2 * SC_BYTES;
  static constexpr int DSTAGES = 2;
  static constexpr int RING_BUDGET = 224 * 1024 - DSTAGES * (DOT_BYTES + DSC_BYTES);  // 227 KB per CTA at most
  static constexpr int STAGES_FIT = RING_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + DSTAGES * (DOT_BYTES + DSC_BYTES) + 1024;
  static constexpr int SHIFT = (8 - A) + (8 - W);
  static_assert(STAGES >= 2, "ring depth");
};

enum : int { kGv4SiteFull = 61, kGv4SiteEmpty, kGv4SiteDotFull, kGv4SiteDotEmpty, kGv4SiteDrain };

// TW (tokenwise backends): no per-group scales; the dot buffers carry the raw int32
// dots, the chain warps add them exactly and apply float(acc) * as[m] * ws (+ bias)
// once per row block (as: one scale per token).
template <int W, int A, bool HI, bool DOTS, bool TW = false, bool WIDE = false>
__global__ void __launch_bounds__(Gemv4Cfg<W, A, HI, WIDE>::THREADS, 1)
    gemv4_group64_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_wgt,
                         const __grid_constant__ CUtensorMap tm_scale, const GemmParams p) {
  using C = Gemv4Cfg<W, A, HI, WIDE>;
  using DotT = typename std::conditional<HI, float4, float2>::type;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t dot_full[C::DSTAGES][2];
  __shared__ __align__(8) uint64_t dot_empty[C::DSTAGES][2];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DotT* dots_smem = reinterpret_cast<DotT*>(smem + C::STAGES * C::STAGE_BYTES);
  float* dsc_smem = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + C::DSTAGES * C::DOT_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, Mb = p.M;  // token boxes are M rows high (M <= TOK)
  const int n_stages = (G + C::GPS - 1) / C::GPS;
  const int n_blocks = (p.N + C::ROWS - 1) / C::ROWS;
  const int my_blocks = (int)blockIdx.x < n_blocks ? (n_blocks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_blocks * n_stages;
  // The next kernel (a dependent launch) may start as SMs come free; it waits for
  // this one before reading what it writes.
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], C::DOT_WARPS);
    }
    for (int d = 0; d < C::DSTAGES; ++d)
      for (int r = 0; r < 2; ++r) {
        mbar_init(&dot_full[d][r], C::QL);
        mbar_init(&dot_empty[d][r], 2);
      }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == C::PRODUCER) {
    // ------------------------------------------------------------ producer
    // Lanes 0 (weights), 1 (tokens) and 2 (scales) issue a stage's three boxes in
    // one instruction.  When the packed rows are not whole 128-byte blocks the
    // maps are 2-D and every 128-byte block is a box of its own: lanes
    // 0..W_BLK-1 the weight blocks, the next A_BLK lanes the token blocks (TOK rows
    // high, so that the swizzle phase of a line is its row), then the scales; the
    // part of a block past the row end is the TMA's zero fill.
    const bool b2d = p.gemv_boxes2d != 0;
    const int lanes = b2d ? C::W_BLK + C::A_BLK + 1 : 3;
    static_assert(C::W_BLK + C::A_BLK + 1 <= 32, "one lane per block");
    if (lane < lanes) {
      const int kind = b2d ? (lane < C::W_BLK ? 0 : lane < C::W_BLK + C::A_BLK ? 1 : 2) : lane;
      const int blk = b2d ? (kind == 0 ? lane : lane - C::W_BLK) : 0;
      if (blk == 0) prefetch_tensormap(kind == 0 ? &tm_wgt : kind == 1 ? &tm_act : &tm_scale);
      const uint32_t mask = lanes == 32 ? 0xffffffffu : ((1u << lanes) - 1u);
      const uint32_t stage_tx = C::W_BYTES + (b2d ? C::A_BLK * C::TOK * 128 : Mb * C::A_BLK * 128) +
                                ((DOTS || TW) ? 0 : Mb * C::GPS * 4);
      // Dependent launch: the weight boxes of the first ring pass are requested before
      // waiting for the previous kernel (they do not depend on it); tokens and scales after.
      auto weight_box = [&](int it) {
        const int s = it % C::STAGES;
        const int rb = (int)blockIdx.x + (it / n_stages) * (int)gridDim.x, st = it % n_stages;
        uint8_t* base = smem + s * C::STAGE_BYTES;
        if (b2d) tma_load_2d(base + blk * (C::ROWS * 128), &tm_wgt, (st * C::W_BLK + blk) * 128, rb * C::ROWS, &full_bar[s]);
        else tma_load_3d(base, &tm_wgt, 0, rb * C::ROWS, st * C::W_BLK, &full_bar[s]);
      };
      const int pre = p.pdl_wait ? min(C::STAGES, total) : 0;
      if (pre > 0) {
        if (lane == 0)
          for (int it = 0; it < pre; ++it) mbar_arrive_expect_tx(&full_bar[it], stage_tx);
        __syncwarp(mask);
        if (kind == 0)
          for (int it = 0; it < pre; ++it) weight_box(it);
        griddep_wait();
      }
      int issued = 0;
      for (int it = 0; it < total; ++it) {
        const int s = it % C::STAGES;
        const bool prefetched = it < pre;
        bool ok = true;
        if (lane == 0 && !prefetched) {
          if (it >= C::STAGES) ok = mbar_wait(&empty_bar[s], ((it / C::STAGES) & 1) ^ 1, kGv4SiteEmpty);
          if (ok) mbar_arrive_expect_tx(&full_bar[s], stage_tx);
        }
        if (!__shfl_sync(mask, ok, 0)) break;
        const int st = it % n_stages;
        uint8_t* base = smem + s * C::STAGE_BYTES;
        if (kind == 0) {
          if (!prefetched) weight_box(it);
        } else if (b2d) {
          if (kind == 1)
            tma_load_2d(base + C::W_BYTES + blk * (C::TOK * 128), &tm_act, (st * C::A_BLK + blk) * 128, 0,
                        &full_bar[s]);
          else if (!DOTS && !TW)
            tma_load_2d(base + C::W_BYTES + C::A_BYTES, &tm_scale, st * C::GPS, 0, &full_bar[s]);
        } else {
          if (lane == 1) tma_load_3d(base + C::W_BYTES, &tm_act, 0, 0, st * C::A_BLK, &full_bar[s]);
          else if (!DOTS && !TW) tma_load_2d(base + C::W_BYTES + C::A_BYTES, &tm_scale, st * C::GPS, 0, &full_bar[s]);
        }
        ++issued;
      }
      // Never leave the CTA with bulk copies still landing in shared memory.
      if (lane == 0) {
        for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it)
          mbar_wait(&full_bar[it % C::STAGES], (it / C::STAGES) & 1, kGv4SiteDrain);
      }
    }
  } else if (warp < C::DOT_WARPS) {
    // ------------------------------------------------------------ dots
    if (DOTS && p.pdl_wait) griddep_wait();  // the dots export writes global memory
    const int r = warp & 1, q = warp >> 1;  // 16-row group, K-lane
    const int gid = lane >> 2, t = lane & 3;
    uint32_t ow0[C::GPQ], ow1[C::GPQ], oa_lo[C::GPQ], oa_hi[C::GPQ];
#pragma unroll
    for (int j = 0; j < C::GPQ; ++j) {
      ow0[j] = swizzled_offset<W>(q * C::GPQ + j, t, r * 16 + gid, C::ROWS);
      ow1[j] = swizzled_offset<W>(q * C::GPQ + j, t, r * 16 + 8 + gid, C::ROWS);
      const int a_box_rows = p.gemv_boxes2d ? C::TOK : Mb;  // token box height
      oa_lo[j] = swizzled_offset<A>(q * C::GPQ + j, t, gid, a_box_rows);
      oa_hi[j] = swizzled_offset<A>(q * C::GPQ + j, t, gid + 8, a_box_rows);
    }
    for (int it = 0; it < total; ++it) {
      const int s = it % C::STAGES, d = it % C::DSTAGES;
      if (!mbar_wait(&full_bar[s], (it / C::STAGES) & 1, kGv4SiteFull)) break;
      if constexpr (!DOTS) {
        if (it >= C::DSTAGES && !mbar_wait(&dot_empty[d][r], ((it / C::DSTAGES) & 1) ^ 1, kGv4SiteDotEmpty)) break;
      }
      const int rb = (int)blockIdx.x + (it / n_stages) * (int)gridDim.x, st = it % n_stages;
      const uint8_t* w_tile = smem + s * C::STAGE_BYTES;
      const uint8_t* a_tile = w_tile + C::W_BYTES;
      if constexpr (!DOTS && !TW) {
        // K-lane 0 copies the stage's scales for its row group's chain warps, so that
        // the stage slot is free once the dots are written.
        if (q == 0) {
          const float4* src = reinterpret_cast<const float4*>(a_tile + C::A_BYTES);
          float4* dst = reinterpret_cast<float4*>(dsc_smem + (d * 2 + r) * (C::TOK * C::GPS));
          for (int i = lane; i < Mb * C::GPS / 4; i += 32) dst[i] = src[i];
        }
      }
#pragma unroll
      for (int j = 0; j < C::GPQ; ++j) {
        // Fragment rows past the last token feed only dots that are never stored:
        // they are not read (zero), which spares the shared-memory bandwidth.
        uint4 a_lo = make_uint4(0, 0, 0, 0), a_hi = make_uint4(0, 0, 0, 0);
        if (gid < Mb) a_lo = load_codes16_at<A>(a_tile + oa_lo[j]);
        if constexpr (HI)
          if (gid + 8 < Mb) a_hi = load_codes16_at<A>(a_tile + oa_hi[j]);
        const uint32_t a0[4] = {a_lo.x, a_hi.x, a_lo.y, a_hi.y};
        const uint32_t a1[4] = {a_lo.z, a_hi.z, a_lo.w, a_hi.w};
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const uint4 wq = load_codes16_at<W>(w_tile + (b ? ow1[j] : ow0[j]));
          int32_t dd[4] = {0, 0, 0, 0};
          mma_s8_16832(dd, a0, wq.x, wq.y);
          mma_s8_16832(dd, a1, wq.z, wq.w);
          const int blk8 = r * 2 + b;  // 8-row block of the 32-row tile
          if constexpr (DOTS) {
            const int g = st * C::GPS + q * C::GPQ + j;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = (i >> 1) * 8 + gid;
              const int n = rb * C::ROWS + blk8 * 8 + 2 * t + (i & 1);
              if (m < p.M && n < p.N && g < G) p.dots[((int64_t)m * p.N + n) * G + g] = dd[i] >> C::SHIFT;
            }
          } else if (gid >= Mb) {
            // No token in this lane's fragment rows: nothing for the chain to read.
          } else if constexpr (TW) {
            // Raw int32 dots (bit patterns in the float slots).
            DotT* dst = dots_smem + ((d * 4 + blk8) * C::GPS + q * C::GPQ + j) * 32 + lane;
            if constexpr (HI)
              *dst = make_float4(__int_as_float(dd[0]), __int_as_float(dd[1]), __int_as_float(dd[2]),
                                 __int_as_float(dd[3]));
            else
              *dst = make_float2(__int_as_float(dd[0]), __int_as_float(dd[1]));
          } else {
            DotT* dst = dots_smem + ((d * 4 + blk8) * C::GPS + q * C::GPQ + j) * 32 + lane;
            if constexpr (HI)
              *dst = make_float4(exact_float(dd[0]), exact_float(dd[1]), exact_float(dd[2]), exact_float(dd[3]));
            else
              *dst = make_float2(exact_float(dd[0]), exact_float(dd[1]));
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        if constexpr (!DOTS) mbar_arrive(&dot_full[d][r]);
        mbar_arrive(&empty_bar[s]);
      }
    }
  } else if constexpr (!DOTS) {
    // ------------------------------------------------------------ chain
    if (p.pdl_wait) griddep_wait();  // activation scales and the output may belong to the previous kernel
    const int blk8 = warp - C::DOT_WARPS, r = blk8 >> 1;  // 8-row block, its 16-row group
    const int gid = lane >> 2, t = lane & 3;
    const bool tok0 = gid < Mb, tok1 = HI && gid + 8 < Mb;
    const bool has_bias = p.bias_dtype != kDtNone;
    const float shift_scale = 1.0f / float(1 << C::SHIFT);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int32_t iacc[4] = {0, 0, 0, 0};
    // Tokenwise: one activation scale per token.
    const float as0 = (TW && tok0) ? __ldg(p.act_scale + gid) : 0.f;
    const float as1 = (TW && tok1) ? __ldg(p.act_scale + gid + 8) : 0.f;
    float ws_pre[2] = {0.f, 0.f}, bias_pre[2] = {0.f, 0.f};
    for (int it = 0; it < total; ++it) {
      const int d = it % C::DSTAGES;
      const int rb = (int)blockIdx.x + (it / n_stages) * (int)gridDim.x, st = it % n_stages;
      if (st == 0) {
        // Weight scales and bias of this row block, loaded early.
#pragma unroll
        for (int i2 = 0; i2 < 2; ++i2) {
          const int n = rb * C::ROWS + blk8 * 8 + 2 * t + i2;
          ws_pre[i2] = n < p.N ? __ldg(p.w_scale + n) : 0.f;
          bias_pre[i2] = (has_bias && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
        }
        acc = make_float4(0.f, 0.f, 0.f, 0.f);
        iacc[0] = iacc[1] = iacc[2] = iacc[3] = 0;
      }
      if (!mbar_wait(&dot_full[d][r], (it / C::DSTAGES) & 1, kGv4SiteDotFull)) break;
      if constexpr (TW) {
        const DotT* dslot = dots_smem + ((d * 4 + blk8) * C::GPS) * 32 + lane;
#pragma unroll
        for (int g = 0; g < C::GPS; ++g) {
          // Lanes without a token read nothing (their sums are never stored).
          const DotT dv = tok0 ? dslot[g * 32] : DotT{};
          iacc[0] += __float_as_int(dv.x);
          iacc[1] += __float_as_int(dv.y);
          if constexpr (HI) {
            iacc[2] += __float_as_int(dv.z);
            iacc[3] += __float_as_int(dv.w);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&dot_empty[d][r]);
        if (st == n_stages - 1) {
          // float(acc) exactly rounded; the 2^-SHIFT of top-bit codes is exact.  Order 0:
          // y = (f * as) * ws (+ bias, fused); order 1: y = f * (as * ws) (+ bias, fused).
          const float f00 = __int2float_rn(iacc[0]) * shift_scale, f01 = __int2float_rn(iacc[1]) * shift_scale;
          const float f10 = __int2float_rn(iacc[2]) * shift_scale, f11 = __int2float_rn(iacc[3]) * shift_scale;
          const bool native = p.rowwise_order != 0;
#pragma unroll
          for (int i2 = 0; i2 < 2; ++i2) {
            const int n = rb * C::ROWS + blk8 * 8 + 2 * t + i2;
            if (n >= p.N) continue;
            const float ws = ws_pre[i2], bias = bias_pre[i2];
            const float f0 = i2 ? f01 : f00, f1 = i2 ? f11 : f10;
            const float m0 = native ? f0 : f0 * as0, s0 = native ? as0 * ws : ws;
            const float m1 = native ? f1 : f1 * as1, s1 = native ? as1 * ws : ws;
            if (tok0) store_scalar(p, (int64_t)gid * p.N + n, has_bias ? fmaf(m0, s0, bias) : m0 * s0);
            if (tok1) store_scalar(p, (int64_t)(gid + 8) * p.N + n, has_bias ? fmaf(m1, s1, bias) : m1 * s1);
          }
        }
        continue;
      }
      const float* sc = dsc_smem + (d * 2 + r) * (C::TOK * C::GPS);
      const DotT* dslot = dots_smem + ((d * 4 + blk8) * C::GPS) * 32 + lane;
      // Groups past the end of K have dot 0 and scale 0 (zero fill): acc += 0 * 0.
#pragma unroll
      for (int g = 0; g < C::GPS; ++g) {
        // Lanes without a token read no dots (their accumulators are never stored).
        const DotT dv = tok0 ? dslot[g * 32] : DotT{};
        const float s0 = tok0 ? sc[gid * C::GPS + g] * shift_scale : 0.f;
        acc.x = fmaf(dv.x, s0, acc.x);
        acc.y = fmaf(dv.y, s0, acc.y);
        if constexpr (HI) {
          const float s1 = tok1 ? sc[(gid + 8) * C::GPS + g] * shift_scale : 0.f;
          acc.z = fmaf(dv.z, s1, acc.z);
          acc.w = fmaf(dv.w, s1, acc.w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dot_empty[d][r]);
      if (st == n_stages - 1) {
#pragma unroll
        for (int i2 = 0; i2 < 2; ++i2) {
          const int n = rb * C::ROWS + blk8 * 8 + 2 * t + i2;
          if (n >= p.N) continue;
          const float ws = ws_pre[i2], bias = bias_pre[i2];
          const float a0v = i2 ? acc.y : acc.x, a1v = i2 ? acc.w : acc.z;
          if (tok0) store_scalar(p, (int64_t)gid * p.N + n, has_bias ? fmaf(a0v, ws, bias) : a0v * ws);
          if (tok1) store_scalar(p, (int64_t)(gid + 8) * p.N + n, has_bias ? fmaf(a1v, ws, bias) : a1v * ws);
        }
      }
    }
  }
}

template <int W, int A, bool HI, bool TW = false, bool WIDE = false>
static cudaError_t launch_gemv4_hi(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& ts,
                                   const GemmParams& p, int num_sms, cudaStream_t stream) {
  using C = Gemv4Cfg<W, A, HI, WIDE>;
  const bool dots = !TW && p.dots != nullptr;
  void (*kernel)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmParams);
  cudaError_t e;
  if constexpr (WIDE) {
    if (dots) return cudaErrorInvalidValue;  // the dots export runs 1024-K stages
    constexpr auto k = gemv4_group64_kernel<W, A, HI, false, TW, true>;
    kernel = k;
    e = ensure_smem_limit<k>(C::SMEM_BYTES);
  } else if constexpr (TW) {
    constexpr auto k = gemv4_group64_kernel<W, A, HI, false, TW>;
    kernel = k;
    e = ensure_smem_limit<k>(C::SMEM_BYTES);
  } else {
    constexpr auto k_dots = gemv4_group64_kernel<W, A, HI, true>;
    constexpr auto k_out = gemv4_group64_kernel<W, A, HI, false>;
    kernel = dots ? k_dots : k_out;
    e = dots ? ensure_smem_limit<k_dots>(C::SMEM_BYTES) : ensure_smem_limit<k_out>(C::SMEM_BYTES);
  }
  if (e != cudaSuccess) return e;
  const int blocks = (p.N + C::ROWS - 1) / C::ROWS;
  const int grid = blocks < num_sms ? blocks : num_sms;
  GemmParams pp = p;
  pp.pdl_wait = 1;
  return launch_pdl(kernel, dim3(grid), C::THREADS, C::SMEM_BYTES, stream, ta, tw, ts, pp);
}

template <int W, int A>
static cudaError_t launch_gemv4_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& ts,
                                  const GemmParams& p, int num_sms, cudaStream_t stream) {
  if (p.M > 8) return launch_gemv4_hi<W, A, true>(ta, tw, ts, p, num_sms, stream);
  if constexpr (W <= 4)
    if (gemv_wide(p.M, W, p.dots != nullptr)) return launch_gemv4_hi<W, A, false, false, true>(ta, tw, ts, p, num_sms, stream);
  return launch_gemv4_hi<W, A, false>(ta, tw, ts, p, num_sms, stream);
}

template <int W, int A>
static cudaError_t launch_gemv4_rowwise(const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p, int num_sms,
                                        cudaStream_t stream) {
  if (p.M > 8) return launch_gemv4_hi<W, A, true, true>(ta, tw, ta, p, num_sms, stream);
  if constexpr (W <= 4)
    if (gemv_wide(p.M, W, false)) return launch_gemv4_hi<W, A, false, true, true>(ta, tw, ta, p, num_sms, stream);
  return launch_gemv4_hi<W, A, false, true>(ta, tw, ta, p, num_sms, stream);
}

template <int W, int A, int MT>
static cudaError_t launch_gemv_t(const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                                 cudaStream_t stream) {
  using C = GemvCfg<W, A, MT>;
  const bool dots = p.dots != nullptr;
  constexpr auto k_dots = gemv_group64_kernel<W, A, MT, true>;
  constexpr auto k_out = gemv_group64_kernel<W, A, MT, false>;
  const cudaError_t e = dots ? ensure_smem_limit<k_dots>(C::SMEM_BYTES) : ensure_smem_limit<k_out>(C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  auto kernel = dots ? k_dots : k_out;
  return launch_pdl(kernel, dim3((p.N + C::ROWS - 1) / C::ROWS), C::THREADS, C::SMEM_BYTES, stream, ta, tw, p);
}

cudaError_t launch_gemv_group64(int W, int A, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap* ts,
                                const GemmParams& p, int num_sms, cudaStream_t stream) {
#define ACTUNE_CASE(WW, AA)                                                                                  \
  if (W == WW && A == AA) {                                                                                  \
    if (ts != nullptr)                                                                                       \
      return launch_gemv4_t<WW, AA>(ta, tw, *ts, p, num_sms, stream);                                        \
    return p.M <= 16 ? launch_gemv_t<WW, AA, 1>(ta, tw, p, stream) : launch_gemv_t<WW, AA, 2>(ta, tw, p, stream); \
  }
  ACTUNE_CASE(2, 2) ACTUNE_CASE(2, 4) ACTUNE_CASE(2, 8)
  ACTUNE_CASE(4, 2) ACTUNE_CASE(4, 4) ACTUNE_CASE(4, 8)
  ACTUNE_CASE(8, 2) ACTUNE_CASE(8, 4) ACTUNE_CASE(8, 8)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

// Row-scaled decode (M <= 16; A = 8 tokenwise, A = 4 per-row A4): the same kernel in
// its TW mode.
cudaError_t launch_gemv_tokenwise(int W, int A, const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p,
                                  int num_sms, cudaStream_t stream) {
#define ACTUNE_CASE(WW, AA) \
  if (W == WW && A == AA) return launch_gemv4_rowwise<WW, AA>(ta, tw, p, num_sms, stream);
  ACTUNE_CASE(2, 8) ACTUNE_CASE(4, 8) ACTUNE_CASE(8, 8)
  ACTUNE_CASE(2, 4) ACTUNE_CASE(4, 4) ACTUNE_CASE(8, 4)
#undef ACTUNE_CASE
  return cudaErrorInvalidValue;
}

}  // namespace actune
