// sg_gemv.cu -- decode GEMV (batch 1..16) for Q4_0 / Q4_K on B200 tensor
// cores (tcgen05, accumulators in TMEM).
//
// Replaces the engine's per-token GEMV routes: forward_linear's Q4_0 path
// (swamp-engine/src/linear.rs:68-87: dequant + f32 row dots) and
// fused_gemv_q4k (swamp-kernels/src/fused_gemv_q4k.rs:59-82, scalar order
// :466-508), plus forward_linear_multi (linear.rs:96-170) when several
// tensors share one x.
//
// Arithmetic. Per 32-element block b of row r (Q4_0: w = d*(q-8); Q4_K:
// w = sv*q - mv with sv = d*sc, mv = dmin*m):
//   y[t][r] = sum_b ( sv_b * sum_{k in b} q_k u_k  -  mv_b * sum_{k in b} u_k )
// The tensor core computes the integer part exactly: A holds f16 (1024+q) or
// (1024+16q) (exact, straight from the nibbles), B holds the activation as
// two f16 parts hi + lo per token (x scaled per token by a power of two so
// the parts keep 22 significant bits; the x16 positions carry x/16). Each
// block gets its own f32 accumulator in TMEM; the epilogue subtracts the
// block's constant part (precomputed per token from the same hi + lo values,
// so the 1024 offset cancels exactly) and applies the block scale in f32.
//
// Data movement is built around one measured fact of the copy engine: each
// issuing thread completes bulk copies one after another at a roughly fixed
// cost per copy, so bandwidth comes from large copies. Work is therefore cut
// in units of 4 chunks (128 rows x 256 K) -- 18 KB of packed weights,
// contiguous in the tile layout -- and each unit's weights and activations
// arrive in one bulk copy each.
//
// Kernels, chained with programmatic dependent launch:
//  1. gemv_xprep_kernel: power-of-two scale per token, f16 hi/lo activation
//     parts written directly in the swizzled UMMA operand layout, unit by
//     unit, with each unit's per-block sums appended; zeroing of the output
//     rows that several CTAs reduce into.
//  2. gemv_kernel<dtype, BP>: one CTA per SM, balanced split -- CTA c takes
//     units [c*T/G, (c+1)*T/G) of the T = row-blocks x units space, crossing
//     row-block (and matrix) boundaries; a row-block seen whole is stored, a
//     shared one is reduced with red.add.
//       warp 0      weight producer: one cp.async.bulk per unit into a
//                   4-slot ring (issued before the wait on the previous
//                   kernel: weights do not depend on it).
//       warp 10     activation producer: one cp.async.bulk per unit (4
//                   operand tiles + block sums) into a 3-slot ring.
//       warp 1      TMEM owner; one thread issues tcgen05.mma (A from TMEM,
//                   M=128, N=2*BP: BP hi token rows + BP lo token rows,
//                   K=16, f16 -> f32), two per 32-block, into a ring of TMEM
//                   accumulator slots.
//       warps 2-5   dequant: one weight row per thread, two 16-byte reads
//                   and 8 lop3 + 2 shifts per 64 K, written with one
//                   tcgen05.st into a tensor-memory A tile (lane = row), so
//                   the dequantized operand never passes through shared
//                   memory.
//       warps 6-9   epilogue: per chunk, tcgen05.ld of the two block
//                   accumulators of its TMEM lane quadrant (warp % 4), block
//                   scales in f32, output rows stored or reduced.
// Every mbarrier wait is bounded (sg_common.cuh).
#include <algorithm>

#include "sg_gemv.cuh"
#include "sg_tc.cuh"

namespace gemv_tc {

constexpr int kUC = 4;                     // chunks per unit
constexpr int kRW = 4;                     // weight unit ring
constexpr int kRX = 3;                     // activation unit ring
constexpr int kACols = 32;                 // TMEM columns of one A tile: 128 lanes x 64 K f16
constexpr int kWU = kUC * SG_TILE_BYTES + 512;  // packed weights of a unit + Q4_K d|dmin
constexpr int kThreads = 352;
constexpr int kMaskWords = 32;             // split row-block bitmask (row-blocks 0..1023)

template <int BP>
struct Cfg {
  static constexpr int N = 2 * BP;                   // MMA N: hi rows then lo rows
  static constexpr int CPG = BP == 8 ? 4 : 2;        // chunks per group (one hand-off between roles)
  static constexpr int GPU = kUC / CPG;              // groups per unit
  static constexpr int SG = 2;                       // groups in flight: A tiles and accumulators in TMEM
  static constexpr int T = N * 128;                  // activation tile bytes (one chunk)
  static constexpr int XU = kUC * T + kUC * 256;     // activation unit: 4 tiles + 4 x block sums
  static constexpr int SCAL = 1024;                  // per chunk: [2][128] u32 row scale words
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W = OFF_X + kRX * XU;
  static constexpr int OFF_SCAL = OFF_W + kRW * kWU;
  // Each CTA takes all 512 TMEM columns, so two CTAs must never share an SM
  // (the second would wait in tcgen05.alloc): ask for more than half of the
  // SM's shared memory.
  static constexpr int SMEM_USED = OFF_SCAL + SG * CPG * SCAL + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static constexpr uint32_t A_COLS = CPG * kACols;   // TMEM columns of a group's A tiles
  static constexpr uint32_t D_COLS = CPG * 2 * N;    // TMEM columns of a group's block accumulators
  static constexpr uint32_t D_COL0 = SG * A_COLS;    // A tiles first, then the accumulators
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(D_COL0 + SG * D_COLS <= TMEM_COLS, "TMEM budget");
  static constexpr uint32_t IDESC = sg_idesc_f16(128, N);
  static_assert(XU % 1024 == 0, "activation units must keep 1024-byte tile alignment");
};

struct Mat {
  const uint8_t* tiles;
  const uint32_t* dd;
  float* y;
  int64_t ldy;
  int n_rb, n_rows, n_sb, rb0;
};

struct Params {
  Mat mats[SG_GEMV_MAX_MATS];
  int n_mats, batch, n_ch, n_sc, accumulate;
  int64_t total;          // row-blocks x units
  const uint8_t* xunits;  // activation units (xprep layout)
  const float* inv;       // [16] per-token 2^-e
  int total_rb;
  int zero_all;                  // more row-blocks than the mask holds: zero every split candidate
  uint32_t split[kMaskWords];    // bit rbg: row-block reduced by more than one CTA (zeroed first)
};

__device__ __forceinline__ int find_mat(const Params& p, int rbg) {
  int m = 0;
#pragma unroll
  for (int i = 1; i < SG_GEMV_MAX_MATS; ++i)
    if (i < p.n_mats && rbg >= p.mats[i].rb0) m = i;
  return m;
}

// Unit cursor: walks the CTA's units without divisions.
struct Cursor {
  int rbg, sc, mi, rb;  // global row-block, unit within it, matrix, row-block within the matrix
  __device__ __forceinline__ void init(const Params& p, int64_t gu) {
    rbg = (int)(gu / p.n_sc);
    sc = (int)(gu % p.n_sc);
    mi = find_mat(p, rbg);
    rb = rbg - p.mats[mi].rb0;
  }
  __device__ __forceinline__ int chunks(const Params& p) const { return min(kUC, p.n_ch - kUC * sc); }
  __device__ __forceinline__ void next(const Params& p) {
    if (++sc == p.n_sc) {
      sc = 0;
      ++rbg;
      ++rb;
      if (mi + 1 < p.n_mats && rbg >= p.mats[mi + 1].rb0) {
        ++mi;
        rb = 0;
      }
    }
  }
};

// ---------------------------------------------------------------- x prep
// Grid (block groups of 8, token rows BP). For token row t < batch: the
// token's max|x| sets s = 2^e (max|x|*s in [2^14, 2^15)); positions k%8 in
// {2,3,6,7} carry x*s/16 (their A values are 1024+16q). u is the value the
// tensor core sees (hi + lo, times 16 at those positions). Token rows
// batch <= t < BT are written as zeros. Unit layout (XU bytes per 4 chunks):
// 4 operand tiles [row 2*BP][128 B, 16-byte segment j of row r at
// ((j ^ (r & 7)) << 4)], rows 0..BT-1 hi parts and BT..2BT-1 lo parts (rows
// from 2*BT on are never read back: their product columns are ignored), then
// per chunk
// sums[blk 2][2][16]: [0] Q4_0: sum (c+8) u, Q4_K: sum c u (c = 1024 or
// 64); [1] sum u.
template <int BP, int BT>
__global__ void __launch_bounds__(256) gemv_xprep_kernel(const float* __restrict__ x, int64_t ldx, int K, int n_blk,
                                                         int q40, uint8_t* __restrict__ xunits,
                                                         float* __restrict__ inv, Params zp, int zero_split) {
  using C = Cfg<BP>;
  pdl_launch_dependents();
  pdl_wait();  // x may come from the previous kernel; scratch and y may still be in use by it
  __shared__ float red[8];
  const int t = blockIdx.y;
  const bool live = t < zp.batch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = x + (int64_t)t * ldx;
  float m = 0.f;
  if (live)
    for (int k = threadIdx.x * 4; k < K; k += 1024) {
      const float4 v = *reinterpret_cast<const float4*>(xr + k);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
  int se = 0;  // scale exponent
  if (m > 0.f && m <= 3.0e38f) {
    const int e = ((__float_as_int(m) >> 23) & 0xFF) - 127;  // m in [2^e, 2^(e+1)) for normal m
    se = max(-126, min(127, 14 - e));
  }
  const float s = __int_as_float((127 + se) << 23);
  if (live && blockIdx.x == 0 && threadIdx.x == 0) inv[t] = __int_as_float((127 - se) << 23);
  const bool scaled = (lane >> 1) & 1;  // k % 8 in {2,3,6,7}
  const float c = scaled ? 64.f : 1024.f;
  const int b = blockIdx.x * 8 + warp;
  if (b < n_blk) {
    const int k = 32 * b + lane;
    const float v = (live && k < K) ? xr[k] : 0.f;
    const float xs = scaled ? v * s * 0.0625f : v * s;
    const __half hi = __float2half_rn(xs);
    const __half lo = __float2half_rn(xs - __half2float(hi));
    const int ch = b >> 1, kc = k & 63, j = kc >> 3;
    uint8_t* unit = xunits + (int64_t)(ch / kUC) * C::XU;
    uint8_t* tile = unit + (ch % kUC) * C::T;
    const int rh = t, rl = BT + t;  // live hi rows, then live lo rows
    *reinterpret_cast<__half*>(tile + rh * 128 + ((j ^ (rh & 7)) << 4) + (kc & 7) * 2) = hi;
    *reinterpret_cast<__half*>(tile + rl * 128 + ((j ^ (rl & 7)) << 4) + (kc & 7) * 2) = lo;
    const float u = (__half2float(hi) + __half2float(lo)) * (scaled ? 16.f : 1.f);
    float a = (q40 ? c + 8.f : c) * u, su = u;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      su += __shfl_xor_sync(0xffffffffu, su, o);
    }
    if (lane == 0) {
      float* sums = reinterpret_cast<float*>(unit + kUC * C::T + (ch % kUC) * 256) + (b & 1) * 32;
      sums[t] = a;
      sums[16 + t] = su;
    }
  }
  if (zero_split && live && blockIdx.x == 0) {
    for (int rbg = warp; rbg < zp.total_rb; rbg += 8) {
      if (!zp.zero_all && !((zp.split[rbg >> 5] >> (rbg & 31)) & 1u)) continue;
      const Mat& mt = zp.mats[find_mat(zp, rbg)];
      float* yr = mt.y + (int64_t)t * mt.ldy + (int64_t)(rbg - mt.rb0) * 128;
      const int nr = min(128, mt.n_rows - (rbg - mt.rb0) * 128);
      for (int r = lane; r < nr; r += 32) yr[r] = 0.f;
    }
  }
}

// ---------------------------------------------------------------- GEMV
// BT: live token columns rounded up to a power of two (<= BP)
template <int DT, int BP, int BT>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(Params p) {
  using C = Cfg<BP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // per group g (CPG chunks): a_full[g % SG] -- its A tiles are in TMEM;
  // d_full[g % SG] -- its MMAs completed; d_free[g % SG] -- its epilogue is
  // done, so its A tiles, accumulators and row scales may be rewritten
  __shared__ __align__(8) uint64_t w_full[kRW], w_empty[kRW], x_full[kRX], x_empty[kRX], a_full[C::SG],
      d_full[C::SG], d_free[C::SG];
  __shared__ uint32_t tmem_base_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int64_t u0 = (int64_t)blockIdx.x * p.total / G, u1 = (int64_t)(blockIdx.x + 1) * p.total / G;
  const int nu = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int r = 0; r < kRW; ++r) {
      mbar_init(&w_full[r], 1);
      mbar_init(&w_empty[r], 4);
    }
    for (int r = 0; r < kRX; ++r) {
      mbar_init(&x_full[r], 1);
      mbar_init(&x_empty[r], 4);
    }
    for (int s = 0; s < C::SG; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&d_full[s], 1);
      mbar_init(&d_free[s], 4);
    }
    mbar_fence_init();
  }
  if (warp == 1) sg_tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  sg_tc_fence_before();
  __syncthreads();
  sg_tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ========================================================= weight producer
    if (lane == 0) {
      Cursor uc;
      uc.init(p, u0);
      int v = 0;
      for (; v < nu; ++v) {
        const int ws = v % kRW;
        if (v >= kRW && !mbar_wait(&w_empty[ws], ((v / kRW) & 1) ^ 1, 0x21)) break;
        const Mat& mt = p.mats[uc.mi];
        const int cnt = uc.chunks(p);
        uint8_t* dst = smem + C::OFF_W + ws * kWU;
        mbar_arrive_expect_tx(&w_full[ws], cnt * SG_TILE_BYTES + (DT == SG_DTYPE_Q4_K ? 512 : 0));
        bulk_g2s(dst, mt.tiles + ((int64_t)uc.rb * p.n_ch + kUC * uc.sc) * SG_TILE_BYTES, cnt * SG_TILE_BYTES,
                 &w_full[ws]);
        if (DT == SG_DTYPE_Q4_K)  // one Q4_K super-block per unit
          bulk_g2s(dst + kUC * SG_TILE_BYTES, mt.dd + ((int64_t)uc.rb * mt.n_sb + uc.sc) * 128, 512, &w_full[ws]);
        uc.next(p);
      }
      if (*(volatile int*)&g_sg_error != 0)  // error path: no copy may land after the CTA exits
        for (int j = max(0, v - kRW); j < v; ++j) mbar_wait_drain(&w_full[j % kRW], (j / kRW) & 1);
    }
  } else if (warp == 10) {
    // ===================================================== activation producer
    if (lane == 0) {
      pdl_wait();  // activations and sums come from the prep kernel
      Cursor uc;
      uc.init(p, u0);
      int v = 0;
      for (; v < nu; ++v) {
        const int xs = v % kRX;
        if (v >= kRX && !mbar_wait(&x_empty[xs], ((v / kRX) & 1) ^ 1, 0x22)) break;
        mbar_arrive_expect_tx(&x_full[xs], C::XU);
        bulk_g2s(smem + C::OFF_X + xs * C::XU, p.xunits + (int64_t)uc.sc * C::XU, C::XU, &x_full[xs]);
        uc.next(p);
      }
      if (*(volatile int*)&g_sg_error != 0)
        for (int j = max(0, v - kRX); j < v; ++j) mbar_wait_drain(&x_full[j % kRX], (j / kRX) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      Cursor uc;
      uc.init(p, u0);
      int g = 0;
      bool ok = true;
      for (int v = 0; v < nu && ok; ++v) {
        const int xs = v % kRX, cnt = uc.chunks(p);
        if (!mbar_wait(&x_full[xs], (v / kRX) & 1, 0x23)) break;
        for (int gi = 0; gi < C::GPU && gi * C::CPG < cnt; ++gi, ++g) {
          const int sg = g % C::SG;
          if (!mbar_wait(&a_full[sg], (g / C::SG) & 1, 0x24) ||
              (g >= C::SG && !mbar_wait(&d_free[sg], ((g / C::SG) & 1) ^ 1, 0x29))) {
            ok = false;
            break;
          }
          sg_tc_fence_after();
          const int gc = min(C::CPG, cnt - gi * C::CPG);
          for (int ci = 0; ci < gc; ++ci) {
            const int cu = gi * C::CPG + ci;  // chunk within the unit
            const uint32_t a0 = tmem + (uint32_t)(sg * C::A_COLS + ci * kACols);
            const uint64_t bd = sg_sdesc(smem_u32(smem + C::OFF_X + xs * C::XU + cu * C::T), SG_SW128);
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
              const uint32_t d = tmem + C::D_COL0 + (uint32_t)(sg * C::D_COLS + (ci * 2 + blk) * C::N);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int ks = 2 * blk + j;  // 16 K = 8 TMEM columns of A, 32 bytes of B
                sg_umma_tmem_a(d, a0 + (uint32_t)(ks * 8), bd + (uint64_t)(ks * 2), C::IDESC, (uint32_t)j);
              }
            }
          }
          sg_umma_commit(&d_full[sg]);
        }
        uc.next(p);
      }
      // every MMA issued must have completed before TMEM is freed (the last
      // commit covers all of them; on the normal path this returns at once)
      if (g > 0) mbar_wait_drain(&d_full[(g - 1) % C::SG], ((g - 1) / C::SG) & 1);
    }
  } else if (warp < 6) {
    // ====================================================== dequant warps
    const int q = warp & 3;  // TMEM lane quadrant: rows 32q .. 32q+31
    const int row = q * 32 + lane;
    Cursor uc;
    uc.init(p, u0);
    int g = 0;
    bool ok = true;
    for (int v = 0; v < nu && ok; ++v) {
      const int ws = v % kRW, cnt = uc.chunks(p);
      if (!__all_sync(0xffffffffu, mbar_wait(&w_full[ws], (v / kRW) & 1, 0x26))) break;
      const uint8_t* wu = smem + C::OFF_W + ws * kWU;
      uint32_t ddw = 0;
      if (DT == SG_DTYPE_Q4_K) ddw = *reinterpret_cast<const uint32_t*>(wu + kUC * SG_TILE_BYTES + row * 4);
      for (int gi = 0; gi < C::GPU && gi * C::CPG < cnt; ++gi, ++g) {
        const int sg = g % C::SG;
        // the group's A tiles, accumulators and scale words were last used by
        // group g - SG: wait until its epilogue has released them
        const bool w = g < C::SG || mbar_wait(&d_free[sg], ((g / C::SG) & 1) ^ 1, 0x27);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        sg_tc_fence_after();
        uint32_t* scal = reinterpret_cast<uint32_t*>(smem + C::OFF_SCAL + sg * C::CPG * C::SCAL);
        const int gc = min(C::CPG, cnt - gi * C::CPG);
        for (int ci = 0; ci < gc; ++ci) {
          const uint8_t* tile = wu + (gi * C::CPG + ci) * SG_TILE_BYTES;
          const uint4 n0 = *reinterpret_cast<const uint4*>(tile + row * 16);
          const uint4 n1 = *reinterpret_cast<const uint4*>(tile + 2048 + row * 16);
          scal[ci * 256 + row] = *reinterpret_cast<const uint32_t*>(tile + SG_TILE_SC_OFF + row * 4);
          if (DT == SG_DTYPE_Q4_K) scal[ci * 256 + 128 + row] = ddw;
          // this thread's row of the A tile: column c holds K pair (2c, 2c+1)
          const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
          uint32_t av[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 d = sg_decode_word_f16(nw[j]);
            av[4 * j] = d.x;
            av[4 * j + 1] = d.y;
            av[4 * j + 2] = d.z;
            av[4 * j + 3] = d.w;
          }
          sg_tmem_st32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(sg * C::A_COLS + ci * kACols), av);
        }
        sg_tmem_st_wait();
        sg_tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sg]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_empty[ws]);  // this warp has read all of the unit's weights
      uc.next(p);
    }
  } else {
    // ============================================================ epilogue warps
    const int q = warp & 3;  // TMEM lane quadrant
    const int row = q * 32 + lane;
    float acc[BT];
#pragma unroll
    for (int t = 0; t < BT; ++t) acc[t] = 0.f;
    bool waited_prev = false;
    Cursor uc;
    uc.init(p, u0);
    bool seg_whole_start = uc.sc == 0;
    int g = 0;
    bool ok = true;
    for (int v = 0; v < nu && ok; ++v) {
      const int xs = v % kRX, cnt = uc.chunks(p);
      if (!__all_sync(0xffffffffu, mbar_wait(&x_full[xs], (v / kRX) & 1, 0x2B))) break;  // block sums
      for (int gi = 0; gi < C::GPU && gi * C::CPG < cnt; ++gi, ++g) {
        const int sg = g % C::SG;
        if (!__all_sync(0xffffffffu, mbar_wait(&d_full[sg], (g / C::SG) & 1, 0x25))) {
          ok = false;
          break;
        }
        sg_tc_fence_after();
        const uint32_t* scal = reinterpret_cast<const uint32_t*>(smem + C::OFF_SCAL + sg * C::CPG * C::SCAL);
        const int gc = min(C::CPG, cnt - gi * C::CPG);
        for (int ci = 0; ci < gc; ++ci) {
          const int cu = gi * C::CPG + ci;
          const float* sums = reinterpret_cast<const float*>(smem + C::OFF_X + xs * C::XU + kUC * C::T + cu * 256);
          const uint32_t scw = scal[ci * 256 + row];
          float sc[2], of[2];
          if (DT == SG_DTYPE_Q4_0) {
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&scw));
            sc[0] = d.x;
            sc[1] = d.y;
            of[0] = of[1] = 0.f;
          } else {
            const uint32_t ddw = scal[ci * 256 + 128 + row];
            const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&ddw));
            sc[0] = dm.x * (float)(scw & 0xFFu);
            sc[1] = dm.x * (float)((scw >> 8) & 0xFFu);
            of[0] = dm.y * (float)((scw >> 16) & 0xFFu);
            of[1] = dm.y * (float)(scw >> 24);
          }
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
            const uint32_t taddr =
                tmem + ((uint32_t)(q * 32) << 16) + C::D_COL0 + (uint32_t)(sg * C::D_COLS + (ci * 2 + blk) * C::N);
            uint32_t hl[2 * BT];  // hi-part columns [0, BT), lo-part columns [BT, 2 BT)
            sg_tmem_ld_n<2 * BT>(taddr, hl);
            sg_tmem_ld_wait();
            const float* s0 = sums + blk * 32;
#pragma unroll
            for (int t = 0; t < BT; ++t) {
              const float dot = (__uint_as_float(hl[t]) + __uint_as_float(hl[BT + t])) - s0[t];
              if (DT == SG_DTYPE_Q4_0) acc[t] = fmaf(sc[blk], dot, acc[t]);
              else acc[t] = fmaf(sc[blk], dot, fmaf(-of[blk], s0[16 + t], acc[t]));
            }
          }
        }
        sg_tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_free[sg]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_empty[xs]);  // this warp is done with the unit's block sums
      // row-block segment finished: store it whole, or reduce it
      const bool rb_end = uc.sc == p.n_sc - 1;
      if (rb_end || v == nu - 1) {
        if (!waited_prev) {
          pdl_wait();  // y: zeroing by the prep kernel, readers of the previous kernel
          waited_prev = true;
        }
        const Mat& mt = p.mats[uc.mi];
        const int grow = uc.rb * 128 + row;
        const bool whole = rb_end && seg_whole_start;
        if (grow < mt.n_rows) {
#pragma unroll
          for (int t = 0; t < BT; ++t) {
            if (t < p.batch) {
              float* yp = mt.y + (int64_t)t * mt.ldy + grow;
              const float val = acc[t] * p.inv[t];
              if (!whole) red_add_f32(yp, val);
              else *yp = p.accumulate ? *yp + val : val;
            }
          }
        }
#pragma unroll
        for (int t = 0; t < BT; ++t) acc[t] = 0.f;
        seg_whole_start = true;  // the next segment starts at unit 0 of its row-block
      }
      uc.next(p);
    }
  }
  pdl_launch_dependents();
  sg_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sg_tc_fence_after();
    sg_tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------ host side
struct Layout {
  uint8_t* xunits;
  float* inv;
  size_t bytes;
};

// scratch: activation units for the larger tile (BP = 16) + per-token scales
Layout layout_of(void* base, int64_t K) {
  auto up = [](size_t v) { return (v + 1023) & ~(size_t)1023; };
  const int64_t n_sc = ((K + 63) / 64 + kUC - 1) / kUC;
  Layout l;
  uint8_t* b = static_cast<uint8_t*>(base);
  const size_t xb = up((size_t)n_sc * Cfg<16>::XU);
  l.xunits = b;
  l.inv = reinterpret_cast<float*>(b + xb);
  l.bytes = xb + 1024;
  return l;
}

template <int DT, int BP, int BT>
cudaError_t launch(const Params& p, int G, const float* x, int64_t ldx, int K, bool zero_split, const Layout& l,
                   cudaStream_t st) {
  using C = Cfg<BP>;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((2 * p.n_ch + 7) / 8), (unsigned)BT);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_xprep_kernel<BP, BT>, x, ldx, K, 2 * p.n_ch, DT == SG_DTYPE_Q4_0 ? 1 : 0,
                                     l.xunits, l.inv, p, zero_split ? 1 : 0);
  if (e != cudaSuccess) return e;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(gemv_kernel<DT, BP, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_done[dev] = 1;
  }
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)G);
  g.blockDim = dim3(kThreads);
  g.dynamicSmemBytes = C::SMEM;
  g.stream = st;
  g.attrs = attr;
  g.numAttrs = 1;
  return cudaLaunchKernelEx(&g, gemv_kernel<DT, BP, BT>, p);
}

}  // namespace gemv_tc

size_t sg_gemv_scratch_bytes(int64_t n_cols) { return gemv_tc::layout_of(nullptr, n_cols).bytes; }

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  using namespace gemv_tc;
  if (n_mats < 1 || n_mats > SG_GEMV_MAX_MATS || batch < 1 || batch > SG_GEMV_MAX_BATCH || !x || !scratch)
    return cudaErrorInvalidValue;
  const SgDevWeight* w0 = mats[0].w;
  const int64_t K = w0->n_cols;
  if ((K & 31) || K > (1 << 28) || ((uintptr_t)x & 15) || (ldx & 3) || ldx < K) return cudaErrorInvalidValue;
  if (scratch_bytes < sg_gemv_scratch_bytes(K) || ((uintptr_t)scratch & 255)) return cudaErrorInvalidValue;
  Params p = {};
  p.n_mats = n_mats;
  p.batch = batch;
  p.n_ch = (int)w0->n_ch;
  p.n_sc = (p.n_ch + kUC - 1) / kUC;
  p.accumulate = accumulate ? 1 : 0;
  int rb = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->n_cols != K || w->dtype != w0->dtype || !mats[i].y || mats[i].ldy < w->n_rows) return cudaErrorInvalidValue;
    p.mats[i] = {w->tiles, w->dd, mats[i].y, mats[i].ldy, (int)w->n_rb, (int)w->n_rows, (int)w->n_sb, rb};
    rb += (int)w->n_rb;
  }
  p.total = (int64_t)rb * p.n_sc;
  const Layout l = layout_of(scratch, K);
  p.xunits = l.xunits;
  p.inv = l.inv;
  // one CTA per SM
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms, p.total));
  p.total_rb = rb;
  p.zero_all = rb > kMaskWords * 32;
  bool split = false;
  for (int c = 1; c < G; ++c) {
    const int64_t gu = (int64_t)c * p.total / G;
    if (gu % p.n_sc == 0) continue;
    split = true;
    const int64_t r = gu / p.n_sc;
    if (r < kMaskWords * 32) p.split[r >> 5] |= 1u << (r & 31);
  }
  const bool zero_split = split && !accumulate;
  const int K32 = (int)K;
#define SG_GEMV_LAUNCH(DT)                                                                     \
  switch (batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16) {           \
    case 1: return launch<DT, 8, 1>(p, G, x, ldx, K32, zero_split, l, st);                      \
    case 2: return launch<DT, 8, 2>(p, G, x, ldx, K32, zero_split, l, st);                      \
    case 4: return launch<DT, 8, 4>(p, G, x, ldx, K32, zero_split, l, st);                      \
    case 8: return launch<DT, 8, 8>(p, G, x, ldx, K32, zero_split, l, st);                      \
    default: return launch<DT, 16, 16>(p, G, x, ldx, K32, zero_split, l, st);                   \
  }
  if (w0->dtype == SG_DTYPE_Q4_0) SG_GEMV_LAUNCH(SG_DTYPE_Q4_0)
  SG_GEMV_LAUNCH(SG_DTYPE_Q4_K)
#undef SG_GEMV_LAUNCH
}
