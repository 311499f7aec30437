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
// Kernels, chained with programmatic dependent launch:
//  1. gemv_xprep_kernel: one CTA per token -- power-of-two scale, f16 hi/lo
//     activations, per-block sums, zeroing of the output rows that several
//     CTAs share.
//  2. gemv_kernel<dtype, BP>: balanced split -- CTA c takes iterations
//     [c*T/G, (c+1)*T/G) of the T = row-blocks x K-chunks space, crossing
//     row-block (and matrix) boundaries; a row-block seen whole is stored, a
//     shared one is reduced with red.add.
//       warp 0     producer: cp.async.bulk of packed weight tiles (4.5 KB per
//                  128 rows x 64 K) into a 7-slot ring -- the first ones
//                  before the wait on the previous kernel, weights do not
//                  depend on it -- then TMA of the activation tiles and block
//                  sums per chunk.
//       warp 1     TMEM owner; one thread issues tcgen05.mma (M=128,
//                  N=2*BP: BP hi token rows + BP lo token rows, K=16, f16 ->
//                  f32), two per 32-block, into a ring of TMEM slots.
//       warps 2-5  dequant: one weight row per thread, 16-byte nibble loads,
//                  4 lop3 per 8 weights into the 128-byte-swizzled A tile.
//       warps 6-9  epilogue: per chunk, tcgen05.ld of the two block
//                  accumulators of its TMEM lane quadrant (warp % 4), block
//                  scales in f32, output rows stored or reduced.
// Rings decouple the roles: weight tiles (freed by the dequant warps), A
// tiles and activation tiles (freed by the MMA commit) and TMEM slots with
// their block sums and row scales (freed by the epilogue); the producer
// serves the weight and activation queues without blocking on either.
// Every mbarrier wait is bounded (sg_common.cuh).
#include <algorithm>

#include "sg_gemv.cuh"
#include "sg_tc.cuh"

namespace gemv_tc {

constexpr int kSA = 3;                // dequantized A tiles (freed by the MMA commit)
constexpr int kPD = 4;                // weight chunks in flight per dequant thread (registers)
constexpr int kA = 128 * 128;         // 128 rows x 64 K f16
constexpr int kThreads = 320;
constexpr int kXLag = 2;              // activation chunks in flight per producer lane

template <int BP>
struct Cfg {
  static constexpr int N = 2 * BP;                   // MMA N: hi rows then lo rows
  static constexpr int SD = BP == 8 ? 8 : 4;         // TMEM slots / block sums / row scales in flight
  static constexpr int SX = BP == 8 ? 6 : 4;         // activation tiles (freed by the MMA commit)
  static constexpr int X = N * 128;                  // activation tile bytes
  static constexpr int SUM = 256;                    // [blk 2][2][16] f32
  static constexpr int SCAL = 1024;                  // [2][128] u32 row scale words
  static constexpr int OFF_X = kSA * kA;
  static constexpr int OFF_SUM = OFF_X + SX * X;
  static constexpr int OFF_SCAL = OFF_SUM + SD * SUM;
  static constexpr int SMEM = OFF_SCAL + SD * SCAL + 1024;
  static constexpr uint32_t TMEM_COLS = SD * 2 * N;  // 256
  static constexpr uint32_t IDESC = sg_idesc_f16(128, N);
};

struct Mat {
  const uint8_t* tiles;
  const uint32_t* dd;
  float* y;
  int64_t ldy;
  int n_rb, n_rows, n_sb, rb0;
};

constexpr int kMaskWords = 32;  // split row-block bitmask (row-blocks 0..1023)

struct Params {
  Mat mats[SG_GEMV_MAX_MATS];
  int n_mats, batch, n_ch, accumulate;
  int64_t total;      // row-blocks x chunks
  const float* sums;  // [2*n_ch][2][16]
  const float* inv;   // [16] per-token 2^-e
  const __half* xh;   // [batch][K] activation parts
  const __half* xl;
  int K;
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

// ---------------------------------------------------------------- x prep
// Grid (block groups, tokens). Each CTA finds its token's max|x| (scale
// s = 2^e puts it in [2^14, 2^15)), then converts 8 blocks of 32: positions
// k%8 in {2,3,6,7} carry x*s/16 (their A values are 1024+16q). u is the value
// the tensor core sees (hi + lo, times 16 at those positions).
// sums[b][0][t] = Q4_0: sum (c+8) u, Q4_K: sum c u   (c = 1024 or 64)
// sums[b][1][t] = sum u
// CTAs with blockIdx.x == 0 also zero their token's outputs in the row-blocks
// that several GEMV CTAs reduce into.
__global__ void __launch_bounds__(256) gemv_xprep_kernel(const float* __restrict__ x, int64_t ldx, int K, int n_blk,
                                                         int q40, __half* __restrict__ xh, __half* __restrict__ xl,
                                                         float* __restrict__ sums, float* __restrict__ inv,
                                                         Params zp, int zero_split) {
  pdl_launch_dependents();
  pdl_wait();  // x may come from the previous kernel; scratch and y may still be in use by it
  __shared__ float red[8];
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = x + (int64_t)t * ldx;
  float m = 0.f;
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
  if (blockIdx.x == 0 && threadIdx.x == 0) inv[t] = __int_as_float((127 - se) << 23);
  const bool scaled = (lane >> 1) & 1;  // k % 8 in {2,3,6,7}
  const float c = scaled ? 64.f : 1024.f;
  const int b = blockIdx.x * 8 + warp;
  if (b < n_blk) {
    const int k = 32 * b + lane;
    const float v = k < K ? xr[k] : 0.f;
    const float xs = scaled ? v * s * 0.0625f : v * s;
    const __half hi = __float2half_rn(xs);
    const __half lo = __float2half_rn(xs - __half2float(hi));
    if (k < K) {
      xh[(int64_t)t * K + k] = hi;
      xl[(int64_t)t * K + k] = lo;
    }
    const float u = (__half2float(hi) + __half2float(lo)) * (scaled ? 16.f : 1.f);
    float a = (q40 ? c + 8.f : c) * u, su = u;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      su += __shfl_xor_sync(0xffffffffu, su, o);
    }
    if (lane == 0) {
      sums[(b * 2 + 0) * 16 + t] = a;
      sums[(b * 2 + 1) * 16 + t] = su;
    }
  }
  if (zero_split && blockIdx.x == 0) {
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
// Chunk cursor: walks the CTA's iterations without divisions.
struct Cursor {
  int rbg, c, mi, rb;  // global row-block, chunk, matrix, row-block within the matrix
  __device__ __forceinline__ void init(const Params& p, int64_t gi) {
    rbg = (int)(gi / p.n_ch);
    c = (int)(gi % p.n_ch);
    mi = find_mat(p, rbg);
    rb = rbg - p.mats[mi].rb0;
  }
  __device__ __forceinline__ void next(const Params& p) {
    if (++c == p.n_ch) {
      c = 0;
      ++rbg;
      ++rb;
      if (mi + 1 < p.n_mats && rbg >= p.mats[mi + 1].rb0) {
        ++mi;
        rb = 0;
      }
    }
  }
};

template <int DT, int BP>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(Params p) {
  using C = Cfg<BP>;
  constexpr int SD = C::SD;
  constexpr int SX = C::SX;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // d_full[i % SD] completes when chunk i's MMAs are done: it also frees A
  // slot i % kSA and activation slot i % SX (kSA, SX <= SD)
  static_assert(kSA <= SD && SX <= SD, "ring sizes");
  __shared__ __align__(8) uint64_t a_full[kSA], x_full[SX], sums_full[SD], d_full[SD], d_free[SD];
  __shared__ uint32_t tmem_base_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * p.total / G, i1 = (int64_t)(blockIdx.x + 1) * p.total / G;
  const int n = (int)(i1 - i0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSA; ++s) mbar_init(&a_full[s], 4);
    for (int s = 0; s < SX; ++s) mbar_init(&x_full[s], 32);
    for (int s = 0; s < SD; ++s) {
      mbar_init(&sums_full[s], 32);
      mbar_init(&d_full[s], 1);
      mbar_init(&d_free[s], 4);
    }
    mbar_fence_init();
  }
  if (warp == 0) {
    // activation rows >= batch are never written: zero every slot once
    uint4* xz = reinterpret_cast<uint4*>(smem + C::OFF_X);
    for (int i = lane; i < SX * C::X / 16; i += 32) xz[i] = make_uint4(0, 0, 0, 0);
  }
  if (warp == 1) sg_tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  sg_tc_fence_before();
  __syncthreads();
  sg_tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ======================================================= activation producer
    // Per chunk: the BP hi + BP lo token rows (64 K each, 128-byte swizzle)
    // and the block sums, copied with cp.async by the 32 lanes; a chunk is
    // published (proxy fence + arrive) kXLag chunks after it was issued.
    pdl_wait();  // activations and sums come from the prep kernel
    Cursor xc;
    xc.init(p, i0);
    const int nrow = 2 * p.batch;  // real rows: hi of each token, then lo
    bool ok = true;
    auto publish = [&](int j) {
      fence_proxy_async_smem();  // generic-proxy copies -> visible to the tensor core
      mbar_arrive(&x_full[j % SX]);
      mbar_arrive(&sums_full[j % SD]);
    };
    for (int i = 0; i < n; ++i) {
      const int sx = i % SX, sd = i % SD;
      bool w = true;
      if (i >= SX) w = mbar_wait(&d_full[(i - SX) % SD], ((i - SX) / SD) & 1, 0x21);
      if (w && i >= SD) w = mbar_wait(&d_free[sd], ((i / SD) & 1) ^ 1, 0x28);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      uint8_t* xt = smem + C::OFF_X + sx * C::X;
      const int k0 = 64 * xc.c;
      for (int e = lane; e < nrow * 8; e += 32) {
        const int rr = e >> 3, j = e & 7;            // rr: 0..batch-1 hi, batch.. lo
        const int t = rr < p.batch ? rr : rr - p.batch;
        const int srow = rr < p.batch ? t : BP + t;  // smem row
        const __half* src = (rr < p.batch ? p.xh : p.xl) + (int64_t)t * p.K + k0 + 8 * j;
        const int valid = p.K - (k0 + 8 * j) >= 8 ? 16 : 0;  // K is a multiple of 32
        cp_async16(xt + srow * 128 + ((j ^ (srow & 7)) << 4), valid ? src : p.xh, valid);
      }
      if (lane < 16)
        cp_async16(smem + C::OFF_SUM + sd * C::SUM + lane * 16, p.sums + (int64_t)xc.c * 64 + lane * 4, 16);
      cp_async_commit();
      xc.next(p);
      if (i >= kXLag) {
        cp_async_wait<kXLag>();
        publish(i - kXLag);
      }
    }
    cp_async_wait<0>();
    if (ok)
      for (int j = max(0, n - kXLag); j < n; ++j) publish(j);
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int sa = i % kSA, sx = i % SX, sd = i % SD;
        if (!mbar_wait(&a_full[sa], (i / kSA) & 1, 0x24) || !mbar_wait(&x_full[sx], (i / SX) & 1, 0x23)) break;
        if (i >= SD && !mbar_wait(&d_free[sd], ((i / SD) & 1) ^ 1, 0x29)) break;
        sg_tc_fence_after();
        const uint64_t ad = sg_sdesc(smem_u32(smem + sa * kA), SG_SW128);
        const uint64_t bd = sg_sdesc(smem_u32(smem + C::OFF_X + sx * C::X), SG_SW128);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          const uint32_t d = tmem + (uint32_t)((sd * 2 + blk) * C::N);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint64_t o = (uint64_t)((2 * blk + j) * 2);  // 16 K = 32 bytes
            sg_umma(d, ad + o, bd + o, C::IDESC, (uint32_t)j);
          }
        }
        sg_umma_commit(&d_full[sd]);
        issued = i + 1;
      }
      // every MMA issued must have completed before TMEM is freed (the last
      // commit covers all of them; on the normal path this returns at once)
      if (issued > 0) mbar_wait_drain(&d_full[(issued - 1) % SD], ((issued - 1) / SD) & 1);
    }
  } else if (warp < 6) {
    // ====================================================== dequant warps
    // One weight row per thread. The row's bytes of each chunk (2 x 16 B of
    // nibbles, its scale word, Q4_K d|dmin) are loaded straight into
    // registers kPD chunks ahead (coalesced: a warp's 32 rows are 512
    // contiguous bytes), so the proxy fence before the tensor core reads the
    // A tile covers only this thread's shared-memory stores.
    const int row = (warp & 3) * 32 + lane;
    const int x7 = row & 7;
    Cursor rc;
    rc.init(p, i0);
    uint4 qa[kPD], qb[kPD];
    uint32_t qs[kPD], qd[kPD];
    auto load = [&](int slot) {
      const Mat& mt = p.mats[rc.mi];
      const uint8_t* tile = mt.tiles + ((int64_t)rc.rb * p.n_ch + rc.c) * SG_TILE_BYTES;
      qa[slot] = __ldcs(reinterpret_cast<const uint4*>(tile + row * 16));
      qb[slot] = __ldcs(reinterpret_cast<const uint4*>(tile + 2048 + row * 16));
      qs[slot] = __ldcs(reinterpret_cast<const unsigned int*>(tile + SG_TILE_SC_OFF) + row);
      if (DT == SG_DTYPE_Q4_K)
        qd[slot] = __ldcs(reinterpret_cast<const unsigned int*>(mt.dd + ((int64_t)rc.rb * mt.n_sb + (rc.c >> 2)) * 128) + row);
      rc.next(p);
    };
#pragma unroll
    for (int j = 0; j < kPD; ++j)
      if (j < n) load(j);
    bool ok = true;
    for (int i0c = 0; i0c < n && ok; i0c += kPD) {
#pragma unroll
      for (int j = 0; j < kPD; ++j) {
        const int i = i0c + j;
        if (i >= n) break;
        const int sa = i % kSA, sd = i % SD;
        const uint4 n0 = qa[j], n1 = qb[j];
        const uint32_t scw = qs[j], ddw = qd[j];
        if (i + kPD < n) load(j);  // refill this register slot kPD chunks ahead
        bool w = true;
        if (i >= kSA) w = mbar_wait(&d_full[(i - kSA) % SD], ((i - kSA) / SD) & 1, 0x27);
        if (w && i >= SD) w = mbar_wait(&d_free[sd], ((i / SD) & 1) ^ 1, 0x2A);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        uint32_t* scal = reinterpret_cast<uint32_t*>(smem + C::OFF_SCAL + sd * C::SCAL);
        scal[row] = scw;
        if (DT == SG_DTYPE_Q4_K) scal[128 + row] = ddw;
        uint8_t* arow = smem + sa * kA + row * 128;
        const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) *reinterpret_cast<uint4*>(arow + ((k ^ x7) << 4)) = sg_decode_word_f16(nw[k]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
    }
  } else {
    // ============================================================ epilogue warps
    const int q = warp & 3;  // TMEM lane quadrant
    const int row = q * 32 + lane;
    float acc[BP];
#pragma unroll
    for (int t = 0; t < BP; ++t) acc[t] = 0.f;
    bool waited_prev = false;
    Cursor cur;
    cur.init(p, i0);
    bool seg_whole_start = cur.c == 0;
    for (int i = 0; i < n; ++i) {
      const int sd = i % SD;
      const uint32_t ph = (i / SD) & 1;
      bool w = mbar_wait(&sums_full[sd], ph, 0x2B);
      if (w) w = mbar_wait(&d_full[sd], ph, 0x25);
      if (!__all_sync(0xffffffffu, w)) break;
      sg_tc_fence_after();
      const float* sums = reinterpret_cast<const float*>(smem + C::OFF_SUM + sd * C::SUM);
      const uint32_t* scal = reinterpret_cast<const uint32_t*>(smem + C::OFF_SCAL + sd * C::SCAL);
      const uint32_t scw = scal[row];
      float sc[2], of[2];
      if (DT == SG_DTYPE_Q4_0) {
        const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&scw));
        sc[0] = d.x;
        sc[1] = d.y;
        of[0] = of[1] = 0.f;
      } else {
        const uint32_t ddw = scal[128 + row];
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&ddw));
        sc[0] = dm.x * (float)(scw & 0xFFu);
        sc[1] = dm.x * (float)((scw >> 8) & 0xFFu);
        of[0] = dm.y * (float)((scw >> 16) & 0xFFu);
        of[1] = dm.y * (float)(scw >> 24);
      }
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((sd * 2 + blk) * C::N);
        float v[C::N];
        if constexpr (C::N == 16) {
          uint32_t rr[16];
          sg_tmem_ld16(taddr, rr);
          sg_tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = __uint_as_float(rr[k]);
        } else {
          uint32_t rr[32];
          sg_tmem_ld32(taddr, rr);
          sg_tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(rr[k]);
        }
        const float* s0 = sums + blk * 32;
#pragma unroll
        for (int t = 0; t < BP; ++t) {
          const float dot = (v[t] + v[BP + t]) - s0[t];
          if (DT == SG_DTYPE_Q4_0) acc[t] = fmaf(sc[blk], dot, acc[t]);
          else acc[t] = fmaf(sc[blk], dot, fmaf(-of[blk], s0[16 + t], acc[t]));
        }
      }
      sg_tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[sd]);
      // row-block segment finished: store it whole, or reduce it
      const bool rb_end = cur.c == p.n_ch - 1;
      if (rb_end || i == n - 1) {
        if (!waited_prev) {
          pdl_wait();  // y: zeroing by the prep kernel, readers of the previous kernel
          waited_prev = true;
        }
        const Mat& mt = p.mats[cur.mi];
        const int grow = cur.rb * 128 + row;
        const bool whole = rb_end && seg_whole_start;
        if (grow < mt.n_rows) {
#pragma unroll
          for (int t = 0; t < BP; ++t) {
            if (t < p.batch) {
              float* yp = mt.y + (int64_t)t * mt.ldy + grow;
              const float val = acc[t] * p.inv[t];
              if (!whole) red_add_f32(yp, val);
              else *yp = p.accumulate ? *yp + val : val;
            }
          }
        }
#pragma unroll
        for (int t = 0; t < BP; ++t) acc[t] = 0.f;
        seg_whole_start = true;  // the next segment starts at chunk 0 of its row-block
      }
      cur.next(p);
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
  __half* xh;
  __half* xl;
  float* sums;
  float* inv;
  size_t bytes;
};

Layout layout_of(void* base, int64_t K) {
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const int64_t n_ch = (K + 63) / 64;
  Layout l;
  uint8_t* b = static_cast<uint8_t*>(base);
  const size_t xb = up((size_t)SG_GEMV_MAX_BATCH * K * 2);
  const size_t sb = up((size_t)2 * n_ch * 2 * 16 * 4);
  l.xh = reinterpret_cast<__half*>(b);
  l.xl = reinterpret_cast<__half*>(b + xb);
  l.sums = reinterpret_cast<float*>(b + 2 * xb);
  l.inv = reinterpret_cast<float*>(b + 2 * xb + sb);
  l.bytes = 2 * xb + sb + 256;
  return l;
}

template <int DT, int BP>
cudaError_t launch_gemv(int G, const Params& p, cudaStream_t st, cudaLaunchAttribute* attr) {
  using C = Cfg<BP>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<DT, BP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_done[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<DT, BP>, p);
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
  p.accumulate = accumulate ? 1 : 0;
  int rb = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->n_cols != K || w->dtype != w0->dtype || !mats[i].y || mats[i].ldy < w->n_rows) return cudaErrorInvalidValue;
    p.mats[i] = {w->tiles, w->dd, mats[i].y, mats[i].ldy, (int)w->n_rb, (int)w->n_rows, (int)w->n_sb, rb};
    rb += (int)w->n_rb;
  }
  p.total = (int64_t)rb * p.n_ch;
  const Layout l = layout_of(scratch, K);
  p.sums = l.sums;
  p.inv = l.inv;
  p.xh = l.xh;
  p.xl = l.xl;
  p.K = (int)K;
  // two CTAs per SM, at least two chunks each
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(2LL * num_sms, p.total / 2));
  p.total_rb = rb;
  p.zero_all = rb > kMaskWords * 32;
  bool split = false;
  for (int c = 1; c < G; ++c) {
    const int64_t gi = (int64_t)c * p.total / G;
    if (gi % p.n_ch == 0) continue;
    split = true;
    const int64_t r = gi / p.n_ch;
    if (r < kMaskWords * 32) p.split[r >> 5] |= 1u << (r & 31);
  }

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((2 * p.n_ch + 7) / 8), (unsigned)batch);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_xprep_kernel, x, ldx, (int)K, 2 * p.n_ch,
                                     w0->dtype == SG_DTYPE_Q4_0 ? 1 : 0, l.xh, l.xl, l.sums, l.inv, p,
                                     (split && !accumulate) ? 1 : 0);
  if (e != cudaSuccess) return e;

  const int BP = batch <= 8 ? 8 : 16;
  if (w0->dtype == SG_DTYPE_Q4_0)
    return BP == 8 ? launch_gemv<SG_DTYPE_Q4_0, 8>(G, p, st, attr) : launch_gemv<SG_DTYPE_Q4_0, 16>(G, p, st, attr);
  return BP == 8 ? launch_gemv<SG_DTYPE_Q4_K, 8>(G, p, st, attr) : launch_gemv<SG_DTYPE_Q4_K, 16>(G, p, st, attr);
}
