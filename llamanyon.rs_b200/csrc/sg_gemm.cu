// sg_gemm.cu -- prefill GEMM (batch > 16 tokens) for Q4_0 / Q4_K on B200:
// tcgen05 tensor cores with the accumulator in TMEM, activations fed by TMA.
//
// Replaces swamp-kernels fused_gemv_q4k_batched (fused_gemv_q4k.rs:527-698),
// which the engine's prefill issues through forward_linear_batch
// (swamp-engine/src/linear.rs:176-239, executor.rs:106-181):
//   y[t][r] = sum_k W[r][k] x[t][k],  W dequantized as swamp-gguf does.
//
// Precision: the reference computes in f32. A Q4_K weight needs up to 24
// significant bits and an activation 24, neither fits one 16-bit operand, and
// a single bf16 product errs by ~2^-9 -- far outside the 1e-3 parity bound. So
// both operands are split into bf16 hi + lo parts and every k-step runs three
// MMAs: A_hi*X_hi + A_hi*X_lo + A_lo*X_hi (A_lo*X_lo is ~2^-16 relative and
// dropped), all accumulating in f32 in TMEM. The weight split truncates (hi =
// top 16 bits of the f32, lo = the exact remainder rounded to bf16: error
// <= 2^-15 relative); the activation split rounds.
//
// Two kernels, chained with programmatic dependent launch:
//  1. gemm_xprep_kernel: x (f32) -> X_hi, X_lo (bf16, [m][K]) in scratch;
//     zeroes the output tiles that more than one CTA reduces into.
//  2. gemm_kernel: persistent, one CTA per SM. Work = tiles of 128 weight
//     rows x 256 tokens, each a run of 64-wide K chunks. Whole tiles are dealt
//     round-robin (data parallel); the tiles left over are cut into equal
//     chunk ranges across all CTAs (stream-K), so every SM gets the same work.
//     warp 0     producer: TMA 2-D loads of X_hi/X_lo tiles (32 K x 256
//                tokens, 64-byte swizzle) and bulk copies of the packed
//                weight tiles (4.5 KB per 128 x 64, + Q4_K d|dmin).
//     warp 1     allocates 512 TMEM columns (two 128 x 256 f32
//                accumulators); one thread issues tcgen05.mma (M=128, N=256,
//                K=16, bf16 -> f32) and tcgen05.commit.
//     warps 2-5, 10-13  dequantize, two sets taking the two K halves of each
//                chunk: one weight row per thread, 32 K per stage, exact f32
//                via FMA from the f16 magic-number decode, split into bf16
//                hi/lo, 16-byte stores into the swizzled A tiles.
//     warps 6-9  epilogue: tcgen05.ld of the finished accumulator (while the
//                MMAs fill the other one), stores -- or red.add for a tile
//                shared with another CTA.
//  Four 48 KB stages (A_hi, A_lo, X_hi, X_lo) + a 3-chunk raw weight ring.
//  Every mbarrier wait is bounded (sg_common.cuh).
#include <algorithm>

#include "sg_gemm.cuh"
#include "sg_tc.cuh"

namespace gemm_tc {

constexpr int BM = 128, BN = 256, BK = 32;
constexpr int kS = 4;  // MMA stages
constexpr int kR = 3;  // raw weight chunk ring
constexpr int A_BYTES = BM * BK * 2;  // 8 KB
constexpr int X_BYTES = BN * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * X_BYTES;
constexpr int RAW_BYTES = SG_TILE6_BYTES + 512;  // the largest tile (Q6_K) + its d / d|dmin words
constexpr int SMEM_BYTES = kS * STAGE_BYTES + kR * RAW_BYTES + 1024;  // + alignment slack
constexpr int kThreads = 448;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdesc = sg_idesc_bf16(BM, BN);

struct GemmParams {
  const uint8_t* tiles;
  const uint32_t* dd;
  int dtype;
  int n_rows, n_ch, n_sb;
  int m;      // tokens
  int n_tt;   // token tiles
  int dp;     // whole tiles per CTA (data-parallel rounds)
  int64_t rem_iters;  // chunk iterations of the leftover tiles, shared by all CTAs
  int accumulate;
  float* y;
  int64_t ldy;
};

// The CTA's work as a sequence of segments (tile, chunk range). Every warp
// walks the same sequence.
template <typename F>
__device__ __forceinline__ void for_each_segment(const GemmParams& p, F&& f) {
  const int G = gridDim.x, c = blockIdx.x;
  for (int s = 0; s < p.dp; ++s) f(c + s * G, 0, p.n_ch);
  const int base = p.dp * G;
  const int64_t it0 = (int64_t)c * p.rem_iters / G, it1 = (int64_t)(c + 1) * p.rem_iters / G;
  for (int64_t it = it0; it < it1;) {
    const int tile = base + (int)(it / p.n_ch);
    const int k0 = (int)(it % p.n_ch);
    const int64_t left = it1 - it;
    const int k1 = left < (int64_t)(p.n_ch - k0) ? k0 + (int)left : p.n_ch;
    f(tile, k0, k1);
    it += k1 - k0;
  }
}

// ---------------------------------------------------------------- x prep
__global__ void __launch_bounds__(256) gemm_xprep_kernel(const float* __restrict__ x, int64_t ldx, int m, int K,
                                                          __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl,
                                                          GemmParams p, int G) {
  pdl_launch_dependents();
  pdl_wait();  // scratch / y may still be in use by the previous kernel
  const int64_t n8 = (int64_t)m * (K / 8);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const int64_t t = i / (K / 8);
    const int k = (int)(i - t * (K / 8)) * 8;
    const float4 a = *reinterpret_cast<const float4*>(x + t * ldx + k);
    const float4 b = *reinterpret_cast<const float4*>(x + t * ldx + k + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      const float2 hf = __bfloat1622float2(h);
      const __nv_bfloat162 l = __floats2bfloat162_rn(v[2 * j] - hf.x, v[2 * j + 1] - hf.y);
      hw[j] = *reinterpret_cast<const uint32_t*>(&h);
      lw[j] = *reinterpret_cast<const uint32_t*>(&l);
    }
    *reinterpret_cast<uint4*>(xh + t * K + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(xl + t * K + k) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  // zero the tiles that a stream-K boundary cuts (reduced with red.add):
  // one warp per (boundary, 32-token slice of the tile); a tile that several
  // boundaries cut is zeroed by the first of them only
  if (!p.accumulate && p.rem_iters > 0) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarp = stride >> 5;
    const int64_t tot = (int64_t)(G - 1) * (BN / 32);
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < tot; i += nwarp) {
      const int cb = 1 + (int)(i / (BN / 32)), ts = (int)(i % (BN / 32));
      const int64_t it = (int64_t)cb * p.rem_iters / G;
      if (it % p.n_ch == 0) continue;
      if (cb > 1) {
        const int64_t prev = (int64_t)(cb - 1) * p.rem_iters / G;
        if (prev % p.n_ch != 0 && prev / p.n_ch == it / p.n_ch) continue;  // an earlier boundary cuts this tile
      }
      const int tile = p.dp * G + (int)(it / p.n_ch);
      const int rb = tile / p.n_tt, tt = tile % p.n_tt;
      const int nr = min(BM, p.n_rows - rb * BM);
      for (int j = 0; j < 32; ++j) {
        const int tok = tt * BN + ts * 32 + j;
        if (tok >= p.m) break;
        float* yr = p.y + (int64_t)tok * p.ldy + (int64_t)rb * BM;
        for (int r = lane; r < nr; r += 32) yr[r] = 0.f;
      }
    }
  }
}

// byte offset of the 16-byte chunk j (8 K) of row r in a K-major
// 64-byte-swizzled tile (rows of 32 elements, 8-row atoms of 512 B)
__device__ __forceinline__ uint32_t sw64_chunk(int r, int j) {
  return (uint32_t)((r >> 3) * 512 + (r & 7) * 64 + (((j ^ (r >> 1)) & 3) << 4));
}

// ---------------------------------------------------------------- GEMM
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t x_full[kS], a_full[kS], s_empty[kS], raw_full[kR], raw_empty[kR], acc_full[2],
      acc_empty[2];
  __shared__ uint32_t tmem_base_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* raw_ring = smem + kS * STAGE_BYTES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&a_full[s], 4);
      mbar_init(&s_empty[s], 1);
    }
    for (int r = 0; r < kR; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], 8);  // both dequant sets
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_fence_init();
    prefetch_tensormap(&map_hi);
    prefetch_tensormap(&map_lo);
  }
  if (warp == 1) sg_tmem_alloc(&tmem_base_sh, kTmemCols);
  sg_tc_fence_before();
  __syncthreads();
  sg_tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0) {
      pdl_wait();  // X_hi/X_lo come from the activation-prep kernel
      int g = 0, rc = 0;  // k-step and raw-chunk counters
      bool ok = true;
      for_each_segment(p, [&](int tile, int k0, int k1) {
        if (!ok) return;
        const int rb = tile / p.n_tt, tt = tile % p.n_tt;
        for (int ch = k0; ch < k1 && ok; ++ch) {
          const int r = rc % kR;
          if (rc >= kR && !mbar_wait(&raw_empty[r], ((rc / kR) & 1) ^ 1, 0x12)) {
            ok = false;
            break;
          }
          uint8_t* rw = raw_ring + r * RAW_BYTES;
          const int tb = sg_tile_bytes(p.dtype);
          const bool has_dd = p.dtype != SG_DTYPE_Q4_0;
          mbar_arrive_expect_tx(&raw_full[r], tb + (has_dd ? 512 : 0));
          bulk_g2s(rw, p.tiles + ((int64_t)rb * p.n_ch + ch) * tb, tb, &raw_full[r]);
          if (has_dd)
            bulk_g2s(rw + tb, p.dd + ((int64_t)rb * p.n_sb + (ch >> 2)) * 128, 512, &raw_full[r]);
          ++rc;
          for (int h = 0; h < 2; ++h) {
            const int s = g % kS;
            if (g >= kS && !mbar_wait(&s_empty[s], ((g / kS) & 1) ^ 1, 0x11)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * STAGE_BYTES;
            mbar_arrive_expect_tx(&x_full[s], 2 * X_BYTES);
            tma_load_2d(st + 2 * A_BYTES, &map_hi, 64 * ch + BK * h, tt * BN, &x_full[s]);
            tma_load_2d(st + 2 * A_BYTES + X_BYTES, &map_lo, 64 * ch + BK * h, tt * BN, &x_full[s]);
            ++g;
          }
        }
      });
      if (*(volatile int*)&g_sg_error != 0) {
        // error path: let every copy still in flight land before the CTA exits
        // (each barrier has at most one phase outstanding)
        for (int j = max(0, g - kS); j < g; ++j) mbar_wait_drain(&x_full[j % kS], (j / kS) & 1);
        for (int j = max(0, rc - kR); j < rc; ++j) mbar_wait_drain(&raw_full[j % kR], (j / kR) & 1);
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      int g = 0, seg = 0;
      bool ok = true;
      for_each_segment(p, [&](int tile, int k0, int k1) {
        (void)tile;
        if (!ok) return;
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[b], ((seg >> 1) & 1) ^ 1, 0x18)) {
          ok = false;
          return;
        }
        sg_tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kk = 0; kk < 2 * (k1 - k0); ++kk) {
          const int s = g % kS;
          const uint32_t ph = (g / kS) & 1;
          if (!mbar_wait(&x_full[s], ph, 0x13) || !mbar_wait(&a_full[s], ph, 0x14)) {
            ok = false;
            break;
          }
          sg_tc_fence_after();
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t ah = sg_sdesc(base, SG_SW64), al = sg_sdesc(base + A_BYTES, SG_SW64);
          const uint64_t xh = sg_sdesc(base + 2 * A_BYTES, SG_SW64);
          const uint64_t xl = sg_sdesc(base + 2 * A_BYTES + X_BYTES, SG_SW64);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t o = (uint64_t)(j * 2);  // K step of 16 bf16 = 32 bytes
            sg_umma(d, ah + o, xh + o, kIdesc, (kk | j) ? 1u : 0u);
            sg_umma(d, ah + o, xl + o, kIdesc, 1u);
            sg_umma(d, al + o, xh + o, kIdesc, 1u);
          }
          sg_umma_commit(&s_empty[s]);
          ++g;
        }
        sg_umma_commit(&acc_full[b]);  // fires when this segment's MMAs have completed
        ++seg;
      });
      // every MMA issued must have completed before TMEM is freed: each k-step
      // ends with a commit, so the last one covers all (also on the error path)
      if (g > 0) mbar_wait_drain(&s_empty[(g - 1) % kS], ((g - 1) / kS) & 1);
    }
  } else if (warp < 6 || warp >= 10) {
    // ====================================================== dequant warps
    // two sets of four (warps 2-5 and 10-13); set s converts the K half h == s
    // of every chunk, so two stages are converted at once
    const int dset = warp < 6 ? 0 : 1;
    const int row = (warp & 3) * 32 + lane;
    int g = 0, rc = 0;
    bool ok = true;
    for_each_segment(p, [&](int tile, int k0, int k1) {
      (void)tile;
      if (!ok) return;
      for (int ch = k0; ch < k1 && ok; ++ch, ++rc) {
        const int r = rc % kR;
        const uint8_t* rw = raw_ring + r * RAW_BYTES;
        for (int h = 0; h < 2; ++h) {
          if (h != dset) {
            ++g;
            continue;
          }
          const int s = g % kS;
          bool w = mbar_wait(&raw_full[r], (rc / kR) & 1, 0x15);
          if (w && g >= kS) w = mbar_wait(&s_empty[s], ((g / kS) & 1) ^ 1, 0x16);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          const uint4 nv = *reinterpret_cast<const uint4*>(rw + h * 2048 + row * 16);
          uint8_t* a_hi = smem + s * STAGE_BYTES;
          uint8_t* a_lo = a_hi + A_BYTES;
          if (p.dtype == SG_DTYPE_Q6_K) {
            // w = (d * sc) * (q - 32), both products exact (q6_k.rs:37-46);
            // q = low nibble | high 2 bits << 4, set side by side by masks
            const uint2 hq = *reinterpret_cast<const uint2*>(rw + SG_TILE6_HI_OFF + (h * 128 + row) * 8);
            const uint32_t scw6 = *reinterpret_cast<const uint32_t*>(rw + SG_TILE6_SC_OFF + row * 4);
            const float d6 = __half2float(
                __ushort_as_half((unsigned short)(*reinterpret_cast<const uint32_t*>(rw + SG_TILE6_BYTES + row * 4) & 0xFFFFu)));
            const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t H = j < 2 ? hq.x : hq.y;
              const uint32_t qa = (nw[j] & 0x0F0F0F0Fu) | (((j & 1) ? H : (H << 4)) & 0x30303030u);
              const uint32_t qb = ((nw[j] >> 4) & 0x0F0F0F0Fu) | (((j & 1) ? (H >> 2) : (H << 2)) & 0x30303030u);
              // K order 0..7: bytes (qa0, qa2, qb0, qb2, qa1, qa3, qb1, qb3)
              const uint32_t sel[8] = {0x7650u, 0x7652u, 0x7650u, 0x7652u, 0x7651u, 0x7653u, 0x7651u, 0x7653u};
              float qv[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                qv[e] = __uint_as_float(__byte_perm((e & 2) ? qb : qa, 0x4B000000u, sel[e])) - 8388640.f;
              const float sw = __fmul_rn(d6, (float)(int8_t)(scw6 >> (8 * (2 * h + (j >> 1)))));
              uint32_t hi[4], lo[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float w0 = __fmul_rn(sw, qv[2 * e]), w1 = __fmul_rn(sw, qv[2 * e + 1]);
                const uint32_t u0 = __float_as_uint(w0), u1 = __float_as_uint(w1);
                hi[e] = __byte_perm(u0, u1, 0x7632);
                const __nv_bfloat162 l = __floats2bfloat162_rn(w0 - __uint_as_float(u0 & 0xFFFF0000u),
                                                               w1 - __uint_as_float(u1 & 0xFFFF0000u));
                lo[e] = *reinterpret_cast<const uint32_t*>(&l);
              }
              const uint32_t off = sw64_chunk(row, j);
              *reinterpret_cast<uint4*>(a_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
              *reinterpret_cast<uint4*>(a_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
          } else {
            const uint32_t scw = *reinterpret_cast<const uint32_t*>(rw + SG_TILE_SC_OFF + row * 4);
            float sv, mv;  // w = sv*q - mv
            if (p.dtype == SG_DTYPE_Q4_0) {
              sv = __half2float(__ushort_as_half((unsigned short)(h ? (scw >> 16) : (scw & 0xFFFFu))));
              mv = 8.f * sv;
            } else {
              const uint32_t ddw = *reinterpret_cast<const uint32_t*>(rw + SG_TILE_BYTES + row * 4);
              const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&ddw));
              sv = __fmul_rn(dm.x, (float)((scw >> (8 * h)) & 0xFFu));
              mv = __fmul_rn(dm.y, (float)((scw >> (16 + 8 * h)) & 0xFFu));
            }
            // f = 1024+q (k%8 in {0,1,4,5}) or 1024+16q ({2,3,6,7}):
            //   w = f*sv - (1024 sv + mv)   or   w = f*(sv/16) - (64 sv + mv)
            const float mulA = sv, addA = -__fadd_rn(1024.f * sv, mv);
            const float mulB = sv * 0.0625f, addB = -__fadd_rn(64.f * sv, mv);
            const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
  #pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 f16 = sg_decode_word_f16(nw[j]);
              const uint32_t fp[4] = {f16.x, f16.y, f16.z, f16.w};
              uint32_t hi[4], lo[4];
  #pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&fp[e]));
                const float mul = (e & 1) ? mulB : mulA, add = (e & 1) ? addB : addA;
                const float w0 = fmaf(f.x, mul, add), w1 = fmaf(f.y, mul, add);
                const uint32_t u0 = __float_as_uint(w0), u1 = __float_as_uint(w1);
                hi[e] = __byte_perm(u0, u1, 0x7632);  // truncated bf16 pair (top halves)
                const __nv_bfloat162 l = __floats2bfloat162_rn(w0 - __uint_as_float(u0 & 0xFFFF0000u),
                                                               w1 - __uint_as_float(u1 & 0xFFFF0000u));
                lo[e] = *reinterpret_cast<const uint32_t*>(&l);
              }
              const uint32_t off = sw64_chunk(row, j);
              *reinterpret_cast<uint4*>(a_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
              *reinterpret_cast<uint4*>(a_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
          }
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&a_full[s]);
            mbar_arrive(&raw_empty[r]);
          }
          ++g;
        }
      }
    });
  } else {
    // ============================================================ epilogue warps
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    const int row_l = quad * 32 + lane;
    int seg = 0;
    bool ok = true;
    bool waited = false;
    for_each_segment(p, [&](int tile, int k0, int k1) {
      if (!ok) return;
      const int b = seg & 1;
      const bool w = mbar_wait(&acc_full[b], (seg >> 1) & 1, 0x17);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        return;
      }
      sg_tc_fence_after();
      if (!waited) {
        pdl_wait();  // y: zeroing by the prep kernel, readers of the previous kernel
        waited = true;
      }
      const int rb = tile / p.n_tt, tt = tile % p.n_tt;
      const int row = rb * BM + row_l;
      const bool whole = (k0 == 0 && k1 == p.n_ch);
#pragma unroll 1
      for (int cb = 0; cb < BN / 32; ++cb) {
        uint32_t v[32];
        sg_tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BN + cb * 32), v);
        sg_tmem_ld_wait();
        if (row < p.n_rows) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int tok = tt * BN + cb * 32 + j;
            if (tok < p.m) {
              float* yp = p.y + (int64_t)tok * p.ldy + row;
              const float val = __uint_as_float(v[j]);
              if (!whole) red_add_f32(yp, val);
              else *yp = p.accumulate ? *yp + val : val;
            }
          }
        }
      }
      sg_tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      ++seg;
    });
  }
  pdl_launch_dependents();
  sg_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sg_tc_fence_after();
    sg_tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------ host side
cudaError_t set_gemm_attr() {
  static uint64_t done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && ((done_mask >> dev) & 1)) return cudaSuccess;
  e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess && dev < 64) done_mask |= (1ull << dev);
  return e;
}

cudaError_t launch(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int m, bool accumulate,
                   void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  if (m < 1 || !w || !x || !y) return cudaErrorInvalidValue;
  const int64_t K = w->n_cols;
  if ((K & 31) || ((uintptr_t)x & 15) || (ldx & 3) || ldx < K || K > (1 << 30) || (int64_t)m * K > (1ll << 40) ||
      ldy < w->n_rows)
    return cudaErrorInvalidValue;
  if (scratch_bytes < sg_gemm_scratch_bytes(m, K)) return cudaErrorInvalidValue;
  __nv_bfloat16* xh = static_cast<__nv_bfloat16*>(scratch);
  __nv_bfloat16* xl = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(scratch) +
                                                        ((((size_t)m * K * 2) + 255) & ~(size_t)255));
  GemmParams p = {};
  p.tiles = w->tiles;
  p.dd = w->dd;
  p.dtype = w->dtype;
  p.n_rows = (int)w->n_rows;
  p.n_ch = (int)w->n_ch;
  p.n_sb = (int)w->n_sb;
  p.m = m;
  p.n_tt = (m + BN - 1) / BN;
  p.accumulate = accumulate ? 1 : 0;
  p.y = y;
  p.ldy = ldy;
  const int64_t tiles = w->n_rb * p.n_tt;
  // persistent grid: one CTA per SM (at least one chunk each)
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms, tiles * p.n_ch));
  p.dp = (int)(tiles / G);
  p.rem_iters = (tiles - (int64_t)p.dp * G) * p.n_ch;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  const int64_t n8 = (int64_t)m * (K / 8);
  cfg.gridDim = dim3((unsigned)std::min<int64_t>((n8 + 255) / 256, (int64_t)num_sms * 8));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_xprep_kernel, x, ldx, m, (int)K, xh, xl, p, G);
  if (e != cudaSuccess) return e;

  CUtensorMap mh, ml;
  if (!sg_make_map_16(&mh, xh, m, K, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B, false) ||
      !sg_make_map_16(&ml, xl, m, K, BK, BN, CU_TENSOR_MAP_SWIZZLE_64B, false))
    return cudaErrorInvalidValue;
  e = set_gemm_attr();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)G);
  g.blockDim = dim3(kThreads);
  g.dynamicSmemBytes = SMEM_BYTES;
  g.stream = st;
  g.attrs = attr;
  g.numAttrs = 1;
  return cudaLaunchKernelEx(&g, gemm_kernel, mh, ml, p);
}

}  // namespace gemm_tc

size_t sg_gemm_scratch_bytes(int64_t m, int64_t n_cols) {
  return 2 * (((size_t)m * (size_t)n_cols * 2 + 255) & ~(size_t)255);
}

cudaError_t sg_gemm(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int m, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  return gemm_tc::launch(w, x, ldx, y, ldy, m, accumulate, scratch, scratch_bytes, num_sms, st);
}
