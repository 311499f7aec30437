// sg_gemv.cu -- decode GEMV (batch 1..16) for Q4_0 / Q4_K on B200.
//
// Replaces the reference's CPU GEMVs: swamp-kernels fused_gemv_q4k
// (fused_gemv_q4k.rs:59-82, scalar body :466-508), its batched form
// (:527-698) and the engine's Q4_0 route (swamp-engine/src/linear.rs:68-87).
// out[b][r] = sum_k W[r][k] * x[b][k], W dequantized exactly as swamp-gguf.
//
// One kernel per call (up to 4 matrices sharing x in one launch). The grid is
// (row-block of 128 rows) x (split K slices), sized to one wave of 4 CTAs per
// SM; the `split` CTAs of a row-block form one thread-block cluster.
//
//  * Each of the 4 warps owns two 16-row tiles of the row-block and streams
//    its K slice with 128-bit loads straight into registers (16 B of nibbles
//    + the scales per tile per 64-wide chunk per lane), prefetched 4 chunks
//    ahead. The first prefetches are issued before griddepcontrol.wait:
//    weights never depend on the previous kernel, so they stream while that
//    kernel drains.
//  * After the wait, the CTA splits its K slice of x exactly into bf16 hi + lo
//    (16 significant bits, full f32 range) in shared memory, laid out as
//    m16n8k16 B fragments. Batch <= 4: one n-tile whose column 2b holds
//    x_hi[b] and 2b+1 x_lo[b] (one mma per k-step); batch 5..16: n-tiles of 8
//    batch columns with separate hi and lo fragments accumulated into the
//    same f32 partial (half the epilogue work of interleaving).
//  * Nibbles decode into bf16 A fragments (shift + lop3 + one bf16x2 fma per
//    pair; q-8 / q are exact in bf16). Per 32-element block, mma.sync
//    accumulates in f32; the block partial is scaled in f32 by d (Q4_0) or
//    d*sc minus the min term dmin*m*sum(x) (Q4_K).
//  * The cluster's K-slice partials are summed on chip through distributed
//    shared memory (each CTA reduces a fixed share of the rows in rank order,
//    so results are reproducible) and written to y. No global scratch, no
//    atomics and no spin-waits: the only synchronisation is __syncthreads and
//    the hardware cluster barrier, which every thread of the cluster reaches.
#include <algorithm>

#include "sg_gemv.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCtasPerSm = 4;
constexpr int kMaxSmem = 55 * 1024;        // fits 4 CTAs per SM
constexpr int kMaxSmemLarge = 110 * 1024;  // hard limit (2 CTAs per SM)

// MODE 0: batch <= 4, [hi|lo] interleaved columns, 1 n-tile
// MODE 1: batch <= 8, hi and lo fragments, 1 n-tile of 8 batches
// MODE 2: batch <= 16, hi and lo fragments, 2 n-tiles
template <int MODE>
struct Frag {
  static constexpr int nt = MODE == 2 ? 2 : 1;        // n-tiles
  static constexpr int nfr = MODE == 0 ? 1 : 2;       // fragments per n-tile (hi, lo)
  static constexpr int chunk_bytes = 4 * nt * nfr * 256;  // per 64-wide chunk
  static constexpr int ncol = MODE == 0 ? 4 : 8 * nt;     // batch columns covered
};

// One packed word -> the four bf16x2 A-fragment registers of m16n8k16 as raw
// magic values: 128+q on rows g (fragment registers 0, 2) and 128+8q on rows
// g+8 (registers 1, 3), both exact in bf16. The kernel removes the 128 (and
// the Q4_0 bias of 8) in the f32 epilogue with the block sum of x.
__device__ __forceinline__ void decode_frag_raw(uint32_t w, uint32_t a[4]) {
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);
  a[1] = lop3_and_or(w >> 1, 0x00780078u, 0x43004300u);
  a[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
  a[3] = lop3_and_or(w >> 9, 0x00780078u, 0x43004300u);
}

__device__ __forceinline__ void mma_bf16(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                         const float z[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z[0]), "f"(z[1]), "f"(z[2]), "f"(z[3]));
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(const float* local, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Per-warp weight ring: each warp streams its two row-tiles' share of every
// chunk (1 KB of nibbles, 128 B of scales, Q4_K also 128 B of d|dmin) with
// cp.async.bulk into a private ring of kStages stages; a stage is refilled by
// the same warp right after it consumed it, so no warp ever waits on another.
constexpr int kStages = 6;
template <int DT>
struct Ring {
  static constexpr int nib = 1024, sc = 128, dd = DT == SG_DTYPE_Q4_K ? 128 : 0;
  static constexpr int stage = nib + sc + dd;
  static constexpr int warp_bytes = kStages * stage;
  static constexpr int bytes = kWarps * warp_bytes;
};

template <int DT>
__device__ __forceinline__ void issue_chunk(uint8_t* st, const uint8_t* tile, const uint32_t* dd_src, int warp,
                                            uint64_t* bar, uint64_t pol) {
  using R = Ring<DT>;
  mbar_arrive_expect_tx(bar, R::stage);
  bulk_g2s_evict_first(st, tile + warp * 1024, R::nib, bar, pol);
  bulk_g2s_evict_first(st + R::nib, tile + SG_TILE_SC_OFF + warp * 128, R::sc, bar, pol);
  if (DT == SG_DTYPE_Q4_K) bulk_g2s(st + R::nib + R::sc, dd_src + warp * 32, R::dd, bar);
}

// x (this CTA's chunks [c0, c0+nc)) -> bf16 hi/lo B fragments in smem, plus
// the per-32 sums of x (of the hi+lo parts the mma sees) for the epilogue.
template <int DT, int MODE>
__device__ __forceinline__ void prepare_x(const SgGemvParams& p, int c0, int nc, uint8_t* smem) {
  using F = Frag<MODE>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // zero the fragments and sums (columns past the batch must read as 0)
  uint4* z = reinterpret_cast<uint4*>(smem);
  const int nz = nc * (F::chunk_bytes + 128) / 16;
  for (int i = threadIdx.x; i < nz; i += kThreads) z[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  uint32_t* xf = reinterpret_cast<uint32_t*>(smem);
  float* xs = reinterpret_cast<float*>(smem + (size_t)nc * F::chunk_bytes);
  const int s4 = lane >> 3, tt = lane & 3, half = (lane >> 2) & 1;
  const int items = nc * p.batch;  // (chunk, live column), one warp each
  for (int it = warp; it < items; it += kWarps) {
    const int i = it / p.batch, b = it - i * p.batch;
    const int k = 64 * (c0 + i) + 2 * lane;
    float2 v = make_float2(0.f, 0.f);
    if (k < p.n_cols) v = *reinterpret_cast<const float2*>(p.x + (int64_t)b * p.ldx + k);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(v.x, v.y);
    const float2 hf = __bfloat1622float2(hi);
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x - hf.x, v.y - hf.y);
    const uint32_t hiw = *reinterpret_cast<const uint32_t*>(&hi), low = *reinterpret_cast<const uint32_t*>(&lo);
    uint32_t* cf = xf + (size_t)i * (F::chunk_bytes / 4);
    if (MODE == 0) {
      // [s4][lane] uint2; column g = 2b (hi) / 2b+1 (lo)
      cf[(s4 * 32 + 4 * (2 * b) + tt) * 2 + half] = hiw;
      cf[(s4 * 32 + 4 * (2 * b + 1) + tt) * 2 + half] = low;
    } else {
      // [s4][nn][hl][lane] uint2; column g = b % 8 of n-tile b / 8
      const int nn = b >> 3, gg = b & 7;
      uint32_t* e = cf + (((s4 * F::nt + nn) * 2) * 32 + 4 * gg + tt) * 2 + half;
      e[0] = hiw;
      e[64] = low;
    }
    {
      const float2 lf = __bfloat1622float2(lo);
      float sum = (hf.x + lf.x) + (hf.y + lf.y);
#pragma unroll
      for (int o = 8; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if ((lane & 15) == 0) xs[(i * 2 + (lane >> 4)) * 16 + b] = sum;
    }
  }
}

template <int DT, int MODE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(SgGemvParams p) {
  using F = Frag<MODE>;
  constexpr int NT = F::nt;
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int split = p.split;
  const int rbg = blockIdx.x / split, ks = blockIdx.x - rbg * split;
  int m = 0;
#pragma unroll
  for (int i = 1; i < SG_GEMV_MAX_MATS; ++i)
    if (i < p.n_mats && rbg >= p.mats[i].rb0) m = i;
  const SgGemvMatP& M = p.mats[m];
  const int rb = rbg - M.rb0;
  const int c0 = (int)((int64_t)ks * p.n_ch / split), c1 = (int)((int64_t)(ks + 1) * p.n_ch / split);
  const int nc = c1 - c0;
  const uint8_t* tb = M.tiles + ((int64_t)rb * p.n_ch + c0) * SG_TILE_BYTES;
  // dd of (row-block, super-block) for this chunk: [rt 8][g 8][hl 2] words
  const uint32_t* ddb = DT == SG_DTYPE_Q4_K ? M.dd + (int64_t)rb * M.n_sb * 128 : nullptr;
  using R = Ring<DT>;
  const size_t xbytes = (size_t)nc * (F::chunk_bytes + 128);
  const size_t ring_off = (xbytes + 127) & ~(size_t)127;
  uint8_t* ring = smem + ring_off + (size_t)warp * R::warp_bytes;
  __shared__ __align__(8) uint64_t wbar[kWarps][kStages];
  uint64_t* bars = wbar[warp];
  const uint64_t pol = policy_evict_first();
  // weights do not depend on the previous kernel: start streaming them now
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    for (int d = 0; d < kStages && d < nc; ++d)
      issue_chunk<DT>(ring + d * R::stage, tb + (int64_t)d * SG_TILE_BYTES, ddb + ((c0 + d) >> 2) * 128, warp, &bars[d],
                      pol);
  }
  __syncwarp();
  pdl_wait();
  prepare_x<DT, MODE>(p, c0, nc, smem);
  __syncthreads();
  const float* xs = reinterpret_cast<const float*>(smem + (size_t)nc * F::chunk_bytes);

  // ---- stream the K slice
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  float acc[2][NT][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int nn = 0; nn < NT; ++nn)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][nn][j] = 0.f;
  const uint2* xfr2 = reinterpret_cast<const uint2*>(smem);

  bool ok = true;
  int issued = nc < kStages ? nc : kStages;
  int i = 0;
  for (; i < nc; ++i) {
    {
      {
        const int slot = i % kStages;
        // every lane acquires the stage; the vote keeps the warp converged even
        // if one lane's bounded wait gave up
        const bool lane_ok = mbar_wait(&bars[slot], (i / kStages) & 1, 6);
        if (!__all_sync(0xffffffffu, lane_ok)) {
          ok = false;
          break;
        }
        const uint8_t* st = ring + slot * R::stage;
        struct {
          uint4 q[2];
          uint2 sc[2];
          uint2 dd[2];
        } cur;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          cur.q[r] = *reinterpret_cast<const uint4*>(st + r * 512 + lane * 16);
          cur.sc[r] = *reinterpret_cast<const uint2*>(st + R::nib + r * 64 + g * 8);
          if (DT == SG_DTYPE_Q4_K) cur.dd[r] = *reinterpret_cast<const uint2*>(st + R::nib + R::sc + r * 64 + g * 8);
        }
        // the stage is in registers now: refill it with the chunk kStages ahead
        __syncwarp();
        if (i + kStages < nc) {
          if (lane == 0) {
            fence_proxy_async_smem();
            issue_chunk<DT>(ring + slot * R::stage, tb + (int64_t)(i + kStages) * SG_TILE_BYTES,
                            ddb + ((c0 + i + kStages) >> 2) * 128, warp, &bars[slot], pol);
          }
          ++issued;
        }
        // per (row-tile, 32-block, row half): acc += alpha * T - beta * S, where
        // T is the mma of the raw magic values (128+q on rows g, 128+8q on rows
        // g+8) and S the block's sum of x, so the bias never enters the decode
        float alpha[2][2][2], beta[2][2][2];  // [r][32-block][hl]
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (DT == SG_DTYPE_Q4_0) {
            const float2 d0 = __half22float2(*reinterpret_cast<const __half2*>(&cur.sc[r].x));
            const float2 d1 = __half22float2(*reinterpret_cast<const __half2*>(&cur.sc[r].y));
            const float dv[2][2] = {{d0.x, d0.y}, {d1.x, d1.y}};
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
              alpha[r][blk][0] = dv[blk][0];
              alpha[r][blk][1] = dv[blk][1] * 0.125f;
              beta[r][blk][0] = dv[blk][0] * 136.f;  // d * (128 + 8)
              beta[r][blk][1] = dv[blk][1] * 24.f;   // d * (128/8 + 8)
            }
          } else {
            const uint32_t scw[2] = {cur.sc[r].x, cur.sc[r].y};
            const uint32_t ddw[2] = {cur.dd[r].x, cur.dd[r].y};
#pragma unroll
            for (int hl = 0; hl < 2; ++hl) {
              const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&ddw[hl]));
#pragma unroll
              for (int sub = 0; sub < 2; ++sub) {
                const float sv = dm.x * (float)((scw[hl] >> (8 * sub)) & 0xFFu);
                const float mv = dm.y * (float)((scw[hl] >> (16 + 8 * sub)) & 0xFFu);
                alpha[r][sub][hl] = hl ? sv * 0.125f : sv;
                beta[r][sub][hl] = fmaf(sv, hl ? 16.f : 128.f, mv);
              }
            }
          }
        }
        const uint2* xfr = xfr2 + (size_t)i * (F::chunk_bytes / 8);
        float tmp[2][NT][4];
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
          uint2 bh[NT], bl[NT];
#pragma unroll
          for (int nn = 0; nn < NT; ++nn) {
            if (MODE == 0) {
              bh[nn] = xfr[s4 * 32 + lane];
            } else {
              bh[nn] = xfr[((s4 * NT + nn) * 2 + 0) * 32 + lane];
              bl[nn] = xfr[((s4 * NT + nn) * 2 + 1) * 32 + lane];
            }
          }
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint32_t w = s4 == 0 ? cur.q[r].x : s4 == 1 ? cur.q[r].y : s4 == 2 ? cur.q[r].z : cur.q[r].w;
            uint32_t a[4];
            decode_frag_raw(w, a);
#pragma unroll
            for (int nn = 0; nn < NT; ++nn) {
              mma_bf16(tmp[r][nn], a, bh[nn].x, bh[nn].y, (s4 & 1) ? tmp[r][nn] : zero4);
              if (MODE != 0) mma_bf16(tmp[r][nn], a, bl[nn].x, bl[nn].y, tmp[r][nn]);
            }
          }
          if (s4 & 1) {
            const int blk = s4 >> 1;
#pragma unroll
            for (int nn = 0; nn < NT; ++nn) {
              // MODE 0: thread t owns batch t (hi col 2t, lo col 2t+1); others: batches 8nn+2t, +1
              float2 sx;
              if (MODE == 0) {
                sx.x = xs[(i * 2 + blk) * 16 + t];
                sx.y = 0.f;
              } else {
                sx = *reinterpret_cast<const float2*>(xs + (i * 2 + blk) * 16 + 8 * nn + 2 * t);
              }
#pragma unroll
              for (int r = 0; r < 2; ++r) {
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[r][nn][j] = fmaf(alpha[r][blk][j >> 1], tmp[r][nn][j], acc[r][nn][j]);
                // the S term applies once per batch column: the hi column only in MODE 0
                acc[r][nn][0] = fmaf(-beta[r][blk][0], sx.x, acc[r][nn][0]);
                acc[r][nn][2] = fmaf(-beta[r][blk][1], sx.x, acc[r][nn][2]);
                if (MODE != 0) {
                  acc[r][nn][1] = fmaf(-beta[r][blk][0], sx.y, acc[r][nn][1]);
                  acc[r][nn][3] = fmaf(-beta[r][blk][1], sx.y, acc[r][nn][3]);
                }
              }
            }
          }
        }
      }
    }
  }
  // a stage that timed out: wait (bounded) for the copies still in flight so
  // none lands after the CTA has exited
  if (!ok)
    for (int j = i; j < issued; ++j)
      if (!mbar_wait_drain(&bars[j % kStages], (j / kStages) & 1)) break;
  pdl_launch_dependents();

  // ---- results: value of (row-tile r, half hl, n-tile nn, column jc) and its batch
  auto out_val = [&](int r, int hl, int nn, int jc, int& b) -> float {
    if (MODE == 0) {
      b = t;  // jc selects hi/lo which are summed below
      return acc[r][nn][2 * hl] + acc[r][nn][2 * hl + 1];
    }
    b = 8 * nn + 2 * t + jc;
    return acc[r][nn][2 * hl + jc];
  };
  constexpr int NJC = MODE == 0 ? 1 : 2;
  if (split == 1) {
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int hl = 0; hl < 2; ++hl) {
        const int row = rb * 128 + (2 * warp + r) * 16 + g + 8 * hl;
        if (row < M.n_rows)
#pragma unroll
          for (int nn = 0; nn < NT; ++nn)
#pragma unroll
            for (int jc = 0; jc < NJC; ++jc) {
              int b;
              const float v = out_val(r, hl, nn, jc, b);
              if (b < p.batch) {
                float* yp = M.y + (int64_t)b * M.ldy + row;
                *yp = p.accumulate ? *yp + v : v;
              }
            }
      }
    return;
  }
  // split-K: partials through distributed shared memory, fixed rank order
  __syncthreads();  // every warp is done with the fragment area
  float* P = reinterpret_cast<float*>(smem);  // [128 rows][16 cols]
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int hl = 0; hl < 2; ++hl)
#pragma unroll
      for (int nn = 0; nn < NT; ++nn)
#pragma unroll
        for (int jc = 0; jc < NJC; ++jc) {
          int b;
          const float v = out_val(r, hl, nn, jc, b);
          P[((2 * warp + r) * 16 + g + 8 * hl) * 16 + b] = v;
        }
  cluster_sync_all();
  const int r0 = ks * 128 / split, r1 = (ks + 1) * 128 / split;
  const int nitems = (r1 - r0) * p.batch;
  for (int it = threadIdx.x; it < nitems; it += kThreads) {
    const int rl = r0 + it / p.batch, b = it % p.batch;
    float v = 0.f;
    for (int q = 0; q < split; ++q) v += ld_dsmem_f32(P + rl * 16 + b, q);
    const int row = rb * 128 + rl;
    if (row < M.n_rows) {
      float* yp = M.y + (int64_t)b * M.ldy + row;
      *yp = p.accumulate ? *yp + v : v;
    }
  }
  cluster_sync_all();  // keep this CTA's partials alive until the whole cluster has read them
}

template <int DT, int MODE>
size_t smem_bytes(int nc_max) {
  // [x fragments + per-32 sums][per-warp weight rings]; the split-K partials
  // (8 KB) reuse the front once the rings are drained
  const size_t frag = ((size_t)nc_max * (Frag<MODE>::chunk_bytes + 128) + 127) & ~(size_t)127;
  return std::max<size_t>(frag + Ring<DT>::bytes, 128 * 16 * sizeof(float));
}

// cudaFuncSetAttribute is per device; remember which devices are done.
template <int DT, int MODE>
cudaError_t set_attrs() {
  static uint64_t done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && ((done_mask >> dev) & 1)) return cudaSuccess;
  e = cudaFuncSetAttribute(gemv_kernel<DT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemLarge);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_kernel<DT, MODE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && dev < 64) done_mask |= (1ull << dev);
  return e;
}

template <int DT, int MODE>
cudaError_t launch(SgGemvParams& p, int total_rb, int num_sms, cudaStream_t st) {
  cudaError_t e = set_attrs<DT, MODE>();
  if (e != cudaSuccess) return e;
  // split: the most K slices per row-block that still fit one wave of CTAs,
  // keeping >= 2 chunks per slice and the fragments within the smem budget
  const int slots = num_sms * kCtasPerSm;
  int split = std::max(1, std::min(16, slots / std::max(1, total_rb)));
  split = std::min(split, std::max(1, p.n_ch / 2));
  while (split < 16 && smem_bytes<DT, MODE>((p.n_ch + split - 1) / split) > (size_t)kMaxSmem) ++split;
  // very long K at batch > 8 may still exceed the 4-CTA budget: run fewer CTAs per SM
  if (smem_bytes<DT, MODE>((p.n_ch + split - 1) / split) > (size_t)kMaxSmemLarge) return cudaErrorInvalidConfiguration;
  p.split = split;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(total_rb * split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<DT, MODE>((p.n_ch + split - 1) / split);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  ++na;
  if (split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = split;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<DT, MODE>, p);
}

template <int DT>
cudaError_t launch_dt(SgGemvParams& p, int total_rb, int num_sms, cudaStream_t st) {
  if (p.batch <= 4) return launch<DT, 0>(p, total_rb, num_sms, st);
  if (p.batch <= 8) return launch<DT, 1>(p, total_rb, num_sms, st);
  return launch<DT, 2>(p, total_rb, num_sms, st);
}

}  // namespace

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    int num_sms, cudaStream_t st) {
  if (n_mats < 1 || n_mats > SG_GEMV_MAX_MATS || batch < 1 || batch > 16) return cudaErrorInvalidValue;
  if (((uintptr_t)x & 7) || (ldx & 1)) return cudaErrorInvalidValue;
  const int dtype = mats[0].w->dtype;
  const int64_t K = mats[0].w->n_cols;
  if (K > (1 << 30)) return cudaErrorInvalidValue;
  SgGemvParams p = {};
  p.n_mats = n_mats;
  p.n_cols = (int)K;
  p.n_ch = (int)mats[0].w->n_ch;
  p.batch = batch;
  p.accumulate = accumulate ? 1 : 0;
  p.x = x;
  p.ldx = ldx;
  int64_t rbs = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->dtype != dtype || w->n_cols != K) return cudaErrorInvalidValue;
    p.mats[i].tiles = w->tiles;
    p.mats[i].dd = w->dd;
    p.mats[i].n_sb = (int)w->n_sb;
    p.mats[i].n_rb = (int)w->n_rb;
    p.mats[i].n_rows = (int)w->n_rows;
    p.mats[i].rb0 = (int)rbs;
    p.mats[i].y = mats[i].y;
    p.mats[i].ldy = mats[i].ldy;
    rbs += w->n_rb;
  }
  if (rbs * 16 > (1ll << 31)) return cudaErrorInvalidValue;
  return dtype == SG_DTYPE_Q4_0 ? launch_dt<SG_DTYPE_Q4_0>(p, (int)rbs, num_sms, st)
                                : launch_dt<SG_DTYPE_Q4_K>(p, (int)rbs, num_sms, st);
}
