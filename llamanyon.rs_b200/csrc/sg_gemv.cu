// sg_gemv.cu -- decode GEMV (batch 1..16) for Q4_0 / Q4_K on B200.
//
// Replaces the reference's CPU GEMVs: swamp-kernels fused_gemv_q4k
// (fused_gemv_q4k.rs:59-82, scalar body :466-508), its batched form
// (:527-698) and the engine's Q4_0 route (swamp-engine/src/linear.rs:68-87).
// out[b][r] = sum_k W[r][k] * x[b][k], W dequantized exactly as swamp-gguf.
//
// Two kernels per call, chained with programmatic dependent launch:
//
// 1. gemv_xprep: one CTA per output column. Scales x[b] by a power of two
//    2^e (so max|x| lands in [2^13, 2^14)), splits it into f16 hi + lo parts
//    (16+ significant bits together; the exact split makes the activation
//    error ~2^-22 relative instead of the 2^-11 of a single f16), and writes
//    them in m16n8k16 B-fragment order. Column 2b holds x_hi[b], column 2b+1
//    x_lo[b], so each thread's C fragment carries both halves of one batch.
//    Also zeroes y and (Q4_K) writes per-32 sums of the scaled x.
//
// 2. gemv_main: persistent, 4 consumer warps + 1 producer warp per CTA. The
//    work list is (matrix, row-block of 128 rows, 64-wide K chunk) units in
//    that order; CTA i takes units [i*U/G, (i+1)*U/G). The producer streams
//    each unit's 4.5 KB of packed weights plus the chunk's activation
//    fragments into a 6-deep shared-memory ring with cp.async.bulk
//    (evict-first for weights), completing on mbarriers. Consumers decode
//    nibbles straight into f16 A fragments (lop3 + one f16x2 op per pair;
//    q-8 resp. q is exact in f16), run mma.sync m16n8k16 with f32
//    accumulation per 32-element block, apply the block's scale in f32 and
//    accumulate. A row-block's partial sums are added to y with red.add when
//    the CTA leaves the row-block (row-blocks split across CTAs at most at
//    the ends of each CTA's range).
//
// The weight loads are issued before griddepcontrol.wait, so a GEMV launched
// behind another kernel starts streaming its (immutable) weights while the
// previous kernel drains; activation-dependent loads come after the wait.
#include <algorithm>

#include "sg_gemv.cuh"

namespace {

constexpr int kStages = 6;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;

template <int DT, int NT>
struct StageGeom {
  static constexpr int qs = 4096;
  static constexpr int sc = 512;
  static constexpr int dd = (DT == SG_DTYPE_Q4_K) ? 512 : 0;
  static constexpr int xf = NT * 1024;
  static constexpr int xs = (DT == SG_DTYPE_Q4_K) ? 128 : 0;
  static constexpr int off_sc = qs;
  static constexpr int off_dd = off_sc + sc;
  static constexpr int off_xf = off_dd + dd;
  static constexpr int off_xs = off_xf + xf;
  static constexpr int bytes = off_xs + xs;
};

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], const uint32_t b[2], const float z[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(z[0]), "f"(z[1]), "f"(z[2]),
        "f"(z[3]));
}

__device__ __forceinline__ void unit_decode(const SgGemvParams& p, int64_t u, int& m, int64_t& rb, int64_t& c) {
  m = 0;
#pragma unroll
  for (int i = 1; i < SG_GEMV_MAX_MATS; ++i)
    if (i < p.n_mats && u >= p.mats[i].unit0) m = i;
  const int64_t local = u - p.mats[m].unit0;
  rb = local / p.n_ch;
  c = local - rb * p.n_ch;
}

// --------------------------------------------------------------------------
// activation prep
// --------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) gemv_xprep_kernel(SgGemvParams p, const float* __restrict__ x, int64_t ldx,
                                                          int NT) {
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output; the scratch may still be in use by the previous GEMV
  const int ncols = 4 * NT;
  const int b = blockIdx.x;
  if (b >= ncols) {
    // zero the outputs (the GEMV accumulates with red.add); skipped when the
    // caller asked for out += W x
    const int64_t zid = (int64_t)(b - ncols) * blockDim.x + threadIdx.x;
    const int64_t zstride = (int64_t)(gridDim.x - ncols) * blockDim.x;
    for (int mi = 0; mi < p.n_mats; ++mi) {
      const int64_t n = p.mats[mi].n_rows;
      const int64_t tot = n * p.batch;
      for (int64_t i = zid; i < tot; i += zstride) {
        const int64_t bb = i / n, r = i - bb * n;
        p.mats[mi].y[bb * p.mats[mi].ldy + r] = 0.f;
      }
    }
    return;
  }
  const bool live = b < p.batch;
  const int64_t K = p.n_cols;
  const float* xb = x + (int64_t)(live ? b : 0) * ldx;
  __shared__ float red[8];
  __shared__ float s_scale;
  float mx = 0.f;
  if (live)
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(xb[k]));
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m2 = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m2 = fmaxf(m2, red[i]);
    int e = 0;
    if (m2 > 0.f && m2 <= 3.0e38f) {
      int ex;
      frexpf(m2, &ex);  // m2 = f * 2^ex, f in [0.5, 1)
      e = 14 - ex;      // m2 * 2^e in [2^13, 2^14)
      e = max(-120, min(120, e));
    }
    const float s = live ? ldexpf(1.f, e) : 0.f;
    s_scale = s;
    if (live) p.inv_scale[b] = ldexpf(1.f, -e);
  }
  __syncthreads();
  const float s = s_scale;
  // fragment entries: (chunk c, k16-step s4, t) -> lanes (4*g + t), g = 2*(b%4) + {0 hi, 1 lo}
  const int n = b >> 2;
  const int ghi = 2 * (b & 3);
  const int64_t items = p.n_ch * 16;
  for (int64_t it = threadIdx.x; it < items; it += blockDim.x) {
    const int t = (int)(it & 3);
    const int s4 = (int)((it >> 2) & 3);
    const int64_t c = it >> 4;
    const int64_t k0 = c * 64 + 16 * s4 + 2 * t;
    float v[4];
    const int64_t ks[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = (live && ks[j] < K) ? xb[ks[j]] * s : 0.f;
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hi[j] = __float2half_rn(v[j]);
      lo[j] = __float2half_rn(v[j] - __half2float(hi[j]));
    }
    uint2 whi, wlo;
    whi.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
    whi.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
    wlo.x = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
    wlo.y = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
    uint2* base = p.xfrag + ((c * 4 + s4) * NT + n) * 32;
    base[4 * ghi + t] = whi;
    base[4 * (ghi + 1) + t] = wlo;
  }
  if (DT == SG_DTYPE_Q4_K) {
    // per-32 sums of the scaled activations: xsum[c][j][b]
    const int64_t nsub = p.n_ch * 2;
    for (int64_t it = threadIdx.x; it < nsub; it += blockDim.x) {
      float acc = 0.f;
      const int64_t k0 = it * 32;
      if (live)
        for (int i = 0; i < 32; ++i)
          if (k0 + i < K) acc += xb[k0 + i] * s;
      p.xsum[it * 16 + b] = acc;
    }
  }
}

// --------------------------------------------------------------------------
// main persistent GEMV
// --------------------------------------------------------------------------
template <int DT, int NT>
__global__ void __launch_bounds__(kThreads) gemv_main_kernel(SgGemvParams p) {
  using G = StageGeom<DT, NT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t U = p.n_units;
  const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      const uint64_t pol = policy_evict_first();
      const int64_t n = u1 - u0;
      const int64_t pre = n < kStages ? n : kStages;
      // weights of the first stages before the grid dependency resolves
      for (int64_t i = 0; i < pre; ++i) {
        int m;
        int64_t rb, c;
        unit_decode(p, u0 + i, m, rb, c);
        const SgGemvMatP& M = p.mats[m];
        uint8_t* st = smem + i * G::bytes;
        mbar_arrive_expect_tx(&full_bar[i], G::bytes);
        const int64_t tile = rb * p.n_ch + c;
        bulk_g2s_evict_first(st, M.qs + tile * 1024, G::qs, &full_bar[i], pol);
        bulk_g2s_evict_first(st + G::off_sc, (const uint8_t*)M.sc + tile * 512, G::sc, &full_bar[i], pol);
        if (DT == SG_DTYPE_Q4_K)
          bulk_g2s(st + G::off_dd, (const uint8_t*)M.dd + (rb * M.n_sb + (c >> 2)) * 512, G::dd, &full_bar[i]);
      }
      pdl_wait();
      for (int64_t i = 0; i < pre; ++i) {
        int m;
        int64_t rb, c;
        unit_decode(p, u0 + i, m, rb, c);
        uint8_t* st = smem + i * G::bytes;
        bulk_g2s(st + G::off_xf, p.xfrag + c * (4 * NT * 32), G::xf, &full_bar[i]);
        if (DT == SG_DTYPE_Q4_K) bulk_g2s(st + G::off_xs, p.xsum + c * 32, G::xs, &full_bar[i]);
      }
      for (int64_t i = pre; i < n; ++i) {
        const int s = (int)(i % kStages);
        const uint32_t ph = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, 1)) break;
        int m;
        int64_t rb, c;
        unit_decode(p, u0 + i, m, rb, c);
        const SgGemvMatP& M = p.mats[m];
        uint8_t* st = smem + s * G::bytes;
        mbar_arrive_expect_tx(&full_bar[s], G::bytes);
        const int64_t tile = rb * p.n_ch + c;
        bulk_g2s_evict_first(st, M.qs + tile * 1024, G::qs, &full_bar[s], pol);
        bulk_g2s_evict_first(st + G::off_sc, (const uint8_t*)M.sc + tile * 512, G::sc, &full_bar[s], pol);
        if (DT == SG_DTYPE_Q4_K)
          bulk_g2s(st + G::off_dd, (const uint8_t*)M.dd + (rb * M.n_sb + (c >> 2)) * 512, G::dd, &full_bar[s]);
        bulk_g2s(st + G::off_xf, p.xfrag + c * (4 * NT * 32), G::xf, &full_bar[s]);
        if (DT == SG_DTYPE_Q4_K) bulk_g2s(st + G::off_xs, p.xsum + c * 32, G::xs, &full_bar[s]);
      }
      // drain: wait until the consumers released every stage still in flight,
      // so no bulk copy outlives the CTA
      for (int64_t i = (n > kStages ? n - kStages : 0); i < n; ++i) {
        const int s = (int)(i % kStages);
        if (!mbar_wait(&empty_bar[s], (uint32_t)((i / kStages) & 1), 2)) break;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  const int g = lane >> 2, t = lane & 3;
  const uint32_t bias_lo = DT == SG_DTYPE_Q4_0 ? SG_BIAS_LO_Q4_0 : SG_BIAS_LO_Q4_K;
  const uint32_t bias_hi = DT == SG_DTYPE_Q4_0 ? SG_BIAS_HI_Q4_0 : SG_BIAS_HI_Q4_K;
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  float acc[2][NT][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][n][j] = 0.f;

  int cur_m = -1;
  int64_t cur_rb = -1;
  auto flush = [&]() {
    if (cur_m < 0) return;
    const SgGemvMatP& M = p.mats[cur_m];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t row = cur_rb * 128 + (2 * warp + r) * 16 + g;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int b = 4 * n + t;
        if (b < p.batch) {
          const float inv = p.inv_scale[b];
          float* yb = M.y + (int64_t)b * M.ldy;
          if (row < M.n_rows) red_add_f32(yb + row, (acc[r][n][0] + acc[r][n][1]) * inv);
          if (row + 8 < M.n_rows) red_add_f32(yb + row + 8, (acc[r][n][2] + acc[r][n][3]) * inv);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][n][j] = 0.f;
      }
    }
  };

  const int64_t n = u1 - u0;
  for (int64_t i = 0; i < n; ++i) {
    const int s = (int)(i % kStages);
    const uint32_t ph = (uint32_t)((i / kStages) & 1);
    int m;
    int64_t rb, c;
    unit_decode(p, u0 + i, m, rb, c);
    if (m != cur_m || rb != cur_rb) {
      flush();
      cur_m = m;
      cur_rb = rb;
    }
    if (!mbar_wait(&full_bar[s], ph, 3)) break;
    const uint8_t* st = smem + s * G::bytes;
    const uint2* xf = reinterpret_cast<const uint2*>(st + G::off_xf);
    uint4 wq[2];
    float dsc[2][2][2];  // [r][blk or sub][hl] : Q4_0 d, Q4_K sv
    float dmn[2][2][2];  // Q4_K mv
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int rt = 2 * warp + r;
      wq[r] = reinterpret_cast<const uint4*>(st)[rt * 32 + lane];
      if (DT == SG_DTYPE_Q4_0) {
        const uint2 dv = *reinterpret_cast<const uint2*>(st + G::off_sc + rt * 64 + g * 8);
        dsc[r][0][0] = __half2float(__ushort_as_half((unsigned short)(dv.x & 0xFFFFu)));
        dsc[r][0][1] = __half2float(__ushort_as_half((unsigned short)(dv.x >> 16)));
        dsc[r][1][0] = __half2float(__ushort_as_half((unsigned short)(dv.y & 0xFFFFu)));
        dsc[r][1][1] = __half2float(__ushort_as_half((unsigned short)(dv.y >> 16)));
      } else {
        const uint2 scm = *reinterpret_cast<const uint2*>(st + G::off_sc + (rt * 16 + g * 2) * 4);
        const uint2 ddv = *reinterpret_cast<const uint2*>(st + G::off_dd + (rt * 16 + g * 2) * 4);
        const uint32_t sw[2] = {scm.x, scm.y};
        const uint32_t dw[2] = {ddv.x, ddv.y};
#pragma unroll
        for (int hl = 0; hl < 2; ++hl) {
          const float d = __half2float(__ushort_as_half((unsigned short)(dw[hl] & 0xFFFFu)));
          const float dm = __half2float(__ushort_as_half((unsigned short)(dw[hl] >> 16)));
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            dsc[r][sub][hl] = d * (float)((sw[hl] >> (8 * sub)) & 0xFFu);
            dmn[r][sub][hl] = dm * (float)((sw[hl] >> (16 + 8 * sub)) & 0xFFu);
          }
        }
      }
    }
    float tmp[2][NT][4];
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      uint32_t bf[NT][2];
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        const uint2 v = xf[(s4 * NT + nn) * 32 + lane];
        bf[nn][0] = v.x;
        bf[nn][1] = v.y;
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t w = s4 == 0 ? wq[r].x : s4 == 1 ? wq[r].y : s4 == 2 ? wq[r].z : wq[r].w;
        uint32_t a[4];
        decode_frag(w, bias_lo, bias_hi, a);
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) mma16816(tmp[r][nn], a, bf[nn], (s4 & 1) ? tmp[r][nn] : zero4);
      }
      if (s4 & 1) {
        const int blk = s4 >> 1;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float d0 = dsc[r][blk][0], d1 = dsc[r][blk][1];
#pragma unroll
          for (int nn = 0; nn < NT; ++nn) {
            acc[r][nn][0] = fmaf(d0, tmp[r][nn][0], acc[r][nn][0]);
            acc[r][nn][1] = fmaf(d0, tmp[r][nn][1], acc[r][nn][1]);
            acc[r][nn][2] = fmaf(d1, tmp[r][nn][2], acc[r][nn][2]);
            acc[r][nn][3] = fmaf(d1, tmp[r][nn][3], acc[r][nn][3]);
            if (DT == SG_DTYPE_Q4_K) {
              const float xs = reinterpret_cast<const float*>(st + G::off_xs)[blk * 16 + 4 * nn + t];
              acc[r][nn][0] = fmaf(-dmn[r][blk][0], xs, acc[r][nn][0]);
              acc[r][nn][2] = fmaf(-dmn[r][blk][1], xs, acc[r][nn][2]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }
  flush();
}

template <int DT, int NT>
cudaError_t launch_main(const SgGemvParams& p, int grid, cudaStream_t st, bool pdl) {
  using G = StageGeom<DT, NT>;
  const size_t smem = (size_t)kStages * G::bytes;
  auto kern = gemv_main_kernel<DT, NT>;
  static bool attr_set = false;  // per (DT,NT) instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int DT>
cudaError_t launch_xprep(const SgGemvParams& p, const float* x, int64_t ldx, int NT, bool accumulate, cudaStream_t st,
                         bool pdl) {
  int64_t ytot = 0;
  for (int i = 0; i < p.n_mats; ++i) ytot += p.mats[i].n_rows * p.batch;
  int zb = (int)std::min<int64_t>(64, (ytot + 2047) / 2048);
  if (zb < 1) zb = 1;
  if (accumulate) zb = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(4 * NT + zb);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_xprep_kernel<DT>, p, x, ldx, NT);
}

template <int DT>
cudaError_t launch_dt(const SgGemvParams& p, int NT, int grid, cudaStream_t st, bool pdl) {
  switch (NT) {
    case 1: return launch_main<DT, 1>(p, grid, st, pdl);
    case 2: return launch_main<DT, 2>(p, grid, st, pdl);
    case 3: return launch_main<DT, 3>(p, grid, st, pdl);
    default: return launch_main<DT, 4>(p, grid, st, pdl);
  }
}

}  // namespace

size_t sg_gemv_scratch_bytes(int64_t n_cols) {
  const int64_t n_ch = (n_cols + 63) / 64;
  const size_t xf = (size_t)n_ch * 4 * 4 * 32 * sizeof(uint2);  // NT = 4 worst case
  const size_t xs = (size_t)n_ch * 32 * sizeof(float);
  return ((xf + 255) & ~(size_t)255) + ((xs + 255) & ~(size_t)255) + 256;
}

int sg_gemv_max_ctas_per_sm() { return 2; }

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  if (n_mats < 1 || n_mats > SG_GEMV_MAX_MATS || batch < 1 || batch > 16) return cudaErrorInvalidValue;
  const int dtype = mats[0].w->dtype;
  const int64_t K = mats[0].w->n_cols;
  SgGemvParams p = {};
  p.n_mats = n_mats;
  p.n_cols = K;
  p.n_ch = mats[0].w->n_ch;
  p.batch = batch;
  int64_t units = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->dtype != dtype || w->n_cols != K) return cudaErrorInvalidValue;
    p.mats[i].qs = w->qs;
    p.mats[i].sc = w->sc;
    p.mats[i].dd = w->dd;
    p.mats[i].n_sb = w->n_sb;
    p.mats[i].n_rows = w->n_rows;
    p.mats[i].unit0 = units;
    p.mats[i].y = mats[i].y;
    p.mats[i].ldy = mats[i].ldy;
    units += w->n_rb * w->n_ch;
  }
  p.n_units = units;
  if (scratch_bytes < sg_gemv_scratch_bytes(K)) return cudaErrorInvalidValue;
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  const size_t xf = (size_t)p.n_ch * 4 * 4 * 32 * sizeof(uint2);
  p.xfrag = reinterpret_cast<uint2*>(sp);
  sp += (xf + 255) & ~(size_t)255;
  p.xsum = reinterpret_cast<float*>(sp);
  sp += (((size_t)p.n_ch * 32 * sizeof(float)) + 255) & ~(size_t)255;
  p.inv_scale = reinterpret_cast<float*>(sp);
  const int NT = (batch + 3) / 4;
  int grid = (int)std::min<int64_t>(units, (int64_t)num_sms * sg_gemv_max_ctas_per_sm());
  if (grid < 1) grid = 1;
  cudaError_t e = dtype == SG_DTYPE_Q4_0 ? launch_xprep<SG_DTYPE_Q4_0>(p, x, ldx, NT, accumulate, st, true)
                                         : launch_xprep<SG_DTYPE_Q4_K>(p, x, ldx, NT, accumulate, st, true);
  if (e != cudaSuccess) return e;
  return dtype == SG_DTYPE_Q4_0 ? launch_dt<SG_DTYPE_Q4_0>(p, NT, grid, st, true)
                                : launch_dt<SG_DTYPE_Q4_K>(p, NT, grid, st, true);
}
