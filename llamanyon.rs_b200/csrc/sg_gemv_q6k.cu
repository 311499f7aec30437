// sg_gemv_q6k.cu -- decode GEMV (batch 1..16) for Q6_K weights on the CUDA
// cores.
//
// Replaces the engine's Q6_K route (swamp-engine/src/linear.rs:48-67:
// fused_gemv_q6k, swamp-kernels/src/fused_gemv_q6k.rs:22-291). Real Q4_K_M
// checkpoints keep a few tensors (output, some ffn_down) in Q6_K; the
// tensor-core GEMV of sg_gemv.cu is built around 4-bit nibbles and 32-element
// scales, so this dtype takes a plain streaming kernel.
//
// Arithmetic: w = d * sc * (q - 32) per 16-element sub-block (q6_k.rs:37-46).
// Each thread owns one weight row of a 128-row block: per 8 weights (one
// nibble word and its high bits) it forms (q - 32) exactly as f32, sums
// (q - 32) * x over the 8 in f32 and adds d * sc times that sum to the row's
// f32 accumulator per token.
//
// Work: CTAs of 128 threads, one per (row-block, K range); the K ranges of a
// row-block (a split of its chunks, so that the grid covers the SMs several
// times) are reduced into y with red.add after the host zeroed y. The
// activations of the CTA's range are staged in shared memory 8 chunks (512 K)
// at a time and read as float4 broadcasts.
#include "sg_gemv_q6k.cuh"

namespace gemv_q6k {

constexpr int kThreads = 128;
constexpr int kWin = 8;  // chunks of x staged at once

struct Params {
  const uint8_t* tiles;
  const uint32_t* dd;
  float* y;
  int64_t ldy;
  const float* x;
  int64_t ldx;
  int n_rows, n_ch, n_sb, batch, ksplit, accumulate;
};

template <int BT>
__global__ void __launch_bounds__(kThreads) gemv_q6k_kernel(Params p) {
  __shared__ __align__(16) float xs[BT][kWin * 64];
  pdl_launch_dependents();
  const int rb = blockIdx.x, ks = blockIdx.y;
  const int r = threadIdx.x;
  const int row = rb * 128 + r;
  const int c0 = (int)((int64_t)ks * p.n_ch / p.ksplit), c1 = (int)((int64_t)(ks + 1) * p.n_ch / p.ksplit);
  float acc[BT];
#pragma unroll
  for (int t = 0; t < BT; ++t) acc[t] = 0.f;
  pdl_wait();  // x and y may come from / still be read by the previous kernel
  for (int w0 = c0; w0 < c1; w0 += kWin) {
    const int nw = min(kWin, c1 - w0);
    __syncthreads();  // the previous window is consumed
    for (int i = threadIdx.x; i < BT * nw * 16; i += kThreads) {
      const int t = i / (nw * 16), e = i - t * nw * 16;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < p.batch) v = *reinterpret_cast<const float4*>(p.x + (int64_t)t * p.ldx + (int64_t)w0 * 64 + 4 * e);
      reinterpret_cast<float4*>(&xs[t][0])[e] = v;
    }
    __syncthreads();
    for (int cw = 0; cw < nw; ++cw) {
      const int c = w0 + cw;
      const uint8_t* tile = p.tiles + ((int64_t)rb * p.n_ch + c) * SG_TILE6_BYTES;
      const uint4 lo0 = *reinterpret_cast<const uint4*>(tile + r * 16);
      const uint4 lo1 = *reinterpret_cast<const uint4*>(tile + (128 + r) * 16);
      const uint2 hi0 = *reinterpret_cast<const uint2*>(tile + SG_TILE6_HI_OFF + r * 8);
      const uint2 hi1 = *reinterpret_cast<const uint2*>(tile + SG_TILE6_HI_OFF + (128 + r) * 8);
      const uint32_t scw = *reinterpret_cast<const uint32_t*>(tile + SG_TILE6_SC_OFF + r * 4);
      const float d = __half2float(__ushort_as_half((unsigned short)(p.dd[((int64_t)rb * p.n_sb + (c >> 2)) * 128 + r] & 0xFFFFu)));
      const uint32_t lw[8] = {lo0.x, lo0.y, lo0.z, lo0.w, lo1.x, lo1.y, lo1.z, lo1.w};
      const uint32_t hw[4] = {hi0.x, hi0.y, hi1.x, hi1.y};
#pragma unroll
      for (int wi = 0; wi < 8; ++wi) {  // nibble word wi: K = 8 wi .. 8 wi + 7 of the chunk
        const int h = wi >> 2, w = wi & 3;
        const uint32_t H = hw[2 * h + (w >> 1)];
        // bytes of K offsets {0,4,1,5} and {2,6,3,7}, high bits beside the nibbles
        uint32_t qa, qb;
        if ((w & 1) == 0) {
          qa = (lw[wi] & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
          qb = ((lw[wi] >> 4) & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
        } else {
          qa = (lw[wi] & 0x0F0F0F0Fu) | (H & 0x30303030u);
          qb = ((lw[wi] >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
        }
        // q - 32 exactly: the bits of 2^23 + q, minus 2^23 + 32
        float qv[8];
        qv[0] = __uint_as_float(__byte_perm(qa, 0x4B000000u, 0x7650)) - 8388640.f;  // K offset 0
        qv[4] = __uint_as_float(__byte_perm(qa, 0x4B000000u, 0x7651)) - 8388640.f;  // 4
        qv[1] = __uint_as_float(__byte_perm(qa, 0x4B000000u, 0x7652)) - 8388640.f;  // 1
        qv[5] = __uint_as_float(__byte_perm(qa, 0x4B000000u, 0x7653)) - 8388640.f;  // 5
        qv[2] = __uint_as_float(__byte_perm(qb, 0x4B000000u, 0x7650)) - 8388640.f;  // 2
        qv[6] = __uint_as_float(__byte_perm(qb, 0x4B000000u, 0x7651)) - 8388640.f;  // 6
        qv[3] = __uint_as_float(__byte_perm(qb, 0x4B000000u, 0x7652)) - 8388640.f;  // 3
        qv[7] = __uint_as_float(__byte_perm(qb, 0x4B000000u, 0x7653)) - 8388640.f;  // 7
        const float s = d * (float)(int8_t)(scw >> (8 * (2 * h + (w >> 1))));  // sub-block 2h + w/2
        const int kx = cw * 64 + 8 * wi;
#pragma unroll
        for (int t = 0; t < BT; ++t) {
          const float4 xa = *reinterpret_cast<const float4*>(&xs[t][kx]);
          const float4 xb = *reinterpret_cast<const float4*>(&xs[t][kx + 4]);
          float part = qv[0] * xa.x;
          part = fmaf(qv[1], xa.y, part);
          part = fmaf(qv[2], xa.z, part);
          part = fmaf(qv[3], xa.w, part);
          part = fmaf(qv[4], xb.x, part);
          part = fmaf(qv[5], xb.y, part);
          part = fmaf(qv[6], xb.z, part);
          part = fmaf(qv[7], xb.w, part);
          acc[t] = fmaf(s, part, acc[t]);
        }
      }
    }
  }
  if (row >= p.n_rows) return;
#pragma unroll
  for (int t = 0; t < BT; ++t) {
    if (t < p.batch) {
      float* yp = p.y + (int64_t)t * p.ldy + row;
      if (p.ksplit > 1) red_add_f32(yp, acc[t]);
      else *yp = p.accumulate ? *yp + acc[t] : acc[t];
    }
  }
}

template <int BT>
cudaError_t launch(const Params& p, int n_rb, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)n_rb, (unsigned)p.ksplit);
  g.blockDim = dim3(kThreads);
  g.stream = st;
  g.attrs = attr;
  g.numAttrs = 1;
  return cudaLaunchKernelEx(&g, gemv_q6k_kernel<BT>, p);
}

}  // namespace gemv_q6k

cudaError_t sg_gemv_q6k(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int batch,
                        bool accumulate, int num_sms, cudaStream_t st) {
  using namespace gemv_q6k;
  if (!w || w->dtype != SG_DTYPE_Q6_K || batch < 1 || batch > 16 || !x || !y) return cudaErrorInvalidValue;
  if ((w->n_cols & 255) || ((uintptr_t)x & 15) || (ldx & 3) || ldx < w->n_cols || ldy < w->n_rows)
    return cudaErrorInvalidValue;
  Params p = {};
  p.tiles = w->tiles;
  p.dd = w->dd;
  p.y = y;
  p.ldy = ldy;
  p.x = x;
  p.ldx = ldx;
  p.n_rows = (int)w->n_rows;
  p.n_ch = (int)w->n_ch;
  p.n_sb = (int)w->n_sb;
  p.batch = batch;
  p.accumulate = accumulate ? 1 : 0;
  const int n_rb = (int)w->n_rb;
  // split K so that the grid covers the SMs about four times, at least 4
  // chunks (256 K) per CTA
  const int want = (4 * num_sms + n_rb - 1) / n_rb;
  p.ksplit = std::max(1, std::min(want, (int)(w->n_ch / 4)));
  if (p.ksplit > 1 && !accumulate) {
    // the K ranges are reduced with red.add into zeroed rows
    for (int t = 0; t < batch; ++t) {
      const cudaError_t e = cudaMemsetAsync(y + (int64_t)t * ldy, 0, (size_t)w->n_rows * sizeof(float), st);
      if (e != cudaSuccess) return e;
    }
  }
  switch (batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16) {
    case 1: return launch<1>(p, n_rb, st);
    case 2: return launch<2>(p, n_rb, st);
    case 4: return launch<4>(p, n_rb, st);
    case 8: return launch<8>(p, n_rb, st);
    default: return launch<16>(p, n_rb, st);
  }
}
