// sg_gemv_mma.cu -- decode GEMV (batch 1..32) for Q4_0 / Q4_K: exact integer
// products on the warp-level tensor-core MMA, block scales in f32.
//
// Replaces the engine's per-token GEMV routes: forward_linear's Q4_0 path
// (swamp-engine/src/linear.rs:68-87: dequant + f32 row dots),
// fused_gemv_q4k (swamp-kernels/src/fused_gemv_q4k.rs:59-82, scalar order
// :466-508), forward_linear_batch at decode batch sizes (linear.rs:176-239)
// and forward_linear_multi (linear.rs:96-170) when several tensors share x.
//
// Arithmetic. Per 32-element block b of row r (Q4_0: w = d*(q-8); Q4_K:
// w = sv*q - mv, sv = d*sc, mv = dmin*m):
//   y[t][r] = sum_b ( sv_b * sum_{k in b} q_k x_k  -  mv_b * sum_{k in b} x_k )
// Per 256-K unit and token, x is scaled by a power of two s (max |x|*s in
// [32, 64)) and rounded to V = rint(x*s*2^14), |V| <= 2^20, split exactly into
// V = d0*2^14 + d1*2^7 + d2 with every digit in [-64, 64] (a signed byte).
// One mma.sync.m16n8k32 (A = 16 weight rows x one 32-block of raw nibbles as
// u8, B = 8 columns of digits as s8) gives sum_k q*digit exactly in s32.
// The only approximation is rounding x to 21 bits per unit (relative 2^-15 of
// the unit's max). Non-finite x makes the unit's 1/s NaN, so every output it
// touches is NaN, as in the reference.
//
// Two column plans:
//   batch 1-2 (per-column): column 3*token + digit, one MMA per block. The
//     accumulators start at the bits of 1.5*2^23 (Q4_0; Q4_K at 0), so the
//     s32 result read as an f32 is 1.5*2^23 + sum q*digit exactly; adding
//     the column's -1.5*2^23 - 8*sum(digits) (from the activation image)
//     gives sum (q-8)*digit exactly; per column acc += d_row * D; each
//     column is scaled by 2^(-7*digit)/s per unit and the digit columns of a
//     token are summed at the end of a row segment.
//   batch 3-32 (combined): 8 tokens per MMA, one MMA per digit, every
//     accumulator starting at the bits of 1.5*2^23. Per (row, token) one
//     subtraction per digit gives D_i exactly (Q4_0's digit 2 takes the
//     token's -1.5*2^23 - 8*sum V instead, rounded once), two FMAs form
//     (D0*128 + D1)*128 + D2 (exact up to the last, which rounds once to
//     f32) and one FMA applies the block scale.
// Pairs of values (the two columns of a row that an MMA leaves in adjacent
// registers) go through the packed f32x2 add/FMA; the loop has no
// integer-to-float conversion and the MMAs' accumulator input is one
// loop-invariant register quad.
// Q4_K keeps the min term apart: per (row, block) m * (sum of the block's x).
//
// Weight layout: the repacked tiles of sg_layout.cuh, unchanged. A warp takes
// 16 rows of a 128-row block; lane (g, t) (g = lane/4, t = lane%4) reads
// word t of rows g and g+8 of each 32-block: its low nibbles (K offsets
// 8t + {0,4,1,5}) are one A register, its high nibbles (8t + {2,6,3,7})
// another. The activation images use the same K order.
//
// Work split: the chunks (128 rows x 64 K, one 4608-byte tile each) of all
// row-blocks of all matrices form one sequence, row-block major; CTA c of G
// takes chunks [c*T/G, (c+1)*T/G) and walks them in pieces, the part of one
// 256-K unit inside its range. Warp 0 lane 0 copies each piece's tiles (and
// the Q4_K d|dmin) with one bulk copy into a ring slot, plus the unit's
// activation image; eight consumer warps each own 16 rows of the piece. The
// weight copies of the first ring slots are issued before the previous
// kernel completes (programmatic dependent launch); activations and outputs
// are touched only after griddepcontrol.wait.
//
// Rows shared by several CTAs (a row-block whose chunks fall in more than one
// CTA range) are summed with red.add: the activation prep kernel, which runs
// before the GEMV in stream order, zeroes the outputs (unless the call
// accumulates), and every CTA adds its segment sums when the segment ends.
// Nothing waits on another CTA, and no state outlives a call, so a CUDA graph
// can replay the kernels any number of times. (The adds of a shared row may
// land in any order, so its last bits can differ from run to run, within
// the rounding of an f32 sum of a few terms.)
#include <algorithm>
#include <climits>

#include "sg_gemv.cuh"

namespace gemv_mma {

constexpr int kUC = 4;                         // chunks per 256-K unit
constexpr int kDdOff = kUC * SG_TILE_BYTES;    // Q4_K d|dmin of the unit's 128 rows (512 B)
constexpr int kXOff = kDdOff + 512;            // activation image within a ring slot
constexpr int kMaxCtas = SG_GEMV_MMA_MAX_CTAS;
constexpr uint32_t kMagic = 0x4B400000u;       // bits of 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;
constexpr uint32_t kNib = 0x0F0F0F0Fu;

// NTG = 0: per-column plan (batch <= 2); NTG = 1..4: groups of 8 tokens.
template <int NTG>
struct Cfg {
  static constexpr bool P = NTG == 0;
  static constexpr int NTOK = P ? 2 : 8 * NTG;     // token slots
  static constexpr int NM = P ? 1 : 3 * NTG;       // MMAs per (16 rows, 32-block)
  static constexpr int NCA = P ? 1 : NTG;          // per-column value areas per block
  static constexpr int PB = NM * 256 + NCA * 32;   // image bytes per 32-block
  static constexpr int INV_OFF = 8 * PB;           // per-unit scales after the 8 blocks
  static constexpr int XU = 8 * PB + 128;          // image bytes per unit
  static constexpr int SLOT = kXOff + XU;          // ring slot: 4 tiles, Q4_K d|dmin, image
  // 16-row tiles per consumer warp (one: 16 consumer warps per SM keep the
  // MMA -> combine chains of the wide batches issuing)
  static constexpr int RT = 1;
  static constexpr int NCW = 8 / RT;               // consumer warps
  static constexpr int THREADS = 32 * (1 + NCW);
  // two CTAs per SM, two ring slots each: about 80 KB of weights in flight
  // per SM. Deeper rings measured slower: when every CTA requests all its
  // tiles at once, they arrive together at the end and the compute cannot
  // overlap the stream.
  static constexpr int CPS = 2;
  static constexpr int R = 2;
  static constexpr int SMEM = R * SLOT + 128;
  // registers: leave room beside the GEMV CTAs for one CTA of the next
  // call's activation prep kernel (128 threads x 40 registers), which under
  // programmatic dependent launch must start while this kernel still runs
  static constexpr int MAXREG = std::min(255, ((65536 - 128 * 40) / (CPS * THREADS)) / 8 * 8);
  static_assert(SLOT % 16 == 0 && XU % 16 == 0, "bulk copies move multiples of 16 bytes");
  static_assert(SMEM * CPS <= 226 * 1024, "shared memory per SM");
};

struct Mat {
  const uint8_t* tiles;
  const uint32_t* dd;
  float* y;
  int64_t ldy;
  int n_rows, n_sb, rb0;
};

struct Params {
  Mat mats[SG_GEMV_MAX_MATS];
  int n_mats, batch, n_ch;
  int64_t total;         // chunks over all row-blocks of all matrices
  const uint8_t* ximg;   // activation unit images
  int accumulate;
};

struct XParams {
  const float* x;
  int64_t ldx;
  int K, batch, n_units;
  uint8_t* ximg;
  // outputs to zero before the GEMV adds into them (n_zero = 0: accumulate)
  float* y[SG_GEMV_MAX_MATS];
  int64_t ldy[SG_GEMV_MAX_MATS];
  int n_rows[SG_GEMV_MAX_MATS];
  int n_zero;
  SgGemvPrologue pro;
};

__device__ __forceinline__ int find_mat(const Params& p, int rbg) {
  int m = 0;
#pragma unroll
  for (int i = 1; i < SG_GEMV_MAX_MATS; ++i)
    if (i < p.n_mats && rbg >= p.mats[i].rb0) m = i;
  return m;
}

__device__ __forceinline__ int64_t cta_start(const Params& p, int b) { return (int64_t)b * p.total / gridDim.x; }
// Piece cursor over the CTA's chunk range [g, g1).
struct Cursor {
  int rbg, c, mi, rb;  // global row-block, chunk within it, matrix, row-block within the matrix
  int g, g1;           // chunk index (the host keeps the total below 2^31)
  int nrb0;            // first global row-block of the next matrix
  __device__ __forceinline__ void init(const Params& p, int64_t g0, int64_t gend) {
    g = (int)g0;
    g1 = (int)gend;
    rbg = g / p.n_ch;
    c = g - rbg * p.n_ch;
    mi = find_mat(p, rbg);
    rb = rbg - p.mats[mi].rb0;
    nrb0 = mi + 1 < p.n_mats ? p.mats[mi + 1].rb0 : INT_MAX;
  }
  __device__ __forceinline__ bool more() const { return g < g1; }
  __device__ __forceinline__ int cnt(const Params& p) const { return min(min(kUC - (c & 3), p.n_ch - c), g1 - g); }
  __device__ __forceinline__ void next(const Params& p) {
    const int n = cnt(p);
    g += n;
    c += n;
    if (c == p.n_ch) {
      c = 0;
      ++rbg;
      ++rb;
      if (rbg >= nrb0) {
        ++mi;
        rb = 0;
        nrb0 = mi + 1 < p.n_mats ? p.mats[mi + 1].rb0 : INT_MAX;
      }
    }
  }
};

// D = A (16 x 32 u8) * B (32 x 8 s8) + C, every accumulator starting at c
// (one loop-invariant register quad)
__device__ __forceinline__ void mma_u8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1, uint32_t c) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

// f16 half h (0: low, 1: high) of a scale word, as the pair (v, v)
__device__ __forceinline__ float2 h2f_pair(uint32_t w, int h) {
  return __half22float2(__half2half2(__ushort_as_half((unsigned short)(w >> (16 * h)))));
}
// byte i of a scale word as the float pair (v, v), exact: the byte is placed
// in the mantissa of 2^23, then 2^23 is subtracted
__device__ __forceinline__ float2 byte_pair(uint32_t w, int i) {
  const float a = __uint_as_float(__byte_perm(w, 0x4B000000u, (uint32_t)i | 0x7650u));
  return __fadd2_rn(make_float2(a, a), make_float2(-8388608.f, -8388608.f));
}
// the pair (c[2*q], c[2*q+1]) of MMA results read as floats: row g (q = 0) or
// g+8 (q = 1) at columns 2t, 2t+1 (adjacent registers)
__device__ __forceinline__ float2 res_pair(const int (&c)[4], int q) {
  return make_float2(__int_as_float(c[2 * q]), __int_as_float(c[2 * q + 1]));
}

// ------------------------------------------------------ activation images
// Image of one unit (256 K), for the plan of Cfg<NTG>:
//   block bu (0..7) at bu*PB:
//     [NM][lane 32][2 words]  B fragments: MMA m, lane (g, t) = the digits of
//                             column g at K offsets 8t+{0,4,1,5} | 8t+{2,6,3,7}
//     [NCA][t 4][2 words]     a value per column (lane t holds columns 2t, 2t+1):
//        per-column plan  Q4_0: f32 -1.5*2^23 - 8*sum(digits), added to the
//                         MMA result (which started at 1.5*2^23) to give
//                         sum (q-8)*digit; Q4_K: sum(digits) (the min term)
//        combined plan    area tg, column c = token 8*tg + c:
//                         Q4_0: f32 -1.5*2^23 - 8*sum(V), added to the
//                         digit-2 result; Q4_K: sum(V) as f32 (the min term)
//   INV_OFF: per-column plan: f32 [col 8] = 2^(-7*digit)/s of the column's
//            token; combined plan: f32 [token 32] = 2^-14/s. NaN when the
//            unit's x holds inf or NaN.
// A warp converts one (unit, token): lane l holds K = 256u + 8l + e,
// e = 0..7, i.e. block l/4 and layout word t = l%4 of it.
struct UnitX {
  uint32_t dig[3][2];  // digit i of the lane's 8 values, bytes in the K order of a weight word
  int dsum[3];         // sum of digit i over the lane's 32-block
  int vsum;            // sum of V over the lane's 32-block
  int se;              // s = 2^se
  bool bad;            // the unit holds inf or NaN
};

__device__ __forceinline__ void load_x8(const float* x, int64_t ldx, int K, int u, int tok, int batch, int lane,
                                        float (&v)[8]) {
  const int k0 = 256 * u + 8 * lane;
  if (tok < batch && k0 < K) {  // K is a multiple of 32: a lane's 8 values are all inside or all past it
    const float* xr = x + (int64_t)tok * ldx + k0;
    const float4 a = *reinterpret_cast<const float4*>(xr);
    const float4 b = *reinterpret_cast<const float4*>(xr + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
  }
}

// 1/sqrt(mean(x^2) + eps) of a row, in sg_rmsnorm_device's order: that
// kernel's thread t (of kSgNormThreads) sums x_i^2 for i = t, t + 512, ... in
// one FMA chain, each warp of 32 chains is reduced by the xor-shuffle tree,
// and the 16 warp sums are added in warp order. The 4 warps of a prep CTA
// replay it together: warp w runs the chain groups w, w + 4, w + 8, w + 12,
// their loads interleaved. Every thread of the CTA must call it (a CTA
// barrier); `active` is false for a padding token slot (result 1).
__device__ __forceinline__ float cta_inv_rms(const float* xr, int n, float eps, bool active, int warp, int lane) {
  constexpr int NG = kSgNormThreads / 32, G4 = NG / 4;
  __shared__ float red[NG];
  if (active) {
    float c[G4];
#pragma unroll
    for (int j = 0; j < G4; ++j) c[j] = 0.f;
    for (int m = 0; m * kSgNormThreads < n; ++m) {
#pragma unroll
      for (int j = 0; j < G4; ++j) {
        const int i = m * kSgNormThreads + 32 * (warp + 4 * j) + lane;
        if (i < n) c[j] = __fmaf_rn(xr[i], xr[i], c[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < G4; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) c[j] += __shfl_xor_sync(0xffffffffu, c[j], o);
      if (lane == 0) red[warp + 4 * j] = c[j];
    }
  }
  __syncthreads();
  if (!active) return 1.f;
  float ss = 0.f;
#pragma unroll
  for (int w = 0; w < NG; ++w) ss += red[w];
  ss = __fdiv_rn(ss, (float)n);
  ss = __fadd_rn(ss, eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(ss));
}

// silu(v) * u, v / (1 + exp(-v)) with each step rounded (sg_silu_mul_device)
__device__ __forceinline__ float silu_mul_pro(float v, float u) {
  return __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
}

// load_x8 with the call's prologue applied (inv: the token's RMSNorm factor)
__device__ __forceinline__ void load_x8_pro(const float* x, int64_t ldx, int K, int u, int tok, int batch, int lane,
                                            const SgGemvPrologue& pro, float inv, float (&v)[8]) {
  load_x8(x, ldx, K, u, tok, batch, lane, v);
  const int k0 = 256 * u + 8 * lane;
  if (pro.kind == SG_PRO_NONE || tok >= batch || k0 >= K) return;
  if (pro.kind == SG_PRO_RMSNORM) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], inv), pro.w[k0 + e]);
  } else {
    const float* ur = pro.x2 + (int64_t)tok * pro.ldx2 + k0;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = silu_mul_pro(v[e], ur[e]);
  }
}

// warp-collective: every lane calls it for the same (unit, token)
__device__ __forceinline__ UnitX unit_x(const float (&v)[8]) {
  UnitX u;
  float m = 0.f;
  bool bad = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    m = fmaxf(m, fabsf(v[e]));
    bad |= !(fabsf(v[e]) <= 3.402823466e38f);  // inf or NaN
  }
  // m >= 0 and not NaN (fmaxf drops NaN): its bits order like its value
  m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
  u.bad = __any_sync(0xffffffffu, bad);
  u.se = 0;
  if (m > 0.f && !u.bad) {
    const int e = ((__float_as_int(m) >> 23) & 0xFF) - 127;  // m in [2^e, 2^(e+1)) for normal m
    u.se = max(-126, min(126, 5 - e));
  }
  const float s = __int_as_float((127 + u.se) << 23);
  int V[8];
  u.vsum = 0;
  u.dsum[0] = u.dsum[1] = u.dsum[2] = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    V[e] = u.bad ? 0 : __float2int_rn((v[e] * s) * 16384.f);
    u.vsum += V[e];
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int pb = 0; pb < 4; ++pb) {
      const int e = (pb & 1) * 4 + (pb >> 1) + 2 * half;  // byte pb: K offsets 0,4,1,5 | 2,6,3,7
      const int d0 = (V[e] + 8192) >> 14;
      const int r0 = V[e] - (d0 << 14);
      const int d1 = (r0 + 64) >> 7;
      const int d2 = r0 - (d1 << 7);
      u.dsum[0] += d0;
      u.dsum[1] += d1;
      u.dsum[2] += d2;
      w0 |= (uint32_t)(d0 & 0xFF) << (8 * pb);
      w1 |= (uint32_t)(d1 & 0xFF) << (8 * pb);
      w2 |= (uint32_t)(d2 & 0xFF) << (8 * pb);
    }
    u.dig[0][half] = w0;
    u.dig[1][half] = w1;
    u.dig[2][half] = w2;
  }
  // sums over the block's 32 K: the 4 lanes of the block
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    u.dsum[i] += __shfl_xor_sync(0xffffffffu, u.dsum[i], 1);
    u.dsum[i] += __shfl_xor_sync(0xffffffffu, u.dsum[i], 2);
  }
  u.vsum += __shfl_xor_sync(0xffffffffu, u.vsum, 1);
  u.vsum += __shfl_xor_sync(0xffffffffu, u.vsum, 2);
  return u;
}

// 1/s times 2^-e (e >= 0), exact also where the result is subnormal
__device__ __forceinline__ float inv_scale(const UnitX& u, float two_pow_minus_e) {
  return u.bad ? __int_as_float(0x7fc00000) : __int_as_float((127 - u.se) << 23) * two_pow_minus_e;
}

// The columns of token tok in a unit image (warp-collective).
template <int DT, int NTG>
__device__ __forceinline__ void store_unit(uint8_t* unit, const UnitX& u, int tok, int lane) {
  using C = Cfg<NTG>;
  const int bu = lane >> 2, t = lane & 3;
  uint8_t* blk = unit + bu * C::PB;
  float* inv = reinterpret_cast<float*>(unit + C::INV_OFF);
  if constexpr (C::P) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int col = 3 * tok + i;
      *reinterpret_cast<uint2*>(blk + (4 * col + t) * 8) = make_uint2(u.dig[i][0], u.dig[i][1]);
      if (t == 0)  // Q4_0: exact (|8 * sum| <= 2^14)
        reinterpret_cast<uint32_t*>(blk + 256)[col] =
            DT == SG_DTYPE_Q4_0 ? __float_as_uint(-kMagicF - (float)(8 * u.dsum[i])) : (uint32_t)u.dsum[i];
      if (lane == 0) inv[col] = inv_scale(u, i == 0 ? 1.f : i == 1 ? 0.0078125f : 6.103515625e-05f);
    }
  } else {
    const int tg = tok >> 3, cc = tok & 7;
#pragma unroll
    for (int i = 0; i < 3; ++i)
      *reinterpret_cast<uint2*>(blk + ((3 * tg + i) * 32 + 4 * cc + t) * 8) = make_uint2(u.dig[i][0], u.dig[i][1]);
    if (t == 0) {  // Q4_0: rounded once (|8 * sum V| <= 2^28)
      uint32_t* ca = reinterpret_cast<uint32_t*>(blk + C::NM * 256 + tg * 32);
      ca[cc] = DT == SG_DTYPE_Q4_0 ? __float_as_uint((float)(-12582912.0 - 8.0 * (double)u.vsum))
                                   : __float_as_uint((float)u.vsum);
    }
    if (lane == 0) inv[tok] = inv_scale(u, 6.103515625e-05f);
  }
}

// The activation images of a call in global memory, and the zeroed outputs
// the GEMV adds into. One warp per (unit, token slot); token slots past the
// batch get zero digits (and in the per-column plan the token 0 warp clears
// columns 6 and 7), so every byte of the image is rewritten by every call.
template <int DT, int NTG>
__global__ void __launch_bounds__(128) xprep_kernel(XParams p) {
  using C = Cfg<NTG>;
  pdl_launch_dependents();
  pdl_wait();  // x may come from the previous kernel, which may also still read the images
  // zero the outputs: every thread of the grid takes a stride of each row
  {
    const int nth = gridDim.x * blockDim.x, tid = blockIdx.x * blockDim.x + threadIdx.x;
    for (int m = 0; m < p.n_zero; ++m)
      for (int b = 0; b < p.batch; ++b) {
        float* yr = p.y[m] + (int64_t)b * p.ldy[m];
        for (int r = tid; r < p.n_rows[m]; r += nth) yr[r] = 0.f;
      }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int u, tok;
  float inv = 1.f;
  if (p.pro.kind == SG_PRO_RMSNORM) {
    // CTA = (token slot, 4 consecutive units): its warps share the token and
    // compute its RMSNorm factor together
    const int gpt = (p.n_units + 3) / 4;
    tok = blockIdx.x / gpt;
    u = (blockIdx.x - tok * gpt) * 4 + warp;
    inv = cta_inv_rms(p.x + (int64_t)min(tok, p.batch - 1) * p.ldx, p.K, p.pro.eps, tok < p.batch, warp, lane);
    if (u >= p.n_units) return;
  } else {
    const int wg = blockIdx.x * 4 + warp;
    if (wg >= p.n_units * C::NTOK) return;
    u = wg / C::NTOK;
    tok = wg - u * C::NTOK;
  }
  float v[8];
  load_x8_pro(p.x, p.ldx, p.K, u, tok, p.batch, lane, p.pro, inv, v);
  store_unit<DT, NTG>(p.ximg + (size_t)u * C::XU, unit_x(v), tok, lane);
  if (C::P && tok == 0)  // columns 6 and 7 hold no token: zero digits, a plain start value, zero scale
    for (int i = lane; i < 8 * 2 * 4; i += 32) {
      const int bu = i >> 3, col = 6 + ((i >> 2) & 1), t = i & 3;
      uint8_t* blk = p.ximg + (size_t)u * C::XU + bu * C::PB;
      *reinterpret_cast<uint2*>(blk + (4 * col + t) * 8) = make_uint2(0u, 0u);
      if (t == 0) reinterpret_cast<uint32_t*>(blk + 256)[col] = DT == SG_DTYPE_Q4_0 ? __float_as_uint(-kMagicF) : 0u;
      if (bu == 0 && t == 0) reinterpret_cast<float*>(p.ximg + (size_t)u * C::XU + C::INV_OFF)[col] = 0.f;
    }
}

// ---------------------------------------------------------------- GEMV
// Values a lane holds for its rows (g, g+8) at the end of a row segment.
//   per-column plan: after the quad reduction, lane t holds (row g + 8*(t>>1),
//                    token t & 1)
//   combined plan:   (row g + 8*(i>>1), token 8*tg + 2t + (i&1)) for i = 0..3
template <int NTG>
struct Seg {
  static constexpr int NV = NTG == 0 ? 1 : 4 * NTG;
  float v[NV];
};

template <int NTG>
__device__ __forceinline__ void seg_coords(int lane, int j, int& rr, int& tok) {
  const int g = lane >> 2, t = lane & 3;
  if constexpr (NTG == 0) {
    rr = g + 8 * (t >> 1);
    tok = t & 1;
  } else {
    const int tg = j >> 2, i = j & 3;
    rr = g + 8 * (i >> 1);
    tok = 8 * tg + 2 * t + (i & 1);
  }
}

template <int DT, int NTG, typename C = Cfg<NTG>>
__global__ void __launch_bounds__(C::THREADS, C::CPS) __maxnreg__(C::MAXREG) gemv_kernel(Params p) {
  constexpr int RT = C::RT;
  // a shared-space array (not a generic pointer): every shared-memory access
  // below is a 32-bit shared address, most of them a constant offset
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[C::R], empty[C::R];

  pdl_launch_dependents();  // the next kernel may start its prologue as SMs free up
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g0 = cta_start(p, blockIdx.x), g1 = cta_start(p, blockIdx.x + 1);
  if (threadIdx.x == 0) {
    for (int r = 0; r < C::R; ++r) {
      mbar_init(&full[r], 1);
      mbar_init(&empty[r], C::NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ================================================================ producer
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();  // weights are read once
    Cursor cur;
    cur.init(p, g0, g1);
    Cursor cx = cur;
    auto issue_w = [&](int s, const Cursor& c) {
      const Mat& mt = p.mats[c.mi];
      const int cnt = c.cnt(p);
      uint8_t* dst = smem + s * C::SLOT;
      mbar_arrive_expect_tx(&full[s], cnt * SG_TILE_BYTES + (DT == SG_DTYPE_Q4_K ? 512 : 0) + C::XU);
      bulk_g2s_evict_first(dst, mt.tiles + ((int64_t)c.rb * p.n_ch + c.c) * SG_TILE_BYTES, cnt * SG_TILE_BYTES,
                           &full[s], pol);
      if (DT == SG_DTYPE_Q4_K)
        bulk_g2s_evict_first(dst + kDdOff, mt.dd + ((int64_t)c.rb * mt.n_sb + (c.c >> 2)) * 128, 512, &full[s], pol);
    };
    auto issue_x = [&](int s, const Cursor& c) {
      bulk_g2s(smem + s * C::SLOT + kXOff, p.ximg + (int64_t)(c.c >> 2) * C::XU, C::XU, &full[s]);
    };
    int v = 0;
    // the first slots' weights do not depend on the previous kernel
    for (; cur.more() && v < C::R; ++v, cur.next(p)) issue_w(v, cur);
    pdl_wait();
    for (int i = 0; i < v; ++i, cx.next(p)) issue_x(i, cx);
    for (; cur.more(); ++v, cur.next(p)) {
      const int s = v % C::R;
      if (!mbar_wait(&empty[s], ((v / C::R) - 1) & 1, 0x41)) break;
      issue_w(s, cur);
      issue_x(s, cur);
    }
    if (*(volatile int*)&g_sg_error != 0)  // error path: no copy may land after the CTA exits
      for (int j = max(0, v - C::R); j < v; ++j) mbar_wait_drain(&full[j % C::R], (j / C::R) & 1);
    return;
  }

  // ================================================================== consumers
  // warp w takes the 16-row tiles w, w + NCW, ... of the row-block
  const int g = lane >> 2, t = lane & 3;
  const int cw = warp - 1;  // consumer index 0..NCW-1
  int r0[RT], r1[RT];
#pragma unroll
  for (int i = 0; i < RT; ++i) {
    r0[i] = 16 * (cw + i * C::NCW) + g;
    r1[i] = r0[i] + 8;
  }
  pdl_wait();  // the images are built and y is zeroed (the prep kernel completed)

  // Sums as pairs of columns (2t, 2t+1) of one row: pair q = row g + 8q
  // (per-column plan: columns; combined plan, at 2*tg + q: tokens 8*tg + 2t
  // and 8*tg + 2t + 1). Per-unit sums are reset at every piece end,
  // per-segment sums at every segment end; the pairs go through the packed
  // f32x2 instructions (an MMA's two results of a row sit in adjacent
  // registers).
  constexpr int NP = C::P ? 2 : 2 * NTG;
  float2 acc[RT][NP], accu[RT][NP], accm[RT][NP];  // accm: Q4_K min term (combined plan)
  int iacc[RT][4], iacm[RT][4];                    // Q4_K per-column plan: integer sums over the unit
#pragma unroll
  for (int r = 0; r < RT; ++r) {
#pragma unroll
    for (int i = 0; i < NP; ++i) acc[r][i] = accu[r][i] = accm[r][i] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) iacc[r][i] = iacm[r][i] = 0;
  }
  const float2 neg_magic = make_float2(-kMagicF, -kMagicF);
  const float2 f128 = make_float2(128.f, 128.f);

  Cursor cur;
  cur.init(p, g0, g1);
  int v = 0;
  for (; cur.more(); ++v, cur.next(p)) {
    const int s = v % C::R;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (v / C::R) & 1, 0x42))) break;
    const uint8_t* slot = smem + s * C::SLOT;
    const uint8_t* xim = slot + kXOff;
    const int cnt = cur.cnt(p), ci0 = cur.c & 3;
    // one 64-K chunk of the piece: j = its tile in the slot, cj = its place in the unit
    auto chunk = [&](const int j, const int cj) {
      const uint8_t* tile = slot + j * SG_TILE_BYTES;
      uint32_t sw0[RT], sw1[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        sw0[r] = *reinterpret_cast<const uint32_t*>(tile + SG_TILE_SC_OFF + r0[r] * 4);
        sw1[r] = *reinterpret_cast<const uint32_t*>(tile + SG_TILE_SC_OFF + r1[r] * 4);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t a[RT][4];
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(tile + h * 2048 + r0[r] * 16 + 4 * t);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(tile + h * 2048 + r1[r] * 16 + 4 * t);
          a[r][0] = w0 & kNib;
          a[r][1] = w1 & kNib;
          a[r][2] = (w0 >> 4) & kNib;
          a[r][3] = (w1 >> 4) & kNib;
        }
        const uint8_t* xb = xim + (2 * cj + h) * C::PB;
        if constexpr (C::P) {
          const uint2 b = *reinterpret_cast<const uint2*>(xb + lane * 8);
          const uint2 ci = *reinterpret_cast<const uint2*>(xb + 256 + t * 8);
#pragma unroll
          for (int r = 0; r < RT; ++r) {
            int d[4];
            mma_u8s8_c(d, a[r][0], a[r][1], a[r][2], a[r][3], b.x, b.y, DT == SG_DTYPE_Q4_0 ? kMagic : 0u);
            if constexpr (DT == SG_DTYPE_Q4_0) {
              // result + (-1.5*2^23 - 8*sum digits) = sum (q-8)*digit, exact
              const float2 corr = make_float2(__uint_as_float(ci.x), __uint_as_float(ci.y));
              accu[r][0] = __ffma2_rn(h2f_pair(sw0[r], h), __fadd2_rn(res_pair(d, 0), corr), accu[r][0]);
              accu[r][1] = __ffma2_rn(h2f_pair(sw1[r], h), __fadd2_rn(res_pair(d, 1), corr), accu[r][1]);
            } else {
              const int sc0 = (sw0[r] >> (8 * h)) & 0xFF, sc1 = (sw1[r] >> (8 * h)) & 0xFF;
              const int m0 = (sw0[r] >> (16 + 8 * h)) & 0xFF, m1 = (sw1[r] >> (16 + 8 * h)) & 0xFF;
              iacc[r][0] += sc0 * d[0];
              iacc[r][1] += sc0 * d[1];
              iacc[r][2] += sc1 * d[2];
              iacc[r][3] += sc1 * d[3];
              iacm[r][0] += m0 * (int)ci.x;
              iacm[r][1] += m0 * (int)ci.y;
              iacm[r][2] += m1 * (int)ci.x;
              iacm[r][3] += m1 * (int)ci.y;
            }
          }
        } else {
          float2 fs[RT][2], ns[RT][2];  // scales of rows g, g+8 as pairs: Q4_0 d; Q4_K sc and m
#pragma unroll
          for (int r = 0; r < RT; ++r) {
            if constexpr (DT == SG_DTYPE_Q4_0) {
              fs[r][0] = h2f_pair(sw0[r], h);
              fs[r][1] = h2f_pair(sw1[r], h);
            } else {
              fs[r][0] = byte_pair(sw0[r], h);  // sc
              fs[r][1] = byte_pair(sw1[r], h);
              ns[r][0] = byte_pair(sw0[r], 2 + h);  // m
              ns[r][1] = byte_pair(sw1[r], 2 + h);
            }
          }
#pragma unroll
          for (int tg = 0; tg < NTG; ++tg) {
            uint2 b[3];
#pragma unroll
            for (int i = 0; i < 3; ++i) b[i] = *reinterpret_cast<const uint2*>(xb + (3 * tg + i) * 256 + lane * 8);
            // tokens 2t, 2t+1: Q4_0 -1.5*2^23 - 8*sum V (the digit-2 offset); Q4_K sum V
            const float2 cv = *reinterpret_cast<const float2*>(xb + C::NM * 256 + tg * 32 + t * 8);
#pragma unroll
            for (int r = 0; r < RT; ++r) {
              int dd[3][4];
#pragma unroll
              for (int i = 0; i < 3; ++i)
                mma_u8s8_c(dd[i], a[r][0], a[r][1], a[r][2], a[r][3], b[i].x, b[i].y, kMagic);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                // digit sums D_i = result - 1.5*2^23 (exact; Q4_0's digit 2 also
                // takes -8*sum V, rounded once); (D0*128 + D1) is exact, *128 + D2
                // rounds once: the pair's sum_k q_k V_k (Q4_0: (q_k - 8) V_k)
                const float2 e0 = __fadd2_rn(res_pair(dd[0], q), neg_magic);
                const float2 e1 = __fadd2_rn(res_pair(dd[1], q), neg_magic);
                const float2 e2 = __fadd2_rn(res_pair(dd[2], q), DT == SG_DTYPE_Q4_0 ? cv : neg_magic);
                const float2 val = __ffma2_rn(__ffma2_rn(e0, f128, e1), f128, e2);
                accu[r][2 * tg + q] = __ffma2_rn(fs[r][q], val, accu[r][2 * tg + q]);
                if constexpr (DT == SG_DTYPE_Q4_K) accm[r][2 * tg + q] = __ffma2_rn(ns[r][q], cv, accm[r][2 * tg + q]);
              }
            }
          }
        }
      }
    };
    bool whole = false;
    if constexpr (NTG <= 2) {
      // a whole unit (the common case): straight-line code, every shared-memory
      // address a constant offset from the slot
      if (cnt == kUC) {
#pragma unroll
        for (int j = 0; j < kUC; ++j) chunk(j, j);
        whole = true;
      }
    }
    if (!whole) {
#pragma unroll 1
      for (int j = 0; j < cnt; ++j) chunk(j, ci0 + j);
    }
    // ---- piece end: apply the unit's 1/s (and Q4_K's d, dmin)
    const float* inv = reinterpret_cast<const float*>(xim + C::INV_OFF);
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      float2 dm[2], nm[2];  // Q4_K: d and -dmin of rows g (0) and g+8 (1), as pairs
      if constexpr (DT == SG_DTYPE_Q4_K) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(slot + kDdOff + (q ? r1[r] : r0[r]) * 4);
          dm[q] = h2f_pair(w, 0);
          const float2 mn = h2f_pair(w, 1);
          nm[q] = make_float2(-mn.x, -mn.y);
        }
      }
      if constexpr (C::P) {
        const float2 iv = *reinterpret_cast<const float2*>(inv + 2 * t);  // columns 2t, 2t+1
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          if constexpr (DT == SG_DTYPE_Q4_0) {
            acc[r][q] = __ffma2_rn(iv, accu[r][q], acc[r][q]);
            accu[r][q] = make_float2(0.f, 0.f);
          } else {
            const float2 ia = make_float2((float)iacc[r][2 * q], (float)iacc[r][2 * q + 1]);
            const float2 im = make_float2((float)iacm[r][2 * q], (float)iacm[r][2 * q + 1]);
            acc[r][q] = __ffma2_rn(iv, __ffma2_rn(dm[q], ia, __fmul2_rn(nm[q], im)), acc[r][q]);
            iacc[r][2 * q] = iacc[r][2 * q + 1] = iacm[r][2 * q] = iacm[r][2 * q + 1] = 0;
          }
        }
      } else {
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) {
          const float2 iv = *reinterpret_cast<const float2*>(inv + 8 * tg + 2 * t);  // tokens 2t, 2t+1 of the group
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int i = 2 * tg + q;
            if constexpr (DT == SG_DTYPE_Q4_0) {
              acc[r][i] = __ffma2_rn(iv, accu[r][i], acc[r][i]);
            } else {
              acc[r][i] = __ffma2_rn(iv, __ffma2_rn(dm[q], accu[r][i], __fmul2_rn(nm[q], accm[r][i])), acc[r][i]);
              accm[r][i] = make_float2(0.f, 0.f);
            }
            accu[r][i] = make_float2(0.f, 0.f);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the slot is free (the next lines touch no shared memory)

    // ---- segment end: the row-block ends here or the CTA's range does
    const bool rb_end = cur.c + cnt == p.n_ch;
    if (!rb_end && cur.g + cnt != cur.g1) continue;
    const Mat& mt = p.mats[cur.mi];
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      Seg<NTG> sv;
      if constexpr (C::P) {
        // column c = 3*token + digit; lane t holds columns 2t (.x) and 2t+1 (.y)
        const int ca = 2 * t, cb = 2 * t + 1;
        float pv[4];
        pv[0] = (ca / 3 == 0 ? acc[r][0].x : 0.f) + (cb / 3 == 0 ? acc[r][0].y : 0.f);  // row g, token 0
        pv[1] = (ca / 3 == 1 ? acc[r][0].x : 0.f) + (cb / 3 == 1 ? acc[r][0].y : 0.f);  // row g, token 1
        pv[2] = (ca / 3 == 0 ? acc[r][1].x : 0.f) + (cb / 3 == 0 ? acc[r][1].y : 0.f);  // row g+8, token 0
        pv[3] = (ca / 3 == 1 ? acc[r][1].x : 0.f) + (cb / 3 == 1 ? acc[r][1].y : 0.f);  // row g+8, token 1
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pv[i] += __shfl_xor_sync(0xffffffffu, pv[i], 1);
          pv[i] += __shfl_xor_sync(0xffffffffu, pv[i], 2);
        }
        sv.v[0] = t == 0 ? pv[0] : t == 1 ? pv[1] : t == 2 ? pv[2] : pv[3];
      } else {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          sv.v[2 * i] = acc[r][i].x;
          sv.v[2 * i + 1] = acc[r][i].y;
        }
      }
#pragma unroll
      for (int i = 0; i < NP; ++i) acc[r][i] = make_float2(0.f, 0.f);
      const int tile_row0 = r0[r] - g;  // first row of the 16-row tile
      // a row-block run by this CTA alone is stored; one shared with other
      // CTAs (zeroed by the prep kernel unless the call accumulates) is added to
      const int64_t lo = (int64_t)cur.rbg * p.n_ch;
      const bool shared = lo < g0 || lo + p.n_ch > g1;
#pragma unroll
      for (int i = 0; i < Seg<NTG>::NV; ++i) {
        int rr, tok;
        seg_coords<NTG>(lane, i, rr, tok);
        const int grow = cur.rb * 128 + tile_row0 + rr;
        if (tok < p.batch && grow < mt.n_rows) {
          float* yp = mt.y + (int64_t)tok * mt.ldy + grow;
          if (shared)
            red_add_f32(yp, sv.v[i]);
          else
            *yp = p.accumulate ? *yp + sv.v[i] : sv.v[i];
        }
      }
    }
  }
}

// ------------------------------------------------------------ host side
inline int ntg_of(int batch) { return batch <= 2 ? 0 : (batch + 7) / 8; }

// workspace: the activation images of a call
template <int NTG>
constexpr size_t ws_bytes(int64_t n_units) {
  return (size_t)n_units * Cfg<NTG>::XU;
}

template <int DT, int NTG>
cudaError_t launch(Params p, XParams xp, int rb_total, int num_sms, cudaStream_t st) {
  using C = Cfg<NTG>;
  p.total = (int64_t)rb_total * p.n_ch;
  if (p.total >= INT_MAX / 2) return cudaErrorInvalidValue;  // the device cursor counts chunks in 32 bits
  // per device, once: the shared-memory size and a carveout that lets CPS
  // CTAs share an SM, then the CTAs per SM that actually fit (one wave)
  static int per_sm[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!per_sm[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<DT, NTG>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_kernel<DT, NTG>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared);
    int n = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kernel<DT, NTG>, C::THREADS, C::SMEM);
    if (e != cudaSuccess) return e;
    per_sm[dev] = std::max(1, std::min(n, C::CPS));
  }
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(std::min(num_sms * per_sm[dev], kMaxCtas), p.total));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t x = {};  // the activation images and zeroed outputs
  x.gridDim = dim3((unsigned)(xp.pro.kind == SG_PRO_RMSNORM ? C::NTOK * ((xp.n_units + 3) / 4)
                                                             : (xp.n_units * C::NTOK + 3) / 4));
  x.blockDim = dim3(128);
  x.stream = st;
  x.attrs = attr;
  x.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&x, xprep_kernel<DT, NTG>, xp);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)G);
  g.blockDim = dim3(C::THREADS);
  g.dynamicSmemBytes = C::SMEM;
  g.stream = st;
  g.attrs = attr;
  g.numAttrs = 1;
  return cudaLaunchKernelEx(&g, gemv_kernel<DT, NTG>, p);
}

}  // namespace gemv_mma

size_t sg_gemv_scratch_bytes(int64_t n_cols, int batch) {
  using namespace gemv_mma;
  const int64_t n_units = (n_cols + 255) / 256;
  switch (ntg_of(batch)) {
    case 0: return ws_bytes<0>(n_units);
    case 1: return ws_bytes<1>(n_units);
    case 2: return ws_bytes<2>(n_units);
    case 3: return ws_bytes<3>(n_units);
    default: return ws_bytes<4>(n_units);
  }
}

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st, const SgGemvPrologue* pro) {
  using namespace gemv_mma;
  if (n_mats < 1 || n_mats > SG_GEMV_MAX_MATS || batch < 1 || batch > SG_GEMV_MAX_BATCH || !x || !scratch)
    return cudaErrorInvalidValue;
  const SgDevWeight* w0 = mats[0].w;
  const int64_t K = w0->n_cols;
  if ((K & 31) || K > (1 << 28) || ((uintptr_t)x & 15) || (ldx & 3) || ldx < K) return cudaErrorInvalidValue;
  if (w0->dtype != SG_DTYPE_Q4_0 && w0->dtype != SG_DTYPE_Q4_K) return cudaErrorInvalidValue;
  if (scratch_bytes < sg_gemv_scratch_bytes(K, batch) || ((uintptr_t)scratch & 255)) return cudaErrorInvalidValue;
  Params p = {};
  p.n_mats = n_mats;
  p.batch = batch;
  p.n_ch = (int)w0->n_ch;
  XParams xp = {};
  int rb = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->n_cols != K || w->dtype != w0->dtype || !mats[i].y || mats[i].ldy < w->n_rows) return cudaErrorInvalidValue;
    p.mats[i] = {w->tiles, w->dd, mats[i].y, mats[i].ldy, (int)w->n_rows, (int)w->n_sb, rb};
    xp.y[i] = mats[i].y;
    xp.ldy[i] = mats[i].ldy;
    xp.n_rows[i] = (int)w->n_rows;
    rb += (int)w->n_rb;
  }
  const int ntg = ntg_of(batch);
  p.ximg = static_cast<uint8_t*>(scratch);
  p.accumulate = accumulate ? 1 : 0;
  xp.x = x;
  xp.ldx = ldx;
  xp.K = (int)K;
  xp.batch = batch;
  xp.n_units = (int)((K + 255) / 256);
  xp.ximg = static_cast<uint8_t*>(scratch);
  xp.n_zero = accumulate ? 0 : n_mats;
  if (pro && pro->kind != SG_PRO_NONE) {
    if ((pro->kind == SG_PRO_RMSNORM && !pro->w) || (pro->kind == SG_PRO_SILU_MUL && (!pro->x2 || pro->ldx2 < K)) ||
        pro->kind > SG_PRO_SILU_MUL)
      return cudaErrorInvalidValue;
    xp.pro = *pro;
  }
#define SG_GEMV_LAUNCH(DT)                                       \
  switch (ntg) {                                                 \
    case 0: return launch<DT, 0>(p, xp, rb, num_sms, st);        \
    case 1: return launch<DT, 1>(p, xp, rb, num_sms, st);        \
    case 2: return launch<DT, 2>(p, xp, rb, num_sms, st);        \
    case 3: return launch<DT, 3>(p, xp, rb, num_sms, st);        \
    default: return launch<DT, 4>(p, xp, rb, num_sms, st);       \
  }
  if (w0->dtype == SG_DTYPE_Q4_0) SG_GEMV_LAUNCH(SG_DTYPE_Q4_0)
  SG_GEMV_LAUNCH(SG_DTYPE_Q4_K)
#undef SG_GEMV_LAUNCH
}
