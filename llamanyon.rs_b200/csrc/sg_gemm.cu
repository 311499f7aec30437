// sg_gemm.cu -- prefill GEMM (batch > 16 tokens) for Q4_0 / Q4_K on B200:
// tcgen05 tensor cores with the accumulator in TMEM, activations fed by TMA.
//
// Replaces swamp-kernels fused_gemv_q4k_batched (fused_gemv_q4k.rs:527-698),
// which the engine's prefill issues through forward_linear_batch
// (swamp-engine/src/linear.rs:176-239, executor.rs:106-181):
//   y[t][r] = sum_k W[r][k] x[t][k],  W dequantized exactly as swamp-gguf.
//
// Precision: the reference computes in f32. A Q4_K weight needs up to 24
// significant bits and an activation 24, neither fits one 16-bit operand, and
// a single bf16 product errs by ~2^-9 -- far outside the 1e-3 parity bound. So
// both operands are split exactly into bf16 hi + lo parts (16 bits each; Q4_0
// weights have at most 15 bits and split without error) and every k-step runs
// three MMAs: A_hi*X_hi + A_hi*X_lo + A_lo*X_hi (A_lo*X_lo is ~2^-16 relative
// and dropped), all accumulating in f32 in TMEM.
//
// Two kernels, chained with programmatic dependent launch:
//  1. gemm_xprep: x (f32) -> X_hi, X_lo (bf16, [m][K]) in scratch; zeroes y
//     when the K dimension is split across CTAs.
//  2. gemm_kernel: one CTA per (128-row block, 256-token tile, K slice).
//     warp 0     producer: TMA 2-D loads of X_hi/X_lo tiles (32 K x 256
//                tokens, 64-byte swizzle) and bulk copies of the packed
//                weight tiles (4.5 KB per 64-wide chunk, + Q4_K d|dmin).
//     warp 1     allocates 256 TMEM columns; one thread issues tcgen05.mma
//                (M=128, N=256, K=16, bf16 -> f32) and tcgen05.commit.
//     warps 2-5  dequantize each 128 x 32 weight slab to exact f32, split it
//                into bf16 hi/lo and write both straight into the UMMA
//                K-major 64-byte-swizzled layout; then the epilogue: tcgen05.ld
//                of the accumulator, stores (or red.add for split K) to y.
//  Four 48 KB stages (A_hi, A_lo, X_hi, X_lo) + a 3-chunk raw weight ring.
//  Every mbarrier wait is bounded (sg_common.cuh).
#include <algorithm>
#include <mutex>

#include "sg_gemm.cuh"

namespace gemm_tc {

constexpr int BM = 128, BN = 256, BK = 32;
constexpr int kS = 4;  // MMA stages
constexpr int kR = 3;  // raw weight chunk ring
constexpr int A_BYTES = BM * BK * 2;  // 8 KB
constexpr int X_BYTES = BN * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * X_BYTES;
constexpr int RAW_BYTES = SG_TILE_BYTES + 512;
constexpr int SMEM_BYTES = kS * STAGE_BYTES + kR * RAW_BYTES + 1024;  // + alignment slack
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;

struct GemmParams {
  const uint8_t* tiles;
  const uint32_t* dd;
  int dtype;
  int n_rows, n_cols, n_ch, n_sb;
  int m;       // tokens
  int n_tt;    // token tiles
  int split;   // K slices
  int accumulate;
  float* y;
  int64_t ldy;
};

// UMMA shared-memory descriptor: K-major, 64-byte swizzle, 8-row atoms 512 B apart.
__device__ __forceinline__ uint64_t sdesc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;           // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;  // stride byte offset: 8 rows x 64 B
  d |= (uint64_t)1 << 46;           // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;           // SWIZZLE_64B
  return d;
}

// instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major, M = 128, N = 256
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// byte offset of element (row, k) in a K-major 64-byte-swizzled tile (rows of 32 bf16)
__device__ __forceinline__ uint32_t sw64_off(int row, int k) {
  return (uint32_t)((row >> 3) * 512 + (row & 7) * 64 + ((((k >> 3) ^ (row >> 1)) & 3) << 4) + (k & 7) * 2);
}

// ---------------------------------------------------------------- x prep
__global__ void __launch_bounds__(256) gemm_xprep_kernel(const float* __restrict__ x, int64_t ldx, int m, int K,
                                                          __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl,
                                                          float* __restrict__ y, int64_t ldy, int n_rows, int zero_y) {
  pdl_launch_dependents();
  pdl_wait();
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
  if (zero_y) {
    const int64_t tot = (int64_t)m * n_rows;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += stride) {
      const int64_t t = i / n_rows, r = i - t * n_rows;
      y[t * ldy + r] = 0.f;
    }
  }
}

// ---------------------------------------------------------------- GEMM
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t x_full[kS], a_full[kS], s_empty[kS], raw_full[kR], raw_empty[kR], acc_full;
  __shared__ uint32_t tmem_base_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_rb = p.n_tt * p.split;
  const int rb = blockIdx.x / per_rb;
  const int rem = blockIdx.x - rb * per_rb;
  const int tt = rem / p.split, ks = rem - tt * p.split;
  const int c0 = (int)((int64_t)ks * p.n_ch / p.split), c1 = (int)((int64_t)(ks + 1) * p.n_ch / p.split);
  const int nchunk = c1 - c0, nk = 2 * nchunk;
  uint8_t* raw_ring = smem + kS * STAGE_BYTES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&a_full[s], 4);
      mbar_init(&s_empty[s], 1);
    }
    for (int r = 0; r < kR; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], 4);
    }
    mbar_init(&acc_full, 1);
    mbar_fence_init();
    prefetch_tensormap(&map_hi);
    prefetch_tensormap(&map_lo);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0) {
      pdl_wait();  // X_hi/X_lo come from the activation-prep kernel
      const int kx0 = 64 * c0, t0 = tt * BN;
      int x_issued = 0, raw_issued = 0;
      for (int kk = 0; kk < nk; ++kk) {
        const int s = kk % kS;
        if (kk >= kS && !mbar_wait(&s_empty[s], ((kk / kS) & 1) ^ 1, 0x11)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&x_full[s], 2 * X_BYTES);
        tma_load_2d(st + 2 * A_BYTES, &map_hi, kx0 + kk * BK, t0, &x_full[s]);
        tma_load_2d(st + 2 * A_BYTES + X_BYTES, &map_lo, kx0 + kk * BK, t0, &x_full[s]);
        x_issued = kk + 1;
        if ((kk & 1) == 0) {
          const int c = kk >> 1, r = c % kR;
          if (c >= kR && !mbar_wait(&raw_empty[r], ((c / kR) & 1) ^ 1, 0x12)) break;
          raw_issued = c + 1;
          uint8_t* rw = raw_ring + r * RAW_BYTES;
          const int ch = c0 + c;
          mbar_arrive_expect_tx(&raw_full[r], SG_TILE_BYTES + (p.dtype == SG_DTYPE_Q4_K ? 512 : 0));
          bulk_g2s(rw, p.tiles + ((int64_t)rb * p.n_ch + ch) * SG_TILE_BYTES, SG_TILE_BYTES, &raw_full[r]);
          if (p.dtype == SG_DTYPE_Q4_K)
            bulk_g2s(rw + SG_TILE_BYTES, p.dd + ((int64_t)rb * p.n_sb + (ch >> 2)) * 128, 512, &raw_full[r]);
        }
      }
      if (*(volatile int*)&g_sg_error != 0) {
        // error path: let every copy still in flight land before the CTA exits
        // (each barrier has at most one phase outstanding)
        for (int j = max(0, x_issued - kS); j < x_issued; ++j) mbar_wait_drain(&x_full[j % kS], (j / kS) & 1);
        for (int j = max(0, raw_issued - kR); j < raw_issued; ++j)
          mbar_wait_drain(&raw_full[j % kR], (j / kR) & 1);
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      for (int kk = 0; kk < nk; ++kk) {
        const int s = kk % kS;
        const uint32_t ph = (kk / kS) & 1;
        if (!mbar_wait(&x_full[s], ph, 0x13) || !mbar_wait(&a_full[s], ph, 0x14)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        const uint64_t ah = sdesc_sw64(base), al = sdesc_sw64(base + A_BYTES);
        const uint64_t xh = sdesc_sw64(base + 2 * A_BYTES), xl = sdesc_sw64(base + 2 * A_BYTES + X_BYTES);
#pragma unroll
        for (int j = 0; j < BK / 16; ++j) {
          const uint64_t o = (uint64_t)(j * 32 >> 4);  // K step of 16 bf16 = 32 bytes
          umma_bf16(tmem, ah + o, xh + o, (kk | j) ? 1u : 0u);
          umma_bf16(tmem, ah + o, xl + o, 1u);
          umma_bf16(tmem, al + o, xh + o, 1u);
        }
        umma_commit(&s_empty[s]);
      }
      umma_commit(&acc_full);  // fires when every MMA above has completed
    }
  } else {
    // ====================================================== dequant warps
    const int dw = warp - 2;
    const int g = lane >> 2, t = lane & 3;
    for (int kk = 0; kk < nk; ++kk) {
      const int s = kk % kS, c = kk >> 1, h = kk & 1, r = c % kR;
      bool ok = true;
      if (h == 0) ok = mbar_wait(&raw_full[r], (c / kR) & 1, 0x15);
      if (ok && kk >= kS) ok = mbar_wait(&s_empty[s], ((kk / kS) & 1) ^ 1, 0x16);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t* rw = raw_ring + r * RAW_BYTES;
      uint8_t* a_hi = smem + s * STAGE_BYTES;
      uint8_t* a_lo = a_hi + A_BYTES;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int rt = 2 * dw + rr;
        const uint2 wv = *reinterpret_cast<const uint2*>(rw + (rt * 32 + lane) * 16 + 8 * h);
        const uint2 scw = *reinterpret_cast<const uint2*>(rw + SG_TILE_SC_OFF + (rt * 8 + g) * 8);
        float mul[2], sub[2];  // row g, row g+8: w = mul * q - sub
        if (p.dtype == SG_DTYPE_Q4_0) {
          const uint32_t dword = h ? scw.y : scw.x;
          const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&dword));
          mul[0] = d.x;
          mul[1] = d.y;
          sub[0] = 8.f * d.x;  // (q - 8) * d == q*d - 8d exactly (both terms exact in f32)
          sub[1] = 8.f * d.y;
        } else {
          const uint2 ddv = *reinterpret_cast<const uint2*>(rw + SG_TILE_BYTES + (rt * 16 + g * 2) * 4);
          const uint32_t sc2[2] = {scw.x, scw.y}, dd2[2] = {ddv.x, ddv.y};
#pragma unroll
          for (int hl = 0; hl < 2; ++hl) {
            const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dd2[hl]));
            mul[hl] = __fmul_rn(dm.x, (float)((sc2[hl] >> (8 * h)) & 0xFFu));
            sub[hl] = __fmul_rn(dm.y, (float)((sc2[hl] >> (16 + 8 * h)) & 0xFFu));
          }
        }
#pragma unroll
        for (int sw = 0; sw < 2; ++sw) {
          const uint32_t w32 = sw ? wv.y : wv.x;
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {  // nibble pairs (p, p+4): same row, k and k+1
            const int hl = pp & 1;
            const int row = rt * 16 + g + 8 * hl;
            const int k = 16 * sw + 2 * t + 8 * ((pp >> 1) & 1);
            const float q0 = (float)((w32 >> (4 * pp)) & 15u), q1 = (float)((w32 >> (4 * pp + 16)) & 15u);
            const float v0 = __fsub_rn(__fmul_rn(mul[hl], q0), sub[hl]);
            const float v1 = __fsub_rn(__fmul_rn(mul[hl], q1), sub[hl]);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(v0, v1);
            const float2 hf = __bfloat1622float2(hi);
            const __nv_bfloat162 lo = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
            const uint32_t off = sw64_off(row, k);
            *reinterpret_cast<__nv_bfloat162*>(a_hi + off) = hi;
            *reinterpret_cast<__nv_bfloat162*>(a_lo + off) = lo;
          }
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[s]);
        if (h == 1 || kk == nk - 1) mbar_arrive(&raw_empty[r]);
      }
    }
    // ============================================================== epilogue
    pdl_wait();  // y may have been zeroed by the activation-prep kernel
    const bool ok = mbar_wait(&acc_full, 0, 0x17);
    if (!ok) mbar_wait_drain(&acc_full, 0);  // the issuer always commits: MMAs must finish before TMEM is freed
    tc_fence_after();
    if (__all_sync(0xffffffffu, ok)) {
      const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31 belong to this warp
      const int row_l = quad * 32 + lane;
      const int row = rb * BM + row_l;
      const bool use_red = p.split > 1;
#pragma unroll 1
      for (int cb = 0; cb < BN / 32; ++cb) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(cb * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
            "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
              "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
              "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < p.n_rows) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int tok = tt * BN + cb * 32 + j;
            if (tok < p.m) {
              float* yp = p.y + (int64_t)tok * p.ldy + row;
              const float val = __uint_as_float(v[j]);
              if (use_red) red_add_f32(yp, val);
              else *yp = p.accumulate ? *yp + val : val;
            }
          }
        }
      }
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 2-D map over a [rows][K] bf16 matrix, box 32 (K) x 256 (rows), 64-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
  if ((K & 31) || ((uintptr_t)x & 15) || (ldx & 3) || K > (1 << 30) || (int64_t)m * K > (1ll << 40))
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
  p.n_cols = (int)K;
  p.n_ch = (int)w->n_ch;
  p.n_sb = (int)w->n_sb;
  p.m = m;
  p.n_tt = (m + BN - 1) / BN;
  p.accumulate = accumulate ? 1 : 0;
  p.y = y;
  p.ldy = ldy;
  const int64_t tiles = w->n_rb * p.n_tt;
  int split = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms / std::max<int64_t>(1, tiles), p.n_ch / 4));
  p.split = std::max(1, split);
  const bool zero_y = p.split > 1 && !accumulate;

  // 1. activation split (+ zero y for the split-K reduction)
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_xprep_kernel, x, ldx, m, (int)K, xh, xl, y, ldy, p.n_rows,
                                     zero_y ? 1 : 0);
  if (e != cudaSuccess) return e;

  // 2. GEMM
  CUtensorMap mh, ml;
  if (!make_map(&mh, xh, m, K) || !make_map(&ml, xl, m, K)) return cudaErrorInvalidValue;
  e = set_gemm_attr();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)(tiles * p.split));
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
