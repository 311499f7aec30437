// sg_ops.cu -- the non-matmul layer operations of a decoder layer on the GPU,
// so that an engine keeps its activations in device memory between the
// quantized linears (swamp-engine/src/executor.rs:403-550 decode step,
// :48-190 batched prefill).
//
//   sg_rmsnorm_device    ops.rs:188-201   rmsnorm
//   sg_rope_create       ops.rs:20-38     init_rope_lut (f32 table, same libm)
//   sg_rope_kv_device    ops.rs:42-80     apply_rope_ufc, then
//                        cache.rs:348-371,412-434  PagedKVCache::save / save_at
//   sg_attention_device  ops.rs:82-186    attention (GQA, causal, softmax)
//   sg_rope_attention_device              the decode step's RoPE + save +
//                        attention for one row per sequence (executor.rs:447-481)
//   sg_attention_prefill_device           the prefill's per-position attention
//                        loop (executor.rs:135-141), blocks of positions per CTA
//   sg_silu_mul_device   ops.rs:203-214   silu, mul_in_place
//   sg_add_device        ops.rs:216-220   add_in_place
//   sg_argmax_device     sampler.rs:94-95 greedy pick (the sampler's fallback)
//   sg_embed_device      executor.rs:416-418 embedding row copy, dequantized
//                        from the GGUF tensor on the device
//
// Numerics. RoPE applies the reference's f32 table with the reference's
// operation order and no FMA contraction: bit-exact. Residual add, SiLU-mul's
// multiply and the embedding rows are exact or single IEEE operations
// (SiLU's exp is CUDA's expf, within 2 ulp of the host libm). RMSNorm and
// attention sum in a different order than the reference's sequential loops:
// tolerance-bound.
//
// KV cache layout. The reference pages its cache in blocks of 32 positions
// with [layer][kv_head][slot][head_dim] per page so that pages can move to
// NVMe. On a 180 GB GPU the cache stays resident, so it is one array per K
// and V: [seq][layer][kv_head][max_seq][head_dim] f32. The positions of one
// (seq, layer, head) are contiguous, and so is any run of them that an
// attention split reads.
#include <cmath>

struct sg_rope_s {
  int head_dim = 0, max_context = 0, device = -1;
  float2* lut = nullptr;  // [max_context][head_dim/2] (cos, sin)
};

struct sg_kv_cache_s {
  int n_layers = 0, n_kv_heads = 0, head_dim = 0, max_seq = 0, n_seqs = 0, device = -1;
  float* k = nullptr;
  float* v = nullptr;
  __host__ __device__ size_t head_off(int seq, int layer, int kvh) const {
    return (((size_t)seq * n_layers + layer) * n_kv_heads + kvh) * (size_t)max_seq * head_dim;
  }
};

namespace ops {

#define SG_DEVERR_BAD_INPUT 0x300  // a device-side index (position, token, sequence) out of range

struct KvView {  // the cache geometry passed by value to kernels
  int n_layers, n_kv_heads, head_dim, max_seq, n_seqs;
  float* k;
  float* v;
  __device__ size_t head_off(int seq, int layer, int kvh) const {
    return (((size_t)seq * n_layers + layer) * n_kv_heads + kvh) * (size_t)max_seq * head_dim;
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Every op kernel is launched with programmatic dependent launch, like the
// linears: it lets the next kernel start its prologue at once and waits for
// the previous kernel's results before its first global access, so a GEMV
// that follows streams its weights while the op still runs.
__device__ __forceinline__ void pdl_enter() {
  pdl_launch_dependents();
  pdl_wait();
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t c = {};
  c.gridDim = grid;
  c.blockDim = block;
  c.dynamicSmemBytes = smem;
  c.stream = st;
  c.attrs = attr;
  c.numAttrs = 1;
  return cudaLaunchKernelEx(&c, kernel, args...);
}

// ------------------------------------------------------------------ rmsnorm
// One CTA per row: ss = sum x^2, ss /= n, ss += eps, inv = 1 / sqrt(ss),
// out = (x * inv) * w, each step one IEEE operation as in ops.rs:190-199;
// only the summation order of ss differs (a tree instead of a running sum).
constexpr int kNormThreads = kSgNormThreads;  // the decode GEMV's RMSNorm prologue replays this order
constexpr int kNormRegs = 8;  // elements per thread kept in registers (rows up to 4096 read once)
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* x, int64_t ldx, const float* __restrict__ w,
                                                              float* out, int64_t ldo, int n, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_launch_dependents();
  // the norm weights are constant: fetch them before waiting for the
  // previous kernel, whose output x is
  float wv[kNormRegs];
#pragma unroll
  for (int u = 0; u < kNormRegs; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    wv[u] = i < n ? w[i] : 0.f;
  }
  pdl_wait();
  const float* xr = x + (int64_t)blockIdx.x * ldx;
  float* orow = out + (int64_t)blockIdx.x * ldo;
  float xv[kNormRegs];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kNormRegs; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    xv[u] = i < n ? xr[i] : 0.f;
    ss = __fmaf_rn(xv[u], xv[u], ss);
  }
  for (int i = threadIdx.x + kNormRegs * kNormThreads; i < n; i += kNormThreads) ss = __fmaf_rn(xr[i], xr[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) ss += red[i];
  ss = __fdiv_rn(ss, (float)n);
  ss = __fadd_rn(ss, eps);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss));
#pragma unroll
  for (int u = 0; u < kNormRegs; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    if (i < n) orow[i] = __fmul_rn(__fmul_rn(xv[u], inv), wv[u]);
  }
  for (int i = threadIdx.x + kNormRegs * kNormThreads; i < n; i += kNormThreads)
    orow[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// -------------------------------------------------------- RoPE + cache store
// One CTA per row. Pair k of every head: (x, y) -> (x cos - y sin, x sin + y cos)
// with each product rounded before the add (ops.rs:77-78). The table row is
// min(pos, max_context - 1) (ops.rs:54). Rotated k and the row's v are then
// stored at position pos of sequence seq in layer `layer` (cache.rs:348-371).
// lut == nullptr stores without rotating.
__global__ void rope_kv_kernel(const float2* __restrict__ lut, int max_context, KvView kv, int layer, float* q,
                               int64_t ldq, float* k, int64_t ldk, const float* v, int64_t ldv, const int32_t* pos,
                               const int32_t* seq, int n_q_heads) {
  pdl_enter();
  const int r = blockIdx.x;
  const int p = pos[r];
  const int s = seq ? seq[r] : 0;
  const int hd = kv.head_dim, half = hd >> 1;
  const bool store_ok = p >= 0 && p < kv.max_seq && s >= 0 && s < kv.n_seqs;
  if (!store_ok || (lut && p < 0)) {
    if (threadIdx.x == 0) sg_set_error(SG_DEVERR_BAD_INPUT);
    return;
  }
  if (lut) {
    const float2* row = lut + (int64_t)min(p, max_context - 1) * half;
    float* qr = q + (int64_t)r * ldq;
    for (int i = threadIdx.x; i < n_q_heads * half; i += blockDim.x) {
      const int h = i / half, j = i - h * half;
      float* e = qr + h * hd + 2 * j;
      const float x0 = e[0], y0 = e[1];
      const float2 cs = row[j];
      e[0] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(y0, cs.y));
      e[1] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(y0, cs.x));
    }
    float* kr = k + (int64_t)r * ldk;
    for (int i = threadIdx.x; i < kv.n_kv_heads * half; i += blockDim.x) {
      const int h = i / half, j = i - h * half;
      float* e = kr + h * hd + 2 * j;
      const float x0 = e[0], y0 = e[1];
      const float2 cs = row[j];
      const float a = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(y0, cs.y));
      const float b = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(y0, cs.x));
      e[0] = a;
      e[1] = b;
      float* c = kv.k + kv.head_off(s, layer, h) + (size_t)p * hd + 2 * j;
      c[0] = a;
      c[1] = b;
    }
  } else {
    const float* kr = k + (int64_t)r * ldk;
    for (int i = threadIdx.x; i < kv.n_kv_heads * hd; i += blockDim.x) {
      const int h = i / hd, j = i - h * hd;
      kv.k[kv.head_off(s, layer, h) + (size_t)p * hd + j] = kr[i];
    }
  }
  const float* vr = v + (int64_t)r * ldv;
  for (int i = threadIdx.x; i < kv.n_kv_heads * hd; i += blockDim.x) {
    const int h = i / hd, j = i - h * hd;
    kv.v[kv.head_off(s, layer, h) + (size_t)p * hd + j] = vr[i];
  }
}

// ---------------------------------------------------------------- attention
// Row r (one query token: sequence seq[r], position pos[r]) attends positions
// 0 .. valid_end = min(pos, seq_len - 1) of its sequence (ops.rs:95), with
// query head h reading KV head h / n_rep (ops.rs:94,105). Scores are
// dot(q, k) * scale, softmax over them, out = sum p v (ops.rs:135-180).
//
// Split: a CTA of 64 threads takes 64 positions of one (row, KV head) and all
// n_rep query heads of that head, so each K and V row is read once per query
// token. One thread copies the split's K and V rows (contiguous in the cache)
// into shared memory with two bulk copies, so a whole split is in flight at
// once. A thread then scores one position against the n_rep queries,
// starting its walk over head_dim at its own offset so that the 8 threads of
// a shared-memory phase touch 8 different banks; each warp sums p v over its
// 32 positions with lanes owning head_dim/32 components. A CTA writes (max m,
// sum l of exp(s - m), sum exp(s - m) v) per query head; the combine kernel
// rescales the splits to the global max and divides by the global sum.
constexpr int kAttnP = 64;        // positions per split
constexpr int kAttnThreads = 64;  // one per position
constexpr int kMaxRep = 8;        // query heads per KV head

struct AttnArgs {
  KvView kv;
  int layer;
  const float* q;
  int64_t ldq;
  const int32_t* pos;
  const int32_t* seq_len;
  const int32_t* seq;
  int n_heads, n_rep, n_split;
  float scale;
  float* ws;  // [row][head][split][HD + 2]
  // decode form only (one row per sequence): RoPE and the cache store of
  // the row's own k and v happen in the split that holds its position
  const float2* lut;
  int max_context;
  const float* k_new;
  int64_t ldk;
  const float* v_new;
  int64_t ldv;
};

template <int HD>
struct AttnSmem {
  static constexpr size_t kTile = (size_t)kAttnP * HD * 4;
  static constexpr size_t kQ = 2 * kTile;
  static constexpr size_t kSc = kQ + (size_t)kMaxRep * HD * 4;
  static constexpr size_t kRed = kSc + (size_t)kMaxRep * kAttnP * 4;
  static constexpr size_t kMl = kRed + (size_t)(kAttnThreads / 32) * kMaxRep * HD * 4;
  static constexpr size_t kBar = kMl + (size_t)kMaxRep * 2 * 4;
  static constexpr size_t kBytes = kBar + 16;
};

__device__ __forceinline__ int attn_valid_end(const AttnArgs& a, int r) {
  const int p = a.pos[r];
  int e = p;
  if (a.seq_len) e = min(e, a.seq_len[r] - 1);
  return min(e, a.kv.max_seq - 1);
}

template <int HD, bool DECODE>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnArgs a) {
  using L = AttnSmem<HD>;
  constexpr int DL = HD / 32;  // components per lane
  constexpr int NC = HD / 4;   // float4 columns per row
  extern __shared__ __align__(128) uint8_t smem[];
  float* ks = reinterpret_cast<float*>(smem);
  float* vs = ks + kAttnP * HD;
  float* qs = reinterpret_cast<float*>(smem + L::kQ);
  float* sc = reinterpret_cast<float*>(smem + L::kSc);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* mls = reinterpret_cast<float*>(smem + L::kMl);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBar);
  __shared__ int ok_flag;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache rows come from the previous kernels
  const int sp = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p = a.pos[r];
  if (DECODE && (p < 0 || p >= a.kv.max_seq)) {  // the row's k and v have no cache slot
    if (tid == 0 && sp == 0) sg_set_error(SG_DEVERR_BAD_INPUT);
    return;
  }
  const int valid_end = attn_valid_end(a, r);
  const int t0 = sp * kAttnP;
  if (valid_end < 0 || t0 > valid_end) return;  // the combine reads splits 0 .. valid_end / 64 only
  const int s = a.seq ? a.seq[r] : 0;
  if (s < 0 || s >= a.kv.n_seqs) {
    if (tid == 0) sg_set_error(SG_DEVERR_BAD_INPUT);
    return;
  }
  const int nv = min(kAttnP, valid_end - t0 + 1);
  // decode: the split holding position p (= valid_end) makes row p itself
  const bool own = DECODE && t0 + nv - 1 == p;
  const int ncopy = own ? nv - 1 : nv;
  const size_t hoff = a.kv.head_off(s, a.layer, g) + (size_t)t0 * HD;
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)ncopy * HD * 4;  // whole rows: a multiple of 16
    mbar_arrive_expect_tx(bar, 2 * bytes);
    if (bytes) {
      bulk_g2s(ks, a.kv.k + hoff, bytes, bar);
      bulk_g2s(vs, a.kv.v + hoff, bytes, bar);
    }
  }
  const int n_rep = a.n_rep;
  const float* qrow = a.q + (int64_t)r * a.ldq + (int64_t)g * n_rep * HD;
  if constexpr (DECODE) {
    // apply_rope_ufc on this group's query heads (ops.rs:57-60,77-78)
    const float2* cs = a.lut + (int64_t)min(p, a.max_context - 1) * (HD / 2);
    for (int i = tid; i < n_rep * HD / 2; i += kAttnThreads) {
      const int h = i / (HD / 2), j = i - h * (HD / 2);
      const float x0 = qrow[h * HD + 2 * j], y0 = qrow[h * HD + 2 * j + 1];
      const float2 c = cs[j];
      qs[h * HD + 2 * j] = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(y0, c.y));
      qs[h * HD + 2 * j + 1] = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(y0, c.x));
    }
    if (own) {
      // this KV head's k (rotated, ops.rs:62-65) and v of position p: to the
      // cache (cache.rs:354-368) and to the tile's last row
      const float* kr = a.k_new + (int64_t)r * a.ldk + (int64_t)g * HD;
      const float* vr = a.v_new + (int64_t)r * a.ldv + (int64_t)g * HD;
      float* kc = a.kv.k + hoff + (size_t)(nv - 1) * HD;
      float* vc = a.kv.v + hoff + (size_t)(nv - 1) * HD;
      for (int j = tid; j < HD / 2; j += kAttnThreads) {
        const float x0 = kr[2 * j], y0 = kr[2 * j + 1];
        const float2 c = cs[j];
        const float k0 = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(y0, c.y));
        const float k1 = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(y0, c.x));
        kc[2 * j] = k0;
        kc[2 * j + 1] = k1;
        ks[(nv - 1) * HD + 2 * j] = k0;
        ks[(nv - 1) * HD + 2 * j + 1] = k1;
      }
      for (int i = tid; i < HD; i += kAttnThreads) {
        const float v0 = vr[i];
        vc[i] = v0;
        vs[(nv - 1) * HD + i] = v0;
      }
    }
  } else {
    for (int i = tid; i < n_rep * HD; i += kAttnThreads) qs[i] = qrow[i];
  }
  if (tid == 0) ok_flag = mbar_wait(bar, 0, 0x40) ? 1 : 0;
  __syncthreads();
  if (!ok_flag) {  // the bounded wait gave up (error recorded): let the copies land, then leave
    if (tid == 0) mbar_wait_drain(bar, 0);
    return;
  }
  mbar_test(bar, 0);  // completed: acquire the copied rows in this thread
  // scores: this thread's position against every query head of the group
  {
    float acc[kMaxRep];
#pragma unroll
    for (int j = 0; j < kMaxRep; ++j) acc[j] = 0.f;
    if (tid < nv) {
      const float4* kr = reinterpret_cast<const float4*>(ks + tid * HD);
#pragma unroll 8
      for (int i = 0; i < NC; ++i) {
        const int c = (i + tid) & (NC - 1);
        const float4 k4 = kr[c];
#pragma unroll
        for (int j = 0; j < kMaxRep; ++j) {
          if (j < n_rep) {
            const float4 q4 = reinterpret_cast<const float4*>(qs + j * HD)[c];
            acc[j] = fmaf(q4.x, k4.x, acc[j]);
            acc[j] = fmaf(q4.y, k4.y, acc[j]);
            acc[j] = fmaf(q4.z, k4.z, acc[j]);
            acc[j] = fmaf(q4.w, k4.w, acc[j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kMaxRep; ++j)
      if (j < n_rep) sc[j * kAttnP + tid] = tid < nv ? acc[j] * a.scale : -INFINITY;
  }
  __syncthreads();
  // split max and exp per query head (one warp per head)
  for (int j = warp; j < n_rep; j += kAttnThreads / 32) {
    float* sj = sc + j * kAttnP;
    const float m = warp_max(fmaxf(sj[lane], sj[lane + 32]));
    const float e0 = expf(sj[lane] - m), e1 = expf(sj[lane + 32] - m);  // exp(-inf) = 0 past nv
    sj[lane] = e0;
    sj[lane + 32] = e1;
    const float l = warp_sum(e0 + e1);
    if (lane == 0) {
      mls[2 * j] = m;
      mls[2 * j + 1] = l;
    }
  }
  __syncthreads();
  // sum p v over this warp's 32 positions, lanes owning DL components each
  {
    float acc[kMaxRep][DL];
#pragma unroll
    for (int j = 0; j < kMaxRep; ++j)
#pragma unroll
      for (int c = 0; c < DL; ++c) acc[j][c] = 0.f;
    const int pb = warp * 32, pe = min(pb + 32, nv);
#pragma unroll 4
    for (int t = pb; t < pe; ++t) {
      const float* vr = vs + t * HD + lane * DL;
      float vv[DL];
      if constexpr (DL % 4 == 0) {
#pragma unroll
        for (int c = 0; c < DL; c += 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(vr + c);
          vv[c] = v4.x;
          vv[c + 1] = v4.y;
          vv[c + 2] = v4.z;
          vv[c + 3] = v4.w;
        }
      } else {
        const float2 v2 = *reinterpret_cast<const float2*>(vr);
        vv[0] = v2.x;
        vv[1] = v2.y;
      }
#pragma unroll
      for (int j = 0; j < kMaxRep; ++j) {
        if (j < n_rep) {
          const float pj = sc[j * kAttnP + t];
#pragma unroll
          for (int c = 0; c < DL; ++c) acc[j][c] = fmaf(pj, vv[c], acc[j][c]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kMaxRep; ++j)
      if (j < n_rep)
#pragma unroll
        for (int c = 0; c < DL; ++c) red[(warp * kMaxRep + j) * HD + lane * DL + c] = acc[j][c];
  }
  __syncthreads();
  for (int i = tid; i < n_rep * HD; i += kAttnThreads) {
    const int j = i / HD, d = i - j * HD;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnThreads / 32; ++w) v += red[(w * kMaxRep + j) * HD + d];
    float* rec = a.ws + (((int64_t)r * a.n_heads + g * n_rep + j) * a.n_split + sp) * (HD + 2);
    rec[2 + d] = v;
    if (d == 0) {
      rec[0] = mls[2 * j];
      rec[1] = mls[2 * j + 1];
    }
  }
}

// One CTA of HD threads per (query head, row): out[d] = sum_s e_s acc_s[d] / L
// with e_s = exp(m_s - M), M = max m_s, L = sum e_s l_s.
template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(AttnArgs a, float* out, int64_t ldo) {
  pdl_enter();
  const int h = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
  const int valid_end = attn_valid_end(a, r);
  float* o = out + (int64_t)r * ldo + (int64_t)h * HD;
  if (valid_end < 0) {
    o[d] = 0.f;
    return;
  }
  const int ns = valid_end / kAttnP + 1;
  const float* rec = a.ws + ((int64_t)r * a.n_heads + h) * a.n_split * (HD + 2);
  // unrolled so that the loads of several splits are in flight at once
  float M = -INFINITY;
#pragma unroll 8
  for (int s = 0; s < ns; ++s) M = fmaxf(M, rec[s * (HD + 2)]);
  float L = 0.f, acc = 0.f;
#pragma unroll 8
  for (int s = 0; s < ns; ++s) {
    const float e = expf(rec[s * (HD + 2)] - M);
    L = fmaf(e, rec[s * (HD + 2) + 1], L);
    acc = fmaf(e, rec[s * (HD + 2) + 2 + d], acc);
  }
  o[d] = acc / L;
}

// ------------------------------------------------------- prefill attention
// All prompt positions of a batch of sequences at once (the batched prefill,
// executor.rs:113-141, where the reference attends each position in turn).
// The row of (sequence s, position t) is s * row_stride_seq + t *
// row_stride_pos; position t attends positions 0..t of its own sequence,
// whose K and V rows the cache already holds.
//
// A CTA of 256 threads takes one (sequence, KV head) and a block of QB
// consecutive positions for all n_rep query heads of that KV head (R = n_rep
// x QB <= 96 query rows, Q in shared memory), and walks the keys 0 .. last
// position of the block in tiles of 32, each brought into shared memory by
// two bulk copies. Per tile: scores S = Q K^T * scale for the 128 x 32 block
// (a thread computes 4 rows x 4 keys; the 8 lanes of a shared-memory phase
// start their walk over head_dim at different float4 columns, so the K and
// Q reads of a phase fall in different banks), the causal mask, an online
// softmax update per row (running max and sum; the O rows are rescaled when
// the max moves), then O += P V (a thread holds 4 rows x 4 dims per tile of
// O in registers). Everything in f32: the same products as the split
// kernel, in another summation order.
constexpr int kPfThreads = 256;
constexpr int kPfRows = 96;   // query rows per CTA (n_rep x QB): 2 CTAs fit an SM's shared memory
constexpr int kPfKeys = 32;   // keys per tile

template <int HD>
struct PfSmem {
  static constexpr size_t kQ = 0;                                            // [R][HD]
  static constexpr size_t kK = kQ + (size_t)kPfRows * HD * 4;                // [32][HD]
  static constexpr size_t kV = kK + (size_t)kPfKeys * HD * 4;                // [32][HD]
  static constexpr size_t kS = kV + (size_t)kPfKeys * HD * 4;                // [R][32]
  static constexpr size_t kM = kS + (size_t)kPfRows * kPfKeys * 4;           // running max [R]
  static constexpr size_t kL = kM + (size_t)kPfRows * 4;                     // running sum [R]
  static constexpr size_t kC = kL + (size_t)kPfRows * 4;                     // rescale [R]
  static constexpr size_t kBar = kC + (size_t)kPfRows * 4;
  static constexpr size_t kBytes = kBar + 16;
};

struct PfArgs {
  KvView kv;
  int layer;
  const float* q;
  int64_t ldq;
  float* out;
  int64_t ldo;
  int n_tokens, n_heads, n_rep, qb;  // qb: positions per CTA (R / n_rep)
  int64_t rs_seq, rs_pos;            // row strides
  float scale;
  // key split: CTA (block, chunk) covers key tiles [chunk * chunk_tiles,
  // (chunk + 1) * chunk_tiles); with n_chunks > 1 it writes (max, sum,
  // unnormalised O) per row to ws and attn_prefill_combine_kernel merges
  int n_blocks, n_chunks, chunk_tiles;
  float* ws;  // [seq][kv head][block][chunk][row R][HD + 2]
};

template <int HD>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(PfArgs a) {
  using L = PfSmem<HD>;
  constexpr int NC = HD / 4;
  constexpr int OT = (kPfRows * HD / 16 + kPfThreads - 1) / kPfThreads;  // 4x4 O tiles per thread
  extern __shared__ __align__(128) uint8_t smem[];
  float* Qs = reinterpret_cast<float*>(smem + L::kQ);
  float* Ks = reinterpret_cast<float*>(smem + L::kK);
  float* Vs = reinterpret_cast<float*>(smem + L::kV);
  float* Ss = reinterpret_cast<float*>(smem + L::kS);
  float* Ms = reinterpret_cast<float*>(smem + L::kM);
  float* Ls = reinterpret_cast<float*>(smem + L::kL);
  float* Cs = reinterpret_cast<float*>(smem + L::kC);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBar);
  __shared__ int ok_flag;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache rows come from the previous kernels
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qblk = blockIdx.x / a.n_chunks, ch = blockIdx.x - qblk * a.n_chunks;
  const int g = blockIdx.y, s = blockIdx.z;
  const int n_rep = a.n_rep, qb = a.qb, R = n_rep * qb;
  const int p0 = qblk * qb;
  if (p0 >= a.n_tokens) return;
  const int p1 = min(a.n_tokens, p0 + qb);  // positions p0 .. p1-1
  const int kt0 = ch * a.chunk_tiles;
  if (kt0 * kPfKeys >= p1) return;  // no key of this chunk precedes the block's last position
  // Q rows: row j * qb + i is query head g * n_rep + j at position p0 + i
  for (int e = tid; e < kPfRows * NC; e += kPfThreads) {
    const int row = e / NC, c = e - row * NC;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < R) {
      const int j = row / qb, i = row - j * qb;
      if (p0 + i < p1)
        v = *reinterpret_cast<const float4*>(a.q + (int64_t)s * a.rs_seq * a.ldq + (int64_t)(p0 + i) * a.rs_pos * a.ldq +
                                             (int64_t)(g * n_rep + j) * HD + 4 * c);
    }
    reinterpret_cast<float4*>(Qs)[e] = v;
  }
  for (int r = tid; r < kPfRows; r += kPfThreads) {
    Ms[r] = -INFINITY;
    Ls[r] = 0.f;
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  float o[OT][16];
#pragma unroll
  for (int u = 0; u < OT; ++u)
#pragma unroll
    for (int e = 0; e < 16; ++e) o[u][e] = 0.f;
  __syncthreads();
  const size_t hoff = a.kv.head_off(s, a.layer, g);
  const int n_tiles = min((p1 + kPfKeys - 1) / kPfKeys, kt0 + a.chunk_tiles);
  for (int kt = kt0; kt < n_tiles; ++kt) {
    const uint32_t ph = (uint32_t)(kt - kt0) & 1u;  // this CTA's copy phase
    const int k0 = kt * kPfKeys, nk = min(kPfKeys, p1 - k0);
    if (tid == 0) {
      const uint32_t bytes = (uint32_t)nk * HD * 4;
      mbar_arrive_expect_tx(bar, 2 * bytes);
      bulk_g2s(Ks, a.kv.k + hoff + (size_t)k0 * HD, bytes, bar);
      bulk_g2s(Vs, a.kv.v + hoff + (size_t)k0 * HD, bytes, bar);
      ok_flag = mbar_wait(bar, ph, 0x41) ? 1 : 0;
    }
    __syncthreads();
    if (!ok_flag) {  // the bounded wait gave up (error recorded): let the copies land, then leave
      if (tid == 0) mbar_wait_drain(bar, ph);
      return;
    }
    mbar_test(bar, ph);  // completed: acquire the copied rows in this thread
    // S = Q K^T * scale: tile t -> rows 4 * (t / 8) .., keys 4 * (t % 8) ..
    for (int t = tid; t < (R / 4) * (kPfKeys / 4); t += kPfThreads) {
      const int rg = t >> 3, kg = t & 7;
      float acc[4][4];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
      if (4 * kg < nk) {
#pragma unroll 4
        for (int i = 0; i < NC; ++i) {
          const int c = (i + kg) & (NC - 1);
          float4 qv[4], kv4[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) qv[x] = reinterpret_cast<const float4*>(Qs + (4 * rg + x) * HD)[c];
#pragma unroll
          for (int y = 0; y < 4; ++y) kv4[y] = reinterpret_cast<const float4*>(Ks + (4 * kg + y) * HD)[c];
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              acc[x][y] = fmaf(qv[x].x, kv4[y].x, acc[x][y]);
              acc[x][y] = fmaf(qv[x].y, kv4[y].y, acc[x][y]);
              acc[x][y] = fmaf(qv[x].z, kv4[y].z, acc[x][y]);
              acc[x][y] = fmaf(qv[x].w, kv4[y].w, acc[x][y]);
            }
        }
      }
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int row = 4 * rg + x;
        const int qp = p0 + (row % qb);
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          const int kj = 4 * kg + y, kp = k0 + kj;
          Ss[row * kPfKeys + kj] = (kj < nk && kp <= qp) ? acc[x][y] * a.scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // online softmax: a warp per 16 rows, a lane per key
    for (int row = warp; row < R; row += kPfThreads / 32) {
      const float sv = Ss[row * kPfKeys + lane];
      const float mt = warp_max(sv);
      const float m_old = Ms[row];
      const float m_new = fmaxf(m_old, mt);
      const float pe = m_new == -INFINITY ? 0.f : expf(sv - m_new);
      const float ls = warp_sum(pe);
      Ss[row * kPfKeys + lane] = pe;
      if (lane == 0) {
        const float corr = m_new == -INFINITY ? 1.f : expf(m_old - m_new);  // exp(-inf) = 0 on the first tile
        Cs[row] = corr;
        Ls[row] = Ls[row] * corr + ls;
        Ms[row] = m_new;
      }
    }
    __syncthreads();
    // O = O * corr + P V: O tile u of this thread -> rows 4 * (i / NC) .., dims 4 * (i % NC) ..
#pragma unroll
    for (int u = 0; u < OT; ++u) {
      const int i = tid + u * kPfThreads;
      const int rg = i / NC, dc = i - rg * NC;
      if (4 * rg >= R) continue;
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const float cr = Cs[4 * rg + x];
#pragma unroll
        for (int y = 0; y < 4; ++y) o[u][4 * x + y] *= cr;
      }
      for (int kj = 0; kj < nk; ++kj) {
        const float4 v4 = reinterpret_cast<const float4*>(Vs + kj * HD)[dc];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float p = Ss[(4 * rg + x) * kPfKeys + kj];
          o[u][4 * x + 0] = fmaf(p, v4.x, o[u][4 * x + 0]);
          o[u][4 * x + 1] = fmaf(p, v4.y, o[u][4 * x + 1]);
          o[u][4 * x + 2] = fmaf(p, v4.z, o[u][4 * x + 2]);
          o[u][4 * x + 3] = fmaf(p, v4.w, o[u][4 * x + 3]);
        }
      }
    }
    __syncthreads();  // K, V and S are rewritten by the next tile
  }
  if (a.n_chunks > 1) {
    // partial of this chunk: (m, l, unnormalised O) per row
    float* rec0 = a.ws + ((((int64_t)s * a.kv.n_kv_heads + g) * a.n_blocks + qblk) * a.n_chunks + ch) * R * (HD + 2);
#pragma unroll
    for (int u = 0; u < OT; ++u) {
      const int i = tid + u * kPfThreads;
      const int rg = i / NC, dc = i - rg * NC;
      if (4 * rg >= R) continue;
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        float* rec = rec0 + (int64_t)(4 * rg + x) * (HD + 2);
        if (dc == 0) {
          rec[0] = Ms[4 * rg + x];
          rec[1] = Ls[4 * rg + x];
        }
#pragma unroll
        for (int y = 0; y < 4; ++y) rec[2 + 4 * dc + y] = o[u][4 * x + y];
      }
    }
    return;
  }
  // out = O / l
#pragma unroll
  for (int u = 0; u < OT; ++u) {
    const int i = tid + u * kPfThreads;
    const int rg = i / NC, dc = i - rg * NC;
    if (4 * rg >= R) continue;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int row = 4 * rg + x;
      const int j = row / qb, qi = row - j * qb;
      if (p0 + qi >= p1) continue;
      const float l = Ls[row];
      float* op = a.out + (int64_t)s * a.rs_seq * a.ldo + (int64_t)(p0 + qi) * a.rs_pos * a.ldo +
                  (int64_t)(g * n_rep + j) * HD + 4 * dc;
      *reinterpret_cast<float4*>(op) =
          make_float4(o[u][4 * x] / l, o[u][4 * x + 1] / l, o[u][4 * x + 2] / l, o[u][4 * x + 3] / l);
    }
  }
}

// Merge the key chunks of the prefill: per row, M = max m_c, L = sum
// exp(m_c - M) l_c, out = sum exp(m_c - M) O_c / L (chunks past a row's
// position hold m = -inf, l = 0, O = 0 and add nothing).
template <int HD>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_combine_kernel(PfArgs a) {
  pdl_enter();
  const int qblk = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
  const int n_rep = a.n_rep, qb = a.qb, R = n_rep * qb;
  const int p0 = qblk * qb;
  const int p1 = min(a.n_tokens, p0 + qb);
  const int nch = min(a.n_chunks, ((p1 + kPfKeys - 1) / kPfKeys + a.chunk_tiles - 1) / a.chunk_tiles);
  const float* base = a.ws + (((int64_t)s * a.kv.n_kv_heads + g) * a.n_blocks + qblk) * a.n_chunks * R * (HD + 2);
  const int64_t cstride = (int64_t)R * (HD + 2);
  for (int e = threadIdx.x; e < R * HD; e += kPfThreads) {
    const int row = e / HD, d = e - row * HD;
    const int j = row / qb, qi = row - j * qb;
    if (p0 + qi >= p1) continue;
    const float* rec = base + (int64_t)row * (HD + 2);
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, rec[c * cstride]);
    float L = 0.f, acc = 0.f;
    for (int c = 0; c < nch; ++c) {
      const float m = rec[c * cstride];
      const float w = m == -INFINITY ? 0.f : expf(m - M);
      L = fmaf(w, rec[c * cstride + 1], L);
      acc = fmaf(w, rec[c * cstride + 2 + d], acc);
    }
    a.out[(int64_t)s * a.rs_seq * a.ldo + (int64_t)(p0 + qi) * a.rs_pos * a.ldo + (int64_t)(g * n_rep + j) * HD + d] =
        acc / L;
  }
}

// ------------------------------------------------------------- elementwise
// g = silu(g) * u with silu(v) = v / (1 + exp(-v)) (ops.rs:203-214).
__device__ __forceinline__ float silu_mul1(float v, float u) {
  return __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
}

// VEC = 4: rows of a multiple of 4 elements with 16-byte aligned rows, one
// float4 per step (the same operations per element as VEC = 1).
template <int VEC>
__global__ void silu_mul_kernel(float* g, int64_t ldg, const float* u, int64_t ldu, int n, int64_t total) {
  pdl_enter();
  const int nv = n / VEC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total / VEC; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / nv, c = (i - row * nv) * VEC;
    float* gp = g + row * ldg + c;
    const float* up = u + row * ldu + c;
    if constexpr (VEC == 4) {
      float4 a = *reinterpret_cast<const float4*>(gp);
      const float4 b = *reinterpret_cast<const float4*>(up);
      a.x = silu_mul1(a.x, b.x);
      a.y = silu_mul1(a.y, b.y);
      a.z = silu_mul1(a.z, b.z);
      a.w = silu_mul1(a.w, b.w);
      *reinterpret_cast<float4*>(gp) = a;
    } else {
      *gp = silu_mul1(*gp, *up);
    }
  }
}

// x += y (ops.rs:216-220).
template <int VEC>
__global__ void add_kernel(float* x, int64_t ldx, const float* y, int64_t ldy, int n, int64_t total) {
  pdl_enter();
  const int nv = n / VEC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total / VEC; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / nv, c = (i - row * nv) * VEC;
    float* xp = x + row * ldx + c;
    const float* yp = y + row * ldy + c;
    if constexpr (VEC == 4) {
      float4 a = *reinterpret_cast<const float4*>(xp);
      const float4 b = *reinterpret_cast<const float4*>(yp);
      a.x = __fadd_rn(a.x, b.x);
      a.y = __fadd_rn(a.y, b.y);
      a.z = __fadd_rn(a.z, b.z);
      a.w = __fadd_rn(a.w, b.w);
      *reinterpret_cast<float4*>(xp) = a;
    } else {
      *xp = __fadd_rn(*xp, *yp);
    }
  }
}

// ------------------------------------------------------------------- argmax
// Greedy pick: the index of the largest logit, the LAST one among equals
// (Iterator::max_by keeps the last maximum, sampler.rs:95; -0.0 == +0.0).
// A row holding a NaN, where the reference's partial_cmp().unwrap() panics,
// gives -1.
//
// Each (value, index) becomes one 64-bit key whose unsigned order is the
// pick's order: the float's bits mapped to an order-preserving integer in
// the high half (-0.0 folded onto +0.0), the index in the low half, so the
// largest key is the largest value and, among equal values, the last index.
// CTAs of 256 threads reduce 4096 logits each to one key; the last CTA of a
// row to finish (counted with an atomic) reduces the row's keys, writes the
// pick and resets the row's counter and NaN flag for the next call.
constexpr int kArgThreads = 256;
constexpr int kArgChunk = 4096;

__device__ __forceinline__ unsigned long long arg_key(float v, int i) {
  if (v == 0.f) v = 0.f;  // -0.0 -> +0.0
  const uint32_t b = __float_as_uint(v);
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (uint32_t)i;
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

__device__ __forceinline__ unsigned long long block_max_key(unsigned long long k, unsigned long long* sk) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) k = umax64(k, __shfl_xor_sync(0xffffffffu, k, o));
  if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = k;
  __syncthreads();
  k = 0;
#pragma unroll
  for (int w = 0; w < kArgThreads / 32; ++w) k = umax64(k, sk[w]);
  return k;
}

__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const float* logits, int64_t ld, int n, int n_chunks,
                                                          unsigned long long* keys, unsigned int* counters,
                                                          unsigned int* nan_flags, int32_t* out) {
  __shared__ unsigned long long sk[kArgThreads / 32];
  __shared__ bool last;
  pdl_enter();
  const int cb = blockIdx.x, r = blockIdx.y;
  const float* row = logits + (int64_t)r * ld;
  const int i0 = cb * kArgChunk, i1 = min(n, i0 + kArgChunk);
  unsigned long long k = 0;
  bool nan = false;
  for (int i = i0 + threadIdx.x; i < i1; i += kArgThreads) {
    const float v = row[i];
    nan |= v != v;
    if (v == v) k = umax64(k, arg_key(v, i));
  }
  if (__syncthreads_or(nan) && threadIdx.x == 0) atomicOr(&nan_flags[r], 1u);
  k = block_max_key(k, sk);
  if (threadIdx.x == 0) {
    keys[(int64_t)r * n_chunks + cb] = k;
    __threadfence();
    last = atomicAdd(&counters[r], 1u) == (unsigned)(n_chunks - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  k = 0;
  for (int c = threadIdx.x; c < n_chunks; c += kArgThreads)
    k = umax64(k, __ldcg(&keys[(int64_t)r * n_chunks + c]));
  k = block_max_key(k, sk);
  if (threadIdx.x == 0) {
    const bool any_nan = __ldcg(&nan_flags[r]) != 0;
    out[r] = any_nan ? -1 : (k == 0 ? n - 1 : (int32_t)(k & 0xFFFFFFFFu));
    counters[r] = 0;
    nan_flags[r] = 0;
  }
}

// ---------------------------------------------------------------- embedding
// out[r] = row tokens[r] of the dequantized table (bit-exact with swamp-gguf's
// dequant, which the reference applies to the whole table at load,
// executor.rs:212).
__global__ void embed_kernel(SgDevWeight w, const int32_t* tokens, float* out, int64_t ldo) {
  pdl_enter();
  const int r = blockIdx.y;
  const int64_t k0 = 8 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (k0 >= w.n_cols) return;
  const int tok = tokens[r];
  float* o = out + (int64_t)r * ldo + k0;
  if (tok < 0 || tok >= w.n_rows) {
    if (k0 == 0) sg_set_error(SG_DEVERR_BAD_INPUT);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
    return;
  }
  float v[8];
  dequant8(w, tok, k0, v);
  reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

unsigned ew_grid(int64_t total, int num_sms) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)num_sms * 8));
}

}  // namespace ops

namespace {
// The single device that the op entry points run on.
int op_device(DevState** out) {
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device entry points need one device per process");
  *out = &g_ctx.devs[0];
  CUDA_TRY(cudaSetDevice((*out)->device));
  return SG_OK;
}

ops::KvView kv_view(const sg_kv_cache_s* c) {
  return ops::KvView{c->n_layers, c->n_kv_heads, c->head_dim, c->max_seq, c->n_seqs, c->k, c->v};
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int HD>
int attention_launch(const ops::AttnArgs& a, dim3 g1, dim3 g2, float* out, int64_t ldo, cudaStream_t st) {
  static int attr_done[64] = {0};
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !attr_done[dev]) {
    CUDA_TRY(cudaFuncSetAttribute(ops::attn_split_kernel<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)ops::AttnSmem<HD>::kBytes));
    CUDA_TRY(cudaFuncSetAttribute(ops::attn_split_kernel<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)ops::AttnSmem<HD>::kBytes));
    attr_done[dev] = 1;
  }
  if (a.lut) {  // decode form: RoPE and the cache store inside the split kernel
    CUDA_TRY(ops::launch(ops::attn_split_kernel<HD, true>, g1, dim3(ops::kAttnThreads), ops::AttnSmem<HD>::kBytes, st,
                         a));
  } else {
    CUDA_TRY(ops::launch(ops::attn_split_kernel<HD, false>, g1, dim3(ops::kAttnThreads), ops::AttnSmem<HD>::kBytes,
                         st, a));
  }
  CUDA_TRY(ops::launch(ops::attn_combine_kernel<HD>, g2, dim3(HD), 0, st, a, out, ldo));
  return SG_OK;
}
// (declared beside run_linear in sg_api.cu)
// The rows of a GEMV prologue, for the calls that do not fuse it (prefill
// GEMM, Q6_K): the same kernels as sg_rmsnorm_device / sg_silu_mul_device.
int apply_prologue(DevState& d, const SgGemvPrologue& pro, const float* x, int64_t ldx, int64_t K, int batch,
                   float* out, cudaStream_t st) {
  if (pro.kind == SG_PRO_RMSNORM) {
    CUDA_TRY(ops::launch(ops::rmsnorm_kernel, dim3(batch), dim3(ops::kNormThreads), 0, st, x, ldx, pro.w, out,
                         (int64_t)K, (int)K, pro.eps));
    return SG_OK;
  }
  CUDA_TRY(cudaMemcpy2DAsync(out, (size_t)K * sizeof(float), x, (size_t)ldx * sizeof(float), (size_t)K * sizeof(float),
                             batch, cudaMemcpyDeviceToDevice, st));
  const int64_t total = K * batch;
  if (K % 4 == 0 && pro.ldx2 % 4 == 0 && aligned16(pro.x2))
    CUDA_TRY(ops::launch(ops::silu_mul_kernel<4>, dim3(ops::ew_grid(total / 4, d.num_sms)), dim3(256), 0, st, out,
                         (int64_t)K, pro.x2, pro.ldx2, (int)K, total));
  else
    CUDA_TRY(ops::launch(ops::silu_mul_kernel<1>, dim3(ops::ew_grid(total, d.num_sms)), dim3(256), 0, st, out,
                         (int64_t)K, pro.x2, pro.ldx2, (int)K, total));
  return SG_OK;
}

}  // namespace

extern "C" {

int sg_rope_create(int head_dim, int max_context, sg_rope_t* out) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (head_dim < 2 || (head_dim & 1) || max_context < 1)
    return fail(SG_ERR_INVALID_ARG, "head_dim %d must be even and >= 2, max_context %d >= 1", head_dim, max_context);
  // init_rope_lut (ops.rs:27-36) in f32 with the host libm the reference
  // calls (powf, cosf, sinf), so the table is the reference's bit for bit
  const int half = head_dim / 2;
  std::vector<float2> lut((size_t)max_context * half);
  const float theta = 10000.0f;
  for (int k = 0; k < half; ++k) {
    const float e = (float)(2 * k) / (float)head_dim;
    const float freq = 1.0f / powf(theta, e);
    for (int m = 0; m < max_context; ++m) {
      const float angle = (float)m * freq;
      lut[(size_t)m * half + k] = make_float2(cosf(angle), sinf(angle));
    }
  }
  auto* r = new sg_rope_s();
  r->head_dim = head_dim;
  r->max_context = max_context;
  r->device = d->device;
  if (cudaMalloc(&r->lut, lut.size() * sizeof(float2)) != cudaSuccess) {
    cudaGetLastError();
    delete r;
    return fail(SG_ERR_OOM, "cannot allocate the RoPE table");
  }
  cudaError_t e = cudaMemcpy(r->lut, lut.data(), lut.size() * sizeof(float2), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(r->lut);
    delete r;
    return fail(SG_ERR_CUDA, "RoPE table upload: %s", cudaGetErrorString(e));
  }
  *out = r;
  return SG_OK;
}

int sg_rope_free(sg_rope_t r) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!r) return fail(SG_ERR_INVALID_ARG, "null handle");
  cudaSetDevice(r->device);
  cudaFree(r->lut);
  delete r;
  return SG_OK;
}

int sg_rope_table(sg_rope_t r, float* dst) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!r || !dst) return fail(SG_ERR_INVALID_ARG, "null pointer");
  CUDA_TRY(cudaSetDevice(r->device));
  CUDA_TRY(cudaMemcpy(dst, r->lut, (size_t)r->max_context * (r->head_dim / 2) * sizeof(float2), cudaMemcpyDeviceToHost));
  return SG_OK;
}

int sg_kv_cache_create(int n_layers, int n_kv_heads, int head_dim, int max_seq, int n_seqs, sg_kv_cache_t* out) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (n_layers < 1 || n_kv_heads < 1 || head_dim < 1 || max_seq < 1 || n_seqs < 1 || (head_dim & 3))
    return fail(SG_ERR_INVALID_ARG, "bad cache geometry (layers %d, kv heads %d, head_dim %d (multiple of 4), max_seq %d, seqs %d)",
                n_layers, n_kv_heads, head_dim, max_seq, n_seqs);
  auto* c = new sg_kv_cache_s();
  c->n_layers = n_layers;
  c->n_kv_heads = n_kv_heads;
  c->head_dim = head_dim;
  c->max_seq = max_seq;
  c->n_seqs = n_seqs;
  c->device = d->device;
  const size_t bytes = c->head_off(n_seqs, 0, 0) * sizeof(float);
  if (cudaMalloc(&c->k, bytes) != cudaSuccess || cudaMalloc(&c->v, bytes) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(c->k);
    delete c;
    return fail(SG_ERR_OOM, "cannot allocate 2 x %zu bytes of KV cache", bytes);
  }
  // pages start zeroed like the reference's alloc_zeroed pages (cache.rs:136)
  cudaError_t e = cudaMemset(c->k, 0, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->v, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->k);
    cudaFree(c->v);
    delete c;
    return fail(SG_ERR_CUDA, "KV cache clear: %s", cudaGetErrorString(e));
  }
  *out = c;
  return SG_OK;
}

int sg_kv_cache_free(sg_kv_cache_t c) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!c) return fail(SG_ERR_INVALID_ARG, "null handle");
  cudaSetDevice(c->device);
  cudaFree(c->k);
  cudaFree(c->v);
  delete c;
  return SG_OK;
}

int sg_kv_cache_ptr(sg_kv_cache_t c, int seq, int layer, int kv_head, float** k, float** v) {
  if (!c || !k || !v) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (seq < 0 || seq >= c->n_seqs || layer < 0 || layer >= c->n_layers || kv_head < 0 || kv_head >= c->n_kv_heads)
    return fail(SG_ERR_INVALID_ARG, "seq %d / layer %d / kv head %d out of range", seq, layer, kv_head);
  *k = c->k + c->head_off(seq, layer, kv_head);
  *v = c->v + c->head_off(seq, layer, kv_head);
  return SG_OK;
}

int sg_rmsnorm_device(const float* x, int64_t ldx, const float* weight, float* out, int64_t ldo, int n, int rows,
                      float eps, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (rows < 0 || n < 1 || ldx < n || ldo < n) return fail(SG_ERR_INVALID_ARG, "bad sizes (n %d, rows %d)", n, rows);
  if (!x || !weight || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (rows == 0) return SG_OK;
  CUDA_TRY(ops::launch(ops::rmsnorm_kernel, dim3(rows), dim3(ops::kNormThreads), 0, (cudaStream_t)stream, x, ldx, weight,
                       out, ldo, n, eps));
  return SG_OK;
}


int sg_rope_kv_device(sg_rope_t rope, sg_kv_cache_t cache, int layer, float* q, int64_t ldq, float* k, int64_t ldk,
                      const float* v, int64_t ldv, const int32_t* pos, const int32_t* seq, int rows, int n_q_heads,
                      void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!cache || !k || !v || !pos || (rope && !q)) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (layer < 0 || layer >= cache->n_layers) return fail(SG_ERR_INVALID_ARG, "layer %d out of range", layer);
  if (rows < 0) return fail(SG_ERR_INVALID_ARG, "negative rows");
  const int hd = cache->head_dim, nkv = cache->n_kv_heads;
  if (ldk < (int64_t)nkv * hd || ldv < (int64_t)nkv * hd)
    return fail(SG_ERR_INVALID_ARG, "k/v row stride below n_kv_heads * head_dim");
  if (rope) {
    if (rope->head_dim != hd) return fail(SG_ERR_INVALID_ARG, "RoPE head_dim %d != cache head_dim %d", rope->head_dim, hd);
    if (n_q_heads < 1 || ldq < (int64_t)n_q_heads * hd) return fail(SG_ERR_INVALID_ARG, "bad q heads / stride");
  }
  if (rows == 0) return SG_OK;
  const float2* lut = rope ? rope->lut : nullptr;
  CUDA_TRY(ops::launch(ops::rope_kv_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream, lut,
                       rope ? rope->max_context : 1, kv_view(cache), layer, q, ldq, k, ldk, v, ldv, pos, seq, n_q_heads));
  return SG_OK;
}

int sg_attention_device(sg_kv_cache_t cache, int layer, const float* q, int64_t ldq, float* out, int64_t ldo,
                        const int32_t* pos, const int32_t* seq_len, const int32_t* seq, int rows, int n_heads,
                        void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!cache || !q || !out || !pos) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (layer < 0 || layer >= cache->n_layers) return fail(SG_ERR_INVALID_ARG, "layer %d out of range", layer);
  const int hd = cache->head_dim, nkv = cache->n_kv_heads;
  if (hd != 64 && hd != 128 && hd != 256) return fail(SG_ERR_UNSUPPORTED, "head_dim %d (64, 128 or 256)", hd);
  if (n_heads < nkv || n_heads % nkv || n_heads / nkv > ops::kMaxRep)
    return fail(SG_ERR_UNSUPPORTED, "n_heads %d over %d KV heads (a multiple, at most %d per KV head)", n_heads, nkv,
                ops::kMaxRep);
  if (rows < 0 || ldq < (int64_t)n_heads * hd || ldo < (int64_t)n_heads * hd)
    return fail(SG_ERR_INVALID_ARG, "bad rows or strides");
  if (!aligned16(q) || (ldq & 3)) return fail(SG_ERR_INVALID_ARG, "q must be 16-byte aligned with ldq % 4 == 0");
  if (rows == 0) return SG_OK;
  ops::AttnArgs a = {};
  a.kv = kv_view(cache);
  a.layer = layer;
  a.q = q;
  a.ldq = ldq;
  a.pos = pos;
  a.seq_len = seq_len;
  a.seq = seq;
  a.n_heads = n_heads;
  a.n_rep = n_heads / nkv;
  a.n_split = (cache->max_seq + ops::kAttnP - 1) / ops::kAttnP;
  a.scale = 1.0f / sqrtf((float)hd);  // ops.rs:93
  const size_t ws_bytes = (size_t)rows * n_heads * a.n_split * (hd + 2) * sizeof(float);
  rc = ensure_buf((void**)&d->attn_ws, &d->attn_ws_bytes, ws_bytes);
  if (rc) return rc;
  a.ws = d->attn_ws;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 g1(a.n_split, nkv, rows), g2(n_heads, rows);
  switch (hd) {
    case 64:
      rc = attention_launch<64>(a, g1, g2, out, ldo, st);
      break;
    case 128:
      rc = attention_launch<128>(a, g1, g2, out, ldo, st);
      break;
    default:
      rc = attention_launch<256>(a, g1, g2, out, ldo, st);
  }
  return rc;
}

int sg_rope_attention_device(sg_rope_t rope, sg_kv_cache_t cache, int layer, const float* q, int64_t ldq, const float* k,
                             int64_t ldk, const float* v, int64_t ldv, float* out, int64_t ldo, const int32_t* pos,
                             const int32_t* seq, int rows, int n_heads, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!rope || !cache || !q || !k || !v || !out || !pos) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (layer < 0 || layer >= cache->n_layers) return fail(SG_ERR_INVALID_ARG, "layer %d out of range", layer);
  const int hd = cache->head_dim, nkv = cache->n_kv_heads;
  if (rope->head_dim != hd) return fail(SG_ERR_INVALID_ARG, "RoPE head_dim %d != cache head_dim %d", rope->head_dim, hd);
  if (hd != 64 && hd != 128 && hd != 256) return fail(SG_ERR_UNSUPPORTED, "head_dim %d (64, 128 or 256)", hd);
  if (n_heads < nkv || n_heads % nkv || n_heads / nkv > ops::kMaxRep)
    return fail(SG_ERR_UNSUPPORTED, "n_heads %d over %d KV heads (a multiple, at most %d per KV head)", n_heads, nkv,
                ops::kMaxRep);
  if (rows < 0 || ldq < (int64_t)n_heads * hd || ldo < (int64_t)n_heads * hd || ldk < (int64_t)nkv * hd ||
      ldv < (int64_t)nkv * hd)
    return fail(SG_ERR_INVALID_ARG, "bad rows or strides");
  if (!aligned16(q) || (ldq & 3)) return fail(SG_ERR_INVALID_ARG, "q must be 16-byte aligned with ldq % 4 == 0");
  if (rows > cache->n_seqs)
    return fail(SG_ERR_INVALID_ARG, "%d rows > %d sequences (one row per sequence)", rows, cache->n_seqs);
  if (rows == 0) return SG_OK;
  ops::AttnArgs a = {};
  a.kv = kv_view(cache);
  a.layer = layer;
  a.q = q;
  a.ldq = ldq;
  a.pos = pos;
  a.seq_len = nullptr;
  a.seq = seq;
  a.n_heads = n_heads;
  a.n_rep = n_heads / nkv;
  a.n_split = (cache->max_seq + ops::kAttnP - 1) / ops::kAttnP;
  a.scale = 1.0f / sqrtf((float)hd);  // ops.rs:93
  a.lut = rope->lut;
  a.max_context = rope->max_context;
  a.k_new = k;
  a.ldk = ldk;
  a.v_new = v;
  a.ldv = ldv;
  rc = ensure_buf((void**)&d->attn_ws, &d->attn_ws_bytes, (size_t)rows * n_heads * a.n_split * (hd + 2) * sizeof(float));
  if (rc) return rc;
  a.ws = d->attn_ws;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 g1(a.n_split, nkv, rows), g2(n_heads, rows);
  switch (hd) {
    case 64:
      return attention_launch<64>(a, g1, g2, out, ldo, st);
    case 128:
      return attention_launch<128>(a, g1, g2, out, ldo, st);
    default:
      return attention_launch<256>(a, g1, g2, out, ldo, st);
  }
}

int sg_attention_prefill_device(sg_kv_cache_t cache, int layer, const float* q, int64_t ldq, float* out, int64_t ldo,
                                int n_seqs, int n_tokens, int64_t row_stride_seq, int64_t row_stride_pos, int n_heads,
                                void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!cache || !q || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (layer < 0 || layer >= cache->n_layers) return fail(SG_ERR_INVALID_ARG, "layer %d out of range", layer);
  const int hd = cache->head_dim, nkv = cache->n_kv_heads;
  if (hd != 64 && hd != 128) return fail(SG_ERR_UNSUPPORTED, "prefill attention: head_dim %d (64 or 128)", hd);
  if (n_heads < nkv || n_heads % nkv || n_heads / nkv > ops::kMaxRep)
    return fail(SG_ERR_UNSUPPORTED, "n_heads %d over %d KV heads (a multiple, at most %d per KV head)", n_heads, nkv,
                ops::kMaxRep);
  if (n_seqs < 0 || n_seqs > cache->n_seqs || n_tokens < 0 || n_tokens > cache->max_seq)
    return fail(SG_ERR_INVALID_ARG, "%d sequences x %d tokens outside the cache (%d x %d)", n_seqs, n_tokens,
                cache->n_seqs, cache->max_seq);
  if (row_stride_seq < 0 || row_stride_pos < 0 || ldq < (int64_t)n_heads * hd || ldo < (int64_t)n_heads * hd)
    return fail(SG_ERR_INVALID_ARG, "bad strides");
  if (!aligned16(q) || (ldq & 3) || !aligned16(out) || (ldo & 3))
    return fail(SG_ERR_INVALID_ARG, "q and out must be 16-byte aligned with row strides that are multiples of 4");
  if (n_seqs == 0 || n_tokens == 0) return SG_OK;
  ops::PfArgs a = {};
  a.kv = kv_view(cache);
  a.layer = layer;
  a.q = q;
  a.ldq = ldq;
  a.out = out;
  a.ldo = ldo;
  a.n_tokens = n_tokens;
  a.n_heads = n_heads;
  a.n_rep = n_heads / nkv;
  a.qb = (ops::kPfRows / a.n_rep) & ~3;  // positions per CTA: n_rep x qb <= 96 rows, whole 4-row groups
  a.rs_seq = row_stride_seq;
  a.rs_pos = row_stride_pos;
  a.scale = 1.0f / sqrtf((float)hd);  // ops.rs:93
  // With fewer CTAs than two per SM, split the keys into chunks of 4 tiles
  // (128 keys), so that the last query blocks (the longest causal rows)
  // spread over several CTAs; with more, the blocks alone fill the GPU and
  // the split only adds the partials' traffic (measured at 512 tokens: one
  // sequence 282 -> 223 us per layer with the split, eight 956 -> 1175 us).
  a.n_blocks = (n_tokens + a.qb - 1) / a.qb;
  const int n_kt = (n_tokens + ops::kPfKeys - 1) / ops::kPfKeys;
  const bool split = (int64_t)a.n_blocks * nkv * n_seqs < 2 * (int64_t)d->num_sms;
  a.chunk_tiles = split ? 4 : n_kt;
  a.n_chunks = (n_kt + a.chunk_tiles - 1) / a.chunk_tiles;
  if (a.n_chunks > 1) {
    const size_t need = (size_t)n_seqs * nkv * a.n_blocks * a.n_chunks * (a.n_rep * a.qb) * (hd + 2) * sizeof(float);
    rc = ensure_buf((void**)&d->attn_ws, &d->attn_ws_bytes, need);
    if (rc) return rc;
    a.ws = d->attn_ws;
  }
  const dim3 grid((unsigned)(a.n_blocks * a.n_chunks), (unsigned)nkv, (unsigned)n_seqs);
  const dim3 cgrid((unsigned)a.n_blocks, (unsigned)nkv, (unsigned)n_seqs);
  cudaStream_t st = (cudaStream_t)stream;
  static int attr_done[64][2] = {};
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (hd == 64) {
    if (dev < 64 && !attr_done[dev][0]) {
      CUDA_TRY(cudaFuncSetAttribute(ops::attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ops::PfSmem<64>::kBytes));
      attr_done[dev][0] = 1;
    }
    CUDA_TRY(ops::launch(ops::attn_prefill_kernel<64>, grid, dim3(ops::kPfThreads), ops::PfSmem<64>::kBytes, st, a));
    if (a.n_chunks > 1) CUDA_TRY(ops::launch(ops::attn_prefill_combine_kernel<64>, cgrid, dim3(ops::kPfThreads), 0, st, a));
  } else {
    if (dev < 64 && !attr_done[dev][1]) {
      CUDA_TRY(cudaFuncSetAttribute(ops::attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)ops::PfSmem<128>::kBytes));
      attr_done[dev][1] = 1;
    }
    CUDA_TRY(ops::launch(ops::attn_prefill_kernel<128>, grid, dim3(ops::kPfThreads), ops::PfSmem<128>::kBytes, st, a));
    if (a.n_chunks > 1) CUDA_TRY(ops::launch(ops::attn_prefill_combine_kernel<128>, cgrid, dim3(ops::kPfThreads), 0, st, a));
  }
  return SG_OK;
}

int sg_silu_mul_device(float* g, int64_t ldg, const float* u, int64_t ldu, int n, int rows, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!g || !u) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (n < 1 || rows < 0 || ldg < n || ldu < n) return fail(SG_ERR_INVALID_ARG, "bad sizes");
  const int64_t total = (int64_t)n * rows;
  if (total == 0) return SG_OK;
  if (n % 4 == 0 && ldg % 4 == 0 && ldu % 4 == 0 && aligned16(g) && aligned16(u))
    CUDA_TRY(ops::launch(ops::silu_mul_kernel<4>, dim3(ops::ew_grid(total / 4, d->num_sms)), dim3(256), 0,
                         (cudaStream_t)stream, g, ldg, u, ldu, n, total));
  else
    CUDA_TRY(ops::launch(ops::silu_mul_kernel<1>, dim3(ops::ew_grid(total, d->num_sms)), dim3(256), 0,
                         (cudaStream_t)stream, g, ldg, u, ldu, n, total));
  return SG_OK;
}

int sg_add_device(float* x, int64_t ldx, const float* y, int64_t ldy, int n, int rows, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!x || !y) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (n < 1 || rows < 0 || ldx < n || ldy < n) return fail(SG_ERR_INVALID_ARG, "bad sizes");
  const int64_t total = (int64_t)n * rows;
  if (total == 0) return SG_OK;
  if (n % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && aligned16(x) && aligned16(y))
    CUDA_TRY(ops::launch(ops::add_kernel<4>, dim3(ops::ew_grid(total / 4, d->num_sms)), dim3(256), 0,
                         (cudaStream_t)stream, x, ldx, y, ldy, n, total));
  else
    CUDA_TRY(ops::launch(ops::add_kernel<1>, dim3(ops::ew_grid(total, d->num_sms)), dim3(256), 0,
                         (cudaStream_t)stream, x, ldx, y, ldy, n, total));
  return SG_OK;
}

int sg_argmax_device(const float* logits, int64_t ld, int n, int rows, int32_t* out, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  if (!logits || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (n < 1 || rows < 0 || ld < n) return fail(SG_ERR_INVALID_ARG, "bad sizes");
  if (rows == 0) return SG_OK;
  // row counters and NaN flags first (zero between calls: the last CTA of a
  // row resets them; their place depends only on the row), then chunk keys
  const int n_chunks = (n + ops::kArgChunk - 1) / ops::kArgChunk;
  const int cap = std::max(rows, d->argmax_rows);
  const size_t need = (size_t)cap * 8 + (size_t)rows * n_chunks * 8;
  if (d->argmax_ws_bytes < need || rows > d->argmax_rows) {
    size_t have = d->argmax_ws_bytes;
    if (rows > d->argmax_rows) have = 0;  // the flags region grows: start over
    rc = ensure_buf(&d->argmax_ws, &have, need);
    if (rc) return rc;
    d->argmax_ws_bytes = have;
    d->argmax_rows = cap;
    CUDA_TRY(cudaMemset(d->argmax_ws, 0, d->argmax_ws_bytes));
  }
  auto* counters = static_cast<unsigned int*>(d->argmax_ws);
  auto* nan_flags = counters + d->argmax_rows;
  auto* keys = reinterpret_cast<unsigned long long*>(counters + 2 * (size_t)d->argmax_rows);
  CUDA_TRY(ops::launch(ops::argmax_kernel, dim3(n_chunks, rows), dim3(ops::kArgThreads), 0, (cudaStream_t)stream, logits,
                       ld, n, n_chunks, keys, counters, nan_flags, out));
  return SG_OK;
}

int sg_embed_device(sg_weight_t table, const int32_t* tokens, int rows, float* out, int64_t ldo, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  DevState* d = nullptr;
  int rc = op_device(&d);
  if (rc) return rc;
  rc = validate_weight(table);
  if (rc) return rc;
  if (table->tp_mode != SG_TP_REPLICATE && g_ctx.world > 1)
    return fail(SG_ERR_INVALID_ARG, "the embedding table must be replicated");
  if (!tokens || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  const SgDevWeight& w = table->shards[0].w;
  if (rows < 0 || ldo < w.n_cols) return fail(SG_ERR_INVALID_ARG, "bad rows or ldo");
  if (!aligned16(out) || (ldo & 3)) return fail(SG_ERR_INVALID_ARG, "out must be 16-byte aligned with ldo % 4 == 0");
  if (rows == 0) return SG_OK;
  const int64_t per_row = w.n_cols / 8;
  const dim3 grid((unsigned)((per_row + 127) / 128), (unsigned)rows);
  CUDA_TRY(ops::launch(ops::embed_kernel, grid, dim3(128), 0, (cudaStream_t)stream, w, tokens, out, ldo));
  return SG_OK;
}

}  // extern "C"
