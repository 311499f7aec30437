// sg_synth.cu -- seeded synthetic GGUF tensors and activations.
//
// The benchmark configurations use random-init weights in the GGUF block
// formats (Q4_0: d uniform in [0.001, 0.01), nibbles uniform 0..15; Q4_K: d,
// dmin in that range, 6-bit scales and mins uniform, packed as
// make_q4k_block does, swamp-kernels/src/fused_gemv_q4k.rs:708-724; Q6_K: int8
// scales and 6-bit values uniform, packed as q6_k.rs:33-46 reads them) and
// N(0,1) activations. Every value is a function of (seed, tensor id, index)
// through splitmix64, so any slice can be regenerated anywhere: the device
// kernel below writes exactly the bytes that the host generator of the test
// oracle writes, and a tensor-parallel shard generates only its own blocks.
//
// Scale draws: u = (24 random bits) * 2^-24, v = 0.001 + 0.009 * u in f32
// (multiply, then add, each rounded), then f16 round-to-nearest-even.

namespace synth {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t draw(uint64_t seed, uint64_t id, uint64_t i) {
  return splitmix64(seed ^ (id << 40) ^ i);
}

// binary32 -> binary16, round to nearest even, for the normal range the
// scale draws occupy (2^-14 <= v < 65520): keep 10 mantissa bits and round on
// the 13 dropped ones.
__device__ __forceinline__ uint16_t f16_bits_rne(float v) {
  const uint32_t x = __float_as_uint(v);
  const uint32_t e = ((x >> 23) & 0xFFu) - 127u + 15u;
  uint32_t h = (e << 10) | ((x >> 13) & 0x3FFu);
  const uint32_t rem = x & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)h;
}

__device__ __forceinline__ uint16_t scale_f16(uint64_t bits24) {
  const float u = (float)(uint32_t)bits24 * (1.0f / 16777216.0f);  // exact
  const float v = __fadd_rn(0.001f, __fmul_rn(0.009f, u));
  return f16_bits_rne(v);
}

// The block is assembled in registers and written with 16-bit stores (every
// block starts on an even byte).
template <int BYTES>
__device__ __forceinline__ void store_block(uint8_t* dst, const uint8_t (&b)[BYTES]) {
  uint16_t* d16 = reinterpret_cast<uint16_t*>(dst);
#pragma unroll
  for (int i = 0; i < BYTES / 2; ++i) d16[i] = (uint16_t)(b[2 * i] | (b[2 * i + 1] << 8));
}

// One thread per GGUF block of the shard: block (row0 + r, cb0 + c) of the
// full tensor, whose global index row * nblk + cb keys its draws.
__global__ void gen_blocks_kernel(int dtype, uint64_t seed, uint64_t id, int64_t nblk, int64_t row0, int64_t nr,
                                  int64_t cb0, int64_t ncb, uint8_t* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nr * ncb) return;
  const int64_t r = t / ncb, c = t - r * ncb;
  const uint64_t b = (uint64_t)((row0 + r) * nblk + cb0 + c);
  if (dtype == SG_DTYPE_Q4_0) {
    uint8_t blk[18];
    const uint64_t r0 = draw(seed, id, 4 * b), r1 = draw(seed, id, 4 * b + 1), r2 = draw(seed, id, 4 * b + 2);
    const uint16_t d = scale_f16(r0 >> 40);
    blk[0] = (uint8_t)d;
    blk[1] = (uint8_t)(d >> 8);
    // nibble i of the block is draw bits 4i.. of r1 (i < 16) or r2; byte j
    // holds nibbles 2j (low) and 2j+1 (high), q4_0.rs:31-32
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint64_t src = j < 8 ? r1 : r2;
      const int i = (2 * j) & 15;
      blk[2 + j] = (uint8_t)(((src >> (4 * i)) & 15) | (((src >> (4 * (i + 1))) & 15) << 4));
    }
    store_block(out + t * 18, blk);
  } else if (dtype == SG_DTYPE_Q4_K) {
    uint8_t blk[144];
    const uint64_t base = 32 * b;
    const uint64_t r0 = draw(seed, id, base), r1 = draw(seed, id, base + 1), r2 = draw(seed, id, base + 2);
    const uint16_t d = scale_f16(r0 >> 40), dm = scale_f16((r0 >> 16) & 0xFFFFFFull);
    uint8_t sc[8], mn[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sc[j] = (uint8_t)((r1 >> (6 * j)) & 63);
      mn[j] = (uint8_t)((r2 >> (6 * j)) & 63);
    }
    blk[0] = (uint8_t)d;
    blk[1] = (uint8_t)(d >> 8);
    blk[2] = (uint8_t)dm;
    blk[3] = (uint8_t)(dm >> 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // the inverse of unpack_scales, q4_k.rs:37-53
      blk[4 + j] = (uint8_t)(sc[j] | ((sc[4 + j] >> 4) << 6));
      blk[8 + j] = (uint8_t)(mn[j] | ((mn[4 + j] >> 4) << 6));
      blk[12 + j] = (uint8_t)((sc[4 + j] & 15) | ((mn[4 + j] & 15) << 4));
    }
    // element e's nibble is bits 4(e%16).. of draw base+3+e/16; byte 32p+i of
    // qs holds elements 64p+i (low) and 64p+32+i (high), q4_k.rs:291-319
    for (int p = 0; p < 4; ++p) {
      const uint64_t lo0 = draw(seed, id, base + 3 + 4 * p), lo1 = draw(seed, id, base + 4 + 4 * p);
      const uint64_t hi0 = draw(seed, id, base + 5 + 4 * p), hi1 = draw(seed, id, base + 6 + 4 * p);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t lo = i < 16 ? lo0 : lo1, hi = i < 16 ? hi0 : hi1;
        blk[16 + 32 * p + i] = (uint8_t)(((lo >> (4 * (i & 15))) & 15) | (((hi >> (4 * (i & 15))) & 15) << 4));
      }
    }
    store_block(out + t * 144, blk);
  } else {  // Q6_K
    uint8_t blk[210];
    const uint64_t base = 40 * b;
    const uint64_t r0 = draw(seed, id, base), r1 = draw(seed, id, base + 1), r2 = draw(seed, id, base + 2);
    const uint16_t d = scale_f16(r0 >> 40);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      blk[192 + j] = (uint8_t)(r1 >> (8 * j));
      blk[200 + j] = (uint8_t)(r2 >> (8 * j));
    }
    blk[208] = (uint8_t)d;
    blk[209] = (uint8_t)(d >> 8);
    // value e = 128h + 32m + l is bits 6(e%8).. of draw base+3+e/8; its low
    // nibble goes to ql[64h + l + 32(m&1)] (shift 4(m>>1)), its high 2 bits
    // to qh[32h + l] (shift 2m), q6_k.rs:33-46
    for (int h = 0; h < 2; ++h) {
      for (int l = 0; l < 32; ++l) {
        uint32_t q[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int e = 128 * h + 32 * m + l;
          q[m] = (uint32_t)((draw(seed, id, base + 3 + (uint64_t)(e >> 3)) >> (6 * (e & 7))) & 63);
        }
        blk[64 * h + l] = (uint8_t)((q[0] & 15) | ((q[2] & 15) << 4));
        blk[64 * h + l + 32] = (uint8_t)((q[1] & 15) | ((q[3] & 15) << 4));
        blk[128 + 32 * h + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
      }
    }
    store_block(out + t * 210, blk);
  }
}

cudaError_t gen_blocks(int dtype, uint64_t seed, uint64_t id, int64_t nblk, int64_t row0, int64_t nr, int64_t cb0,
                       int64_t ncb, uint8_t* out, cudaStream_t st) {
  const int64_t n = nr * ncb;
  if (n == 0) return cudaSuccess;
  const int T = 128;
  gen_blocks_kernel<<<(unsigned)((n + T - 1) / T), T, 0, st>>>(dtype, seed, id, nblk, row0, nr, cb0, ncb, out);
  return cudaGetLastError();
}

}  // namespace synth

namespace {
struct SynthFill : RawFill {
  int dtype;
  uint64_t seed, id;
  int64_t nblk;
  cudaError_t fill(DevState& d, uint8_t* raw, int64_t row0, int64_t nr, int64_t cb0, int64_t ncb) override {
    return synth::gen_blocks(dtype, seed, id, nblk, row0, nr, cb0, ncb, raw, d.stream);
  }
};
}  // namespace

extern "C" {

int sg_synth_weight(int dtype, uint64_t seed, uint64_t tensor_id, int64_t n_rows, int64_t n_cols, int tp_mode,
                    sg_weight_t* out) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  SynthFill f;
  f.dtype = dtype;
  f.seed = seed;
  f.id = tensor_id;
  f.nblk = n_cols / std::max<int64_t>(1, block_of(dtype));
  return register_weight(f, dtype, n_rows, n_cols, tp_mode, out);
}

int sg_synth_blocks(int dtype, uint64_t seed, uint64_t tensor_id, int64_t n_rows, int64_t n_cols, void* dst,
                    int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (!dst) return fail(SG_ERR_INVALID_ARG, "null dst");
  int64_t r0, nr, c0, nc;
  int rc = shard_plan(dtype, n_rows, n_cols, SG_TP_REPLICATE, 1, 0, &r0, &nr, &c0, &nc);
  if (rc) return rc;
  DevState& d = g_ctx.devs[0];
  CUDA_TRY(cudaSetDevice(d.device));
  const int64_t nblk = n_cols / block_of(dtype);
  const size_t bytes = (size_t)(n_rows * nblk) * block_bytes(dtype);
  uint8_t* out = static_cast<uint8_t*>(dst);
  if (!(flags & SG_FLAG_DEVICE_PTRS)) {
    rc = ensure_buf((void**)&d.ybuf, &d.ybuf_bytes, bytes);
    if (rc) return rc;
    out = reinterpret_cast<uint8_t*>(d.ybuf);
  }
  CUDA_TRY(synth::gen_blocks(dtype, seed, tensor_id, nblk, 0, n_rows, 0, nblk, out, d.stream));
  if (!(flags & SG_FLAG_DEVICE_PTRS)) CUDA_TRY(cudaMemcpyAsync(dst, out, bytes, cudaMemcpyDeviceToHost, d.stream));
  CUDA_TRY(cudaStreamSynchronize(d.stream));
  return SG_OK;
}

int sg_synth_x(uint64_t seed, uint64_t tensor_id, int64_t n, float* dst) {
  if (!dst || n < 0) return fail(SG_ERR_INVALID_ARG, "bad arguments");
  // N(0,1) by Box-Muller in double from two draws per pair, rounded once to f32
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t j = 0; 2 * j < n; ++j) {
    const uint64_t ra = synth::draw(seed, tensor_id, 2 * (uint64_t)j);
    const uint64_t rb = synth::draw(seed, tensor_id, 2 * (uint64_t)j + 1);
    const double u1 = ((double)(ra >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(rb >> 11) * (1.0 / 9007199254740992.0);
    const double rad = std::sqrt(-2.0 * std::log(u1));
    dst[2 * j] = (float)(rad * std::cos(two_pi * u2));
    if (2 * j + 1 < n) dst[2 * j + 1] = (float)(rad * std::sin(two_pi * u2));
  }
  return SG_OK;
}

}  // extern "C"
