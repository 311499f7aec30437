// sg_layout.cu -- repack GGUF Q4_0/Q4_K blocks into the device tile layout,
// and the bit-exact dequantizer that reads the tile layout back to f32.
//
// Dequant arithmetic follows swamp-gguf exactly:
//   Q4_0 (swamp-gguf/src/quant/q4_0.rs:24-35):  w = (float)(q - 8) * d
//   Q4_K (swamp-gguf/src/quant/q4_k.rs:297-317): w = RN(RN(d*sc) * q) - RN(dmin*m)
// with no FMA contraction, so the result is the reference's f32 bit pattern.
#include "sg_layout.cuh"

namespace {

__device__ __forceinline__ uint32_t raw_nibble(int dtype, const uint8_t* raw, int64_t n_rows, int64_t n_cols,
                                               int64_t row, int64_t k) {
  if (row >= n_rows || k >= n_cols) return 0u;
  if (dtype == SG_DTYPE_Q4_0) {
    const int64_t nb = n_cols / 32;
    const int64_t b = k >> 5;
    const int i = (int)(k & 31);
    const uint8_t byte = raw[(row * nb + b) * 18 + 2 + (i >> 1)];  // q4_0.rs:31
    return (i & 1) ? (byte >> 4) : (byte & 15u);                    // q4_0.rs:32
  } else if (dtype == SG_DTYPE_Q6_K) {
    // the low 4 bits of q (q6_k.rs:33-36): element 128h + 32m + l of a block
    const int64_t nsb = n_cols / 256;
    const int e = (int)(k & 255), h = e >> 7, m = (e >> 5) & 3, l = e & 31;
    const uint8_t byte = raw[(row * nsb + (k >> 8)) * 210 + 64 * h + l + 32 * (m & 1)];
    return (byte >> (4 * (m >> 1))) & 15u;
  } else {
    const int64_t nsb = n_cols / 256;
    const int64_t sb = k >> 8;
    const int e = (int)(k & 255), p = e >> 6, h = (e >> 5) & 1, i = e & 31;
    const uint8_t byte = raw[(row * nsb + sb) * 144 + 16 + 32 * p + i];  // q4_k.rs:292,302,315
    return h ? (byte >> 4) : (byte & 15u);
  }
}

// one thread per (tile, half, row): the 16-byte nibble vector of that row
__global__ void repack_qs_kernel(int dtype, const uint8_t* __restrict__ raw, int64_t n_rows, int64_t n_cols,
                                 int64_t n_rb, int64_t n_ch, uint8_t* __restrict__ tiles) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n_rb * n_ch * 256;
  if (tid >= total) return;
  const int r = (int)(tid & 127);
  const int h = (int)((tid >> 7) & 1);
  const int64_t tile = tid >> 8;  // rb * n_ch + c
  const int64_t rb = tile / n_ch, c = tile % n_ch;
  const int64_t row = rb * 128 + r;
  uint32_t words[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t k = c * 64 + 32 * h + 8 * w + j;
      v |= raw_nibble(dtype, raw, n_rows, n_cols, row, k) << sg_nib_pos(j);
    }
    words[w] = v;
  }
  *reinterpret_cast<uint4*>(tiles + tile * sg_tile_bytes(dtype) + (h * 128 + r) * 16) =
      make_uint4(words[0], words[1], words[2], words[3]);
}

// Q6_K high 2-bit plane: one thread per (tile, half, row), two words
__global__ void repack_q6_hi_kernel(const uint8_t* __restrict__ raw, int64_t n_rows, int64_t n_cols, int64_t n_rb,
                                    int64_t n_ch, uint8_t* __restrict__ tiles) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n_rb * n_ch * 256;
  if (tid >= total) return;
  const int r = (int)(tid & 127), h = (int)((tid >> 7) & 1);
  const int64_t tile = tid >> 8, rb = tile / n_ch, c = tile % n_ch;
  const int64_t row = rb * 128 + r;
  uint32_t words[2] = {0u, 0u};
  if (row < n_rows) {
    const int64_t nsb = n_cols / 256;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
      const int kk = 32 * h + i;
      const int64_t k = c * 64 + kk;
      const int e = (int)(k & 255), hb = e >> 7, m = (e >> 5) & 3, l = e & 31;
      const uint8_t qh = raw[(row * nsb + (k >> 8)) * 210 + 128 + 32 * hb + l];  // q6_k.rs:33-36
      words[sg_q6_hi_word(kk)] |= (uint32_t)((qh >> (2 * m)) & 3u) << sg_q6_hi_bit(kk);
    }
  }
  reinterpret_cast<uint2*>(tiles + tile * SG_TILE6_BYTES + SG_TILE6_HI_OFF)[h * 128 + r] = make_uint2(words[0], words[1]);
}

// unpack_scales (swamp-gguf/src/quant/q4_k.rs:37-53)
__device__ __forceinline__ void q4k_unpack(const uint8_t* s, int j, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = s[j] & 63u;
    m = s[j + 4] & 63u;
  } else {
    sc = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
    m = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
  }
}

// one thread per (tile, row): the row's scale word
__global__ void repack_scales_kernel(int dtype, const uint8_t* __restrict__ raw, int64_t n_rows, int64_t n_cols,
                                     int64_t n_rb, int64_t n_ch, uint8_t* __restrict__ tiles) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n_rb * n_ch * 128;
  if (tid >= total) return;
  const int r = (int)(tid & 127);
  const int64_t tile = tid >> 7, rb = tile / n_ch, c = tile % n_ch;
  const int64_t row = rb * 128 + r;
  uint32_t out = 0;
  if (row < n_rows && dtype == SG_DTYPE_Q6_K) {
    // the int8 scales of the chunk's four 16-element sub-blocks (q6_k.rs:37-46:
    // element e of a block uses sc[e / 16])
    const uint8_t* blk = raw + (row * (n_cols / 256) + (c >> 2)) * 210 + 192 + 4 * (c & 3);
    out = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) | ((uint32_t)blk[3] << 24);
  } else if (row < n_rows) {
    if (dtype == SG_DTYPE_Q4_0) {
      const int64_t nb = n_cols / 32;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const int64_t b = c * 2 + blk;
        if (b < nb) {
          const uint8_t* p = raw + (row * nb + b) * 18;  // q4_0.rs:24
          out |= ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << (16 * blk);
        }
      }
    } else {
      const int64_t nsb = n_cols / 256;
      const uint8_t* blk = raw + (row * nsb + (c >> 2)) * 144;
      const int a = 2 * (int)(c & 3);
      uint32_t sa, ma, sb, mb;
      q4k_unpack(blk + 4, a, sa, ma);
      q4k_unpack(blk + 4, a + 1, sb, mb);
      out = sa | (sb << 8) | (ma << 16) | (mb << 24);
    }
  }
  if (dtype == SG_DTYPE_Q6_K) reinterpret_cast<uint32_t*>(tiles + tile * SG_TILE6_BYTES + SG_TILE6_SC_OFF)[r] = out;
  else reinterpret_cast<uint32_t*>(tiles + tile * SG_TILE_BYTES + SG_TILE_SC_OFF)[r] = out;
}

// Q4_K d|dmin, Q6_K d: one thread per (rb, superblock, row); bytes = block bytes.
__global__ void repack_q4k_dd_kernel(const uint8_t* __restrict__ raw, int64_t n_rows, int64_t n_cols,
                                     int64_t n_rb, int64_t n_sb, uint32_t* __restrict__ dd, int bytes) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n_rb * n_sb * 128;
  if (tid >= total) return;
  const int r = (int)(tid & 127);
  const int64_t tile = tid >> 7, rb = tile / n_sb, sb = tile % n_sb;
  const int64_t row = rb * 128 + r;
  uint32_t out = 0;
  if (row < n_rows && bytes == 144) {
    const uint8_t* blk = raw + (row * n_sb + sb) * 144;  // q4_k.rs:281-282
    out = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) | ((uint32_t)blk[3] << 24);
  } else if (row < n_rows) {
    const uint8_t* blk = raw + (row * n_sb + sb) * 210;  // q6_k.rs:28: d at 208
    out = (uint32_t)blk[208] | ((uint32_t)blk[209] << 8);
  }
  dd[tid] = out;
}

// The 8 weights k0 .. k0+7 (k0 % 8 == 0) of one row, bit-exact.
__device__ __forceinline__ void dequant8(const SgDevWeight& w, int64_t row, int64_t k0, float out[8]) {
  const int64_t rb = row >> 7;
  const int r = (int)(row & 127);
  const int64_t c = k0 >> 6;
  const int kk0 = (int)(k0 & 63);
  const uint8_t* tile = w.tiles + (rb * w.n_ch + c) * sg_tile_bytes(w.dtype);
  if (w.dtype == SG_DTYPE_Q6_K) {
    // q6_k.rs:37-46: w = d * (f32)sc * (f32)(q - 32), both products exact
    const uint32_t scw = reinterpret_cast<const uint32_t*>(tile + SG_TILE6_SC_OFF)[r];
    const uint32_t ddw = w.dd[(rb * w.n_sb + (c >> 2)) * 128 + r];
    const float d = __half2float(__ushort_as_half((unsigned short)(ddw & 0xFFFFu)));
    const uint2 hw = reinterpret_cast<const uint2*>(tile + SG_TILE6_HI_OFF)[(kk0 >> 5) * 128 + r];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int kk = kk0 + i;
      const uint32_t hword = sg_q6_hi_word(kk) ? hw.y : hw.x;
      const int q = (int)(tile_nibble(tile, r, kk) | (((hword >> sg_q6_hi_bit(kk)) & 3u) << 4));
      const float sc = (float)(int8_t)(scw >> (8 * ((kk & 63) >> 4)));
      out[i] = __fmul_rn(__fmul_rn(d, sc), (float)(q - 32));
    }
    return;
  }
  const uint32_t scw = reinterpret_cast<const uint32_t*>(tile + SG_TILE_SC_OFF)[r];
  if (w.dtype == SG_DTYPE_Q4_0) {
    const uint32_t dw = (kk0 >> 5) ? (scw >> 16) : (scw & 0xFFFFu);
    const float d = __half2float(__ushort_as_half((unsigned short)dw));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = (int)tile_nibble(tile, r, kk0 + i);
      out[i] = __fmul_rn((float)(q - 8), d);
    }
  } else {
    const uint32_t scm = scw;
    const uint32_t ddw = w.dd[(rb * w.n_sb + (c >> 2)) * 128 + r];
    const float d = __half2float(__ushort_as_half((unsigned short)(ddw & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(ddw >> 16)));
    const int sub = kk0 >> 5;
    const float sv = __fmul_rn(d, (float)((scm >> (8 * sub)) & 0xFFu));
    const float mv = __fmul_rn(dmin, (float)((scm >> (16 + 8 * sub)) & 0xFFu));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = (int)tile_nibble(tile, r, kk0 + i);
      out[i] = __fsub_rn(__fmul_rn(sv, (float)q), mv);
    }
  }
}

// Dequantize 8 consecutive k of one row per thread.
__global__ void dequant_kernel(SgDevWeight w, float* __restrict__ dst, int64_t ld) {
  const int64_t kq = w.n_cols / 8;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= w.n_rows * kq) return;
  const int64_t row = tid / kq;
  const int64_t k0 = (tid % kq) * 8;
  float out[8];
  dequant8(w, row, k0, out);
  float4* o = reinterpret_cast<float4*>(dst + row * ld + k0);
  o[0] = make_float4(out[0], out[1], out[2], out[3]);
  o[1] = make_float4(out[4], out[5], out[6], out[7]);
}

inline unsigned nblocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

size_t sg_layout_bytes(int dtype, int64_t n_rows, int64_t n_cols) {
  const int64_t n_rb = (n_rows + 127) / 128;
  const int64_t n_ch = (n_cols + 63) / 64;
  size_t b = (size_t)(n_rb * n_ch) * sg_tile_bytes(dtype);
  if (dtype == SG_DTYPE_Q4_K || dtype == SG_DTYPE_Q6_K) b += (size_t)(n_rb * (n_cols / 256)) * 512;
  return b;
}

int sg_layout_alloc(SgDevWeight* w, int dtype, int64_t n_rows, int64_t n_cols) {
  w->dtype = dtype;
  w->n_rows = n_rows;
  w->n_cols = n_cols;
  w->n_rb = (n_rows + 127) / 128;
  w->n_ch = (n_cols + 63) / 64;
  w->n_sb = dtype == SG_DTYPE_Q4_K || dtype == SG_DTYPE_Q6_K ? n_cols / 256 : 0;
  w->tiles = nullptr;
  w->dd = nullptr;
  const size_t tile_bytes = (size_t)(w->n_rb * w->n_ch) * sg_tile_bytes(dtype);
  const size_t dd_bytes = (size_t)(w->n_rb * w->n_sb) * 512;
  if (cudaMalloc(&w->tiles, tile_bytes) != cudaSuccess) return -1;
  if (dd_bytes && cudaMalloc(&w->dd, dd_bytes) != cudaSuccess) {
    sg_layout_free(w);
    return -1;
  }
  return 0;
}

void sg_layout_free(SgDevWeight* w) {
  if (w->tiles) cudaFree(w->tiles);
  if (w->dd) cudaFree(w->dd);
  w->tiles = nullptr;
  w->dd = nullptr;
}

cudaError_t sg_layout_repack(const SgDevWeight* w, const uint8_t* raw_dev, cudaStream_t st) {
  const int T = 256;
  const int64_t nq = w->n_rb * w->n_ch * 256;
  repack_qs_kernel<<<nblocks(nq, T), T, 0, st>>>(w->dtype, raw_dev, w->n_rows, w->n_cols, w->n_rb, w->n_ch,
                                                 w->tiles);
  const int64_t ns = w->n_rb * w->n_ch * 128;
  repack_scales_kernel<<<nblocks(ns, T), T, 0, st>>>(w->dtype, raw_dev, w->n_rows, w->n_cols, w->n_rb, w->n_ch,
                                                     w->tiles);
  if (w->dtype == SG_DTYPE_Q6_K)
    repack_q6_hi_kernel<<<nblocks(nq, T), T, 0, st>>>(raw_dev, w->n_rows, w->n_cols, w->n_rb, w->n_ch, w->tiles);
  if (w->dtype == SG_DTYPE_Q4_K || w->dtype == SG_DTYPE_Q6_K) {
    const int64_t nd = w->n_rb * w->n_sb * 128;
    repack_q4k_dd_kernel<<<nblocks(nd, T), T, 0, st>>>(raw_dev, w->n_rows, w->n_cols, w->n_rb, w->n_sb, w->dd,
                                                         w->dtype == SG_DTYPE_Q4_K ? 144 : 210);
  }
  return cudaGetLastError();
}

cudaError_t sg_layout_dequant(const SgDevWeight* w, float* dst, int64_t ld, cudaStream_t st) {
  const int T = 256;
  const int64_t n = w->n_rows * (w->n_cols / 8);
  if (n == 0) return cudaSuccess;
  dequant_kernel<<<nblocks(n, T), T, 0, st>>>(*w, dst, ld);
  return cudaGetLastError();
}
