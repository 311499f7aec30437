// sg_layout.cuh -- the device-resident weight layout.
//
// A registered GGUF tensor (swamp-gguf layout: row-major, each row a run of
// 18-byte Q4_0 or 144-byte Q4_K blocks; TensorInfo.shape[0] = n_cols = K,
// shape[1] = n_rows = N, swamp-gguf/src/tensor_info.rs:10-16) is repacked
// once, losslessly, into a tile layout that both kernels stream directly:
//
//   row-block  = 128 rows (N padded to 128), row-tile = 16 rows (the mma M)
//   chunk      = 64 consecutive K (Q4_0 K padded to 64 with zero-scale blocks)
//
//   qs  [rb][chunk][rt 8][lane 32][s 4] uint32   4096 B per (rb, chunk)
//       lane = 4g + t. Word s holds the 8 nibbles of one m16n8k16 A fragment
//       for k16-step s: bit 4p..4p+3 = q(row 16rt + g + 8*(p&1),
//       k = 64*chunk + 16s + 2t + 8*((p>>1)&1) + ((p>>2)&1)), so a warp's
//       512 B load per row-tile is one coalesced 16 B per lane and a fragment
//       decodes with one shift and four lop3 ops.
//   Q4_0 scales  [rb][chunk][rt 8][g 8][blk 2][hl 2] fp16 (d of the 32-block
//       blk of the chunk, row 16rt+g+8hl)                  512 B per (rb, chunk)
//   Q4_K scm     [rb][chunk][rt 8][g 8][hl 2] uint32: bytes (sc_a, sc_b, m_a,
//       m_b) of the chunk's two 32-element sub-blocks a = 2*(chunk%4), b = a+1,
//       already unpacked from the 12-byte 6-bit form      512 B per (rb, chunk)
//   Q4_K dd      [rb][superblock][rt 8][g 8][hl 2] uint32: d | dmin << 16
//                                                          512 B per (rb, sb)
//
// Q4_0 keeps exactly 18 B per 32 weights. Q4_K stores 148 B per 256 weights
// instead of 144 (the 6-bit scale/min pairs are kept one byte each so the
// kernels skip the unpack); roofline bytes are still counted at 144.
#pragma once
#include "sg_common.cuh"

struct SgDevWeight {
  int dtype;
  int64_t n_rows, n_cols;  // logical sizes of this shard (N, K)
  int64_t n_rb, n_ch, n_sb;
  uint32_t* qs;  // n_rb * n_ch * 1024 words
  void* sc;      // Q4_0: __half[n_rb*n_ch*256]; Q4_K: uint32[n_rb*n_ch*128]
  uint32_t* dd;  // Q4_K: uint32[n_rb*n_sb*128]; Q4_0: nullptr
};

// Decode one packed-nibble word into the four f16x2 A-fragment registers of
// m16n8k16, values (q - bias). 1024+q is built by OR-ing q into the mantissa
// of 1024.0h; the upper nibble of each byte lands as 1024+16q and is rescaled
// by an exact fma.
__device__ __forceinline__ void decode_frag(uint32_t w, uint32_t bias_lo, uint32_t bias_hi, uint32_t a[4]) {
  const uint32_t w8 = w >> 8;
  uint32_t r0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  uint32_t r1 = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  uint32_t r2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  uint32_t r3 = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
  const uint32_t sixteenth = 0x2C002C00u;  // 1/16 in both halves
  asm("sub.f16x2 %0, %1, %2;" : "=r"(a[0]) : "r"(r0), "r"(bias_lo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a[1]) : "r"(r1), "r"(sixteenth), "r"(bias_hi));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(a[2]) : "r"(r2), "r"(bias_lo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a[3]) : "r"(r3), "r"(sixteenth), "r"(bias_hi));
}

// bias constants: lo-nibble path subtracts (1024 + c); hi-nibble path computes
// (1024+16q)/16 - (64 + c) = q - c. Q4_0 uses c = 8, Q4_K c = 0.
#define SG_BIAS_LO_Q4_0 0x64086408u  // 1032.0h
#define SG_BIAS_HI_Q4_0 0xD480D480u  // -72.0h
#define SG_BIAS_LO_Q4_K 0x64006400u  // 1024.0h
#define SG_BIAS_HI_Q4_K 0xD400D400u  // -64.0h

// Nibble at (row-in-block r, k-in-chunk kk) inside one (rb, chunk) tile.
__device__ __forceinline__ uint32_t tile_nibble(const uint32_t* tile, int r, int kk) {
  const int rt = r >> 4, rr = r & 15, g = rr & 7, hl = rr >> 3;
  const int s = kk >> 4, k16 = kk & 15, hi8 = k16 >> 3, t = (k16 & 7) >> 1, j = k16 & 1;
  const uint32_t w = tile[(rt * 32 + (4 * g + t)) * 4 + s];
  const int sh = (j ? 16 : 0) + (hi8 ? 8 : 0) + (hl ? 4 : 0);
  return (w >> sh) & 15u;
}

#ifdef __cplusplus
// host-side launchers (sg_layout.cu)
int sg_layout_alloc(SgDevWeight* w, int dtype, int64_t n_rows, int64_t n_cols);
void sg_layout_free(SgDevWeight* w);
cudaError_t sg_layout_repack(const SgDevWeight* w, const uint8_t* raw_dev, cudaStream_t st);
cudaError_t sg_layout_dequant(const SgDevWeight* w, float* dst, int64_t ld, cudaStream_t st);
size_t sg_layout_bytes(int dtype, int64_t n_rows, int64_t n_cols);
#endif
