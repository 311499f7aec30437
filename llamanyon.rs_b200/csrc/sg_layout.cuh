// sg_layout.cuh -- the device-resident weight layout.
//
// A registered GGUF tensor (swamp-gguf layout: row-major, each row a run of
// 18-byte Q4_0 or 144-byte Q4_K blocks; TensorInfo.shape[0] = n_cols = K,
// shape[1] = n_rows = N, swamp-gguf/src/tensor_info.rs:10-16) is repacked
// once, losslessly, into a tile layout that both kernels stream directly:
//
//   row-block  = 128 rows (N padded to 128), row-tile = 16 rows (the mma M)
//   chunk      = 64 consecutive K (Q4_0 K padded to 64 with zero-scale blocks)
//   tile       = one (row-block, chunk): 4608 contiguous bytes, tiles ordered
//                row-block major, so a row-block's K run is one contiguous span
//
//   tile bytes [0, 4096): nibbles [rt 8][lane 32][s 4] uint32
//       lane = 4g + t. Word s holds the 8 nibbles of one m16n8k16 A fragment
//       for k16-step s: bit 4p..4p+3 = q(row 16rt + g + 8*(p&1),
//       k = 64*chunk + 16s + 2t + 8*((p>>1)&1) + ((p>>2)&1)), so a warp's
//       512 B per row-tile is one 16-byte vector per lane and a fragment
//       decodes with shifts and lop3.
//   tile bytes [4096, 4608): scales [rt 8][g 8][2] (32-bit each)
//       Q4_0: two f16 d per word: [blk 2][hl 2] -> word0 = (d(blk0,g), d(blk0,g+8)),
//             word1 = (d(blk1,g), d(blk1,g+8)); blk = the chunk's 32-block
//       Q4_K: word hl (row g + 8hl) = bytes (sc_a, sc_b, m_a, m_b) of the
//             chunk's two 32-element sub-blocks a = 2*(chunk%4), b = a+1,
//             unpacked from the 12-byte 6-bit form
//   Q4_K dd [rb][superblock][rt 8][g 8][hl 2] uint32: d | dmin << 16 (512 B)
//
// Q4_0 keeps exactly 18 B per 32 weights. Q4_K stores 148 B per 256 weights
// instead of 144 (the 6-bit scale/min pairs are kept one byte each so the
// kernels skip the unpack); roofline bytes are still counted at 144.
#pragma once
#include "sg_common.cuh"

#define SG_TILE_BYTES 4608
#define SG_TILE_SC_OFF 4096

struct SgDevWeight {
  int dtype;
  int64_t n_rows, n_cols;  // logical sizes of this shard (N, K)
  int64_t n_rb, n_ch, n_sb;
  uint8_t* tiles;  // n_rb * n_ch * SG_TILE_BYTES
  uint32_t* dd;    // Q4_K: uint32[n_rb*n_sb*128]; Q4_0: nullptr
};

// Nibble at (row-in-block r, k-in-chunk kk) inside one tile.
__device__ __forceinline__ uint32_t tile_nibble(const uint8_t* tile, int r, int kk) {
  const int rt = r >> 4, rr = r & 15, g = rr & 7, hl = rr >> 3;
  const int s = kk >> 4, k16 = kk & 15, hi8 = k16 >> 3, t = (k16 & 7) >> 1, j = k16 & 1;
  const uint32_t w = reinterpret_cast<const uint32_t*>(tile)[(rt * 32 + (4 * g + t)) * 4 + s];
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
