// sg_layout.cuh -- the device-resident weight layout.
//
// A registered GGUF tensor (swamp-gguf layout: row-major, each row a run of
// 18-byte Q4_0 or 144-byte Q4_K blocks; TensorInfo.shape[0] = n_cols = K,
// shape[1] = n_rows = N, swamp-gguf/src/tensor_info.rs:10-16) is repacked
// once, losslessly, into a tile layout that every kernel streams directly:
//
//   row-block  = 128 rows (N padded to 128); one row per dequantizing thread
//   chunk      = 64 consecutive K (Q4_0 K padded to 64 with zero-scale blocks)
//   tile       = one (row-block, chunk): 4608 contiguous bytes, tiles ordered
//                row-block major, so a row-block's K run is one contiguous span
//
//   tile bytes [0, 4096): nibbles [half 2][row 128][word 4] uint32
//       word w of (half h, row r) holds the 8 nibbles of K = 64*chunk + 32h +
//       8w + j, j = 0..7, nibble j at bit 16*(j&1) + 4*(j>>1). A thread reads
//       its row's 32 K as one 16-byte vector, and four lop3 per word (plus
//       one shift by 8) turn it into f16 pairs (1024+q) for j = 0,1,4,5 and
//       (1024+16q) for j = 2,3,6,7 without any further shifting.
//   tile bytes [4096, 4608): one 32-bit scale word per row
//       Q4_0: f16 bits of d(block 0) | d(block 1) << 16, the chunk's two
//             32-blocks
//       Q4_K: bytes (sc_a, sc_b, m_a, m_b) of the chunk's two 32-element
//             sub-blocks a = 2*(chunk%4), b = a+1, unpacked from the 12-byte
//             6-bit form
//   Q4_K dd [rb][superblock][row 128] uint32: d | dmin << 16 (512 B)
//
// Q4_0 keeps exactly 18 B per 32 weights. Q4_K stores 148 B per 256 weights
// instead of 144 (the 6-bit scale/min pairs are kept one byte each so the
// kernels skip the unpack); roofline bytes are still counted at 144.
//
// Q6_K (6-bit q, 16-element sub-blocks with int8 scales, f16 d per 256;
// swamp-gguf/src/quant/q6_k.rs) uses 6656-byte tiles:
//   [0, 4096)    the low 4 bits of q, exactly as the Q4 nibble words
//   [4096, 6144) the high 2 bits: [half 2][row 128][word 2]; word i covers
//                nibble words 2i and 2i+1; its byte b holds, for the bytes b
//                that one mask makes of each nibble word (K offsets {0,4,1,5}
//                of the low nibbles, {2,6,3,7} of the high ones), the high
//                bits of word 2i's low / high nibble at bits 0-1 / 2-3 and of
//                word 2i+1's at bits 4-5 / 6-7 -- two masks and a shift put
//                them next to the nibbles
//   [6144, 6656) one word per row: the int8 scales of the chunk's four
//                16-element sub-blocks
//   dd [rb][superblock][row 128] uint32: the f16 d (low half)
// 208 B per 256 weights instead of 210.
#pragma once
#include "sg_common.cuh"

#define SG_TILE_BYTES 4608
#define SG_TILE_SC_OFF 4096
#define SG_TILE6_BYTES 6656
#define SG_TILE6_HI_OFF 4096
#define SG_TILE6_SC_OFF 6144

__host__ __device__ constexpr int sg_tile_bytes(int dtype) { return dtype == SG_DTYPE_Q6_K ? SG_TILE6_BYTES : SG_TILE_BYTES; }

struct SgDevWeight {
  int dtype;
  int64_t n_rows, n_cols;  // logical sizes of this shard (N, K)
  int64_t n_rb, n_ch, n_sb;
  uint8_t* tiles;  // n_rb * n_ch * sg_tile_bytes(dtype)
  uint32_t* dd;    // Q4_K, Q6_K: uint32[n_rb*n_sb*128]; Q4_0: nullptr
};

// Bit position of nibble j (0..7) inside its 32-bit word.
__host__ __device__ constexpr int sg_nib_pos(int j) { return 16 * (j & 1) + 4 * (j >> 1); }

// Q6_K: position of the high 2 bits of (k-in-chunk kk) in the high plane:
// word index (of the row's two per half) and bit offset
__host__ __device__ constexpr int sg_q6_hi_word(int kk) { return (kk & 31) >> 4; }
__host__ __device__ constexpr int sg_q6_hi_bit(int kk) {
  return 8 * (((kk & 1) << 1) | ((kk >> 2) & 1)) + 2 * ((kk >> 1) & 1) + 4 * ((kk >> 3) & 1);
}

// Nibble at (row-in-block r, k-in-chunk kk) inside one tile.
__device__ __forceinline__ uint32_t tile_nibble(const uint8_t* tile, int r, int kk) {
  const int h = kk >> 5, w = (kk >> 3) & 3, j = kk & 7;
  const uint32_t word = reinterpret_cast<const uint32_t*>(tile)[(h * 128 + r) * 4 + w];
  return (word >> sg_nib_pos(j)) & 15u;
}

#ifdef __cplusplus
// host-side launchers (sg_layout.cu)
int sg_layout_alloc(SgDevWeight* w, int dtype, int64_t n_rows, int64_t n_cols);
void sg_layout_free(SgDevWeight* w);
cudaError_t sg_layout_repack(const SgDevWeight* w, const uint8_t* raw_dev, cudaStream_t st);
cudaError_t sg_layout_dequant(const SgDevWeight* w, float* dst, int64_t ld, cudaStream_t st);
size_t sg_layout_bytes(int dtype, int64_t n_rows, int64_t n_cols);
#endif
