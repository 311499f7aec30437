// sg_tc.cuh -- Blackwell tensor-core plumbing shared by the decode GEMV and
// the prefill GEMM: UMMA shared-memory/instruction descriptors, tcgen05.mma
// (kind::f16: bf16 or f16 operands, f32 accumulate, one CTA), commit, TMEM allocation and loads, and the
// host-side TMA tensor-map encoder (resolved through the runtime's driver
// entry point, so the library links no libcuda).
#pragma once
#include <cuda.h>

#include <mutex>

#include "sg_common.cuh"

// ---------------------------------------------------------------- descriptors
// UMMA shared-memory descriptor for a K-major operand tile with 8-row atoms:
// SWIZZLE_64B (rows of 64 B, atoms 512 B apart) or SWIZZLE_128B (rows of
// 128 B, atoms 1024 B apart). The tile base must be aligned to the atom.
enum SgSwizzle { SG_SW64 = 4, SG_SW128 = 2 };

__device__ __forceinline__ uint64_t sg_sdesc(uint32_t saddr, SgSwizzle sw) {
  const uint32_t sbo = sw == SG_SW128 ? 1024u : 512u;
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;  // stride byte offset between 8-row atoms
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)sw << 61;                // swizzle mode
  return d;
}

// instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major
__host__ __device__ constexpr uint32_t sg_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major
__host__ __device__ constexpr uint32_t sg_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// instruction descriptor: kind::i8, A = u8, B = s8, D = s32, both K-major
__host__ __device__ constexpr uint32_t sg_idesc_u8s8(int M, int N) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// kind::i8 MMA (K = 32 bytes per instruction), A in tensor memory (M lanes x
// K/4 columns, 4 consecutive K bytes per 32-bit column), B in shared memory
__device__ __forceinline__ void sg_umma_i8_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// the same, issued only when `issue` is nonzero (a predicate instead of a
// branch: the issuing thread runs straight-line code)
__device__ __forceinline__ void sg_umma_i8_tmem_a_if(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                     uint32_t accumulate, uint32_t issue) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 q, %5, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(issue));
}

__device__ __forceinline__ void sg_umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// same, with the A operand in tensor memory (M lanes x K/2 columns of f16 pairs)
__device__ __forceinline__ void sg_umma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// arrive on bar once every tcgen05.mma this thread issued so far has completed
__device__ __forceinline__ void sg_umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void sg_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void sg_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ------------------------------------------------------------------- TMEM
// whole-warp calls; ncols a power of two >= 32
__device__ __forceinline__ void sg_tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void sg_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// 32 lanes x 16 / 32 consecutive 32-bit columns (lane quadrant = warp % 4)
__device__ __forceinline__ void sg_tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void sg_tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
// 32 lanes x N consecutive 32-bit columns, N in {1, 2, 4, 8, 16, 32}
template <int N>
__device__ __forceinline__ void sg_tmem_ld_n(uint32_t taddr, uint32_t (&v)[N]) {
  if constexpr (N == 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v[0]) : "r"(taddr));
  } else if constexpr (N == 2) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "r"(taddr));
  } else if constexpr (N == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
  } else if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
  } else if constexpr (N == 16) {
    sg_tmem_ld16(taddr, v);
  } else {
    static_assert(N == 32, "tcgen05.ld width");
    sg_tmem_ld32(taddr, v);
  }
}

__device__ __forceinline__ void sg_tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns from registers (lane quadrant = warp % 4)
__device__ __forceinline__ void sg_tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
// 32 lanes x N consecutive 32-bit columns from registers, N in {1, 4, 8}
template <int N>
__device__ __forceinline__ void sg_tmem_st_n(uint32_t taddr, const uint32_t (&v)[N]) {
  if constexpr (N == 1) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v[0]) : "memory");
  } else if constexpr (N == 4) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
  } else {
    static_assert(N == 8, "tcgen05.st width");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
  }
}

// 32 lanes x 16 consecutive 32-bit columns from registers
__device__ __forceinline__ void sg_tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void sg_tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------- nibble decoding
// f16 pairs from one layout word (nibble j at bit 16*(j&1) + 4*(j>>1)):
//   .x = (1024+q0, 1024+q1),    .y = (1024+16*q2, 1024+16*q3),
//   .z = (1024+q4, 1024+q5),    .w = (1024+16*q6, 1024+16*q7)   (low half first)
// 0x6400 is f16 1024, whose unit in the last place is 1, so every value is
// exact; nibbles at bits 4..7 land in mantissa bits 4..7 (x16).
__device__ __forceinline__ uint4 sg_decode_word_f16(uint32_t w) {
  const uint32_t w8 = w >> 8;
  uint4 r;
  r.x = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  r.y = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  r.z = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  r.w = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
  return r;
}

// ------------------------------------------------------------- host side
#ifdef __CUDACC__
typedef CUresult (*SgEncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline SgEncodeTiledFn sg_encode_fn() {
  static SgEncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<SgEncodeTiledFn>(f);
  });
  return fn;
}

// 2-D map over a row-major [rows][cols] matrix of 16-bit elements (bf16 or
// f16), box box_cols x box_rows; elements outside the matrix read as zero.
inline bool sg_make_map_16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_cols,
                           int box_rows, CUtensorMapSwizzle sw, bool f16) {
  SgEncodeTiledFn fn = sg_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
            dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The decode activations as a 4-D map: [chunk][part][row][64] over the
// row-major part buffers (part 0 = hi, part 1 = lo, `part_stride` bytes
// apart; rows `row_stride` bytes apart, each a multiple of 64 elements), so
// one box of {64, box_rows, 2, chunks} brings, per chunk, box_rows hi rows
// followed by box_rows lo rows: a K-major 128-byte-swizzled UMMA operand
// tile of 2*box_rows rows. Rows >= rows and chunks >= n_chunks read as zero.
inline bool sg_make_map_parts(CUtensorMap* map, const void* base, int64_t rows, int64_t row_stride,
                              int64_t part_stride, int64_t n_chunks, int box_rows, int box_chunks) {
  SgEncodeTiledFn fn = sg_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {64, (cuuint64_t)rows, 2, (cuuint64_t)n_chunks};
  const cuuint64_t strides[3] = {(cuuint64_t)row_stride, (cuuint64_t)part_stride, 128};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 2, (cuuint32_t)box_chunks};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
#endif
