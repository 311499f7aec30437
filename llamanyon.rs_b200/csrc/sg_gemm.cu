// sg_gemm.cu -- prefill path for batches above 16 tokens.
//
// Replaces swamp-kernels fused_gemv_q4k_batched (fused_gemv_q4k.rs:527-698),
// which the engine's prefill issues through forward_linear_batch
// (swamp-engine/src/linear.rs:176-239, executor.rs:106-181).
//
// Current implementation: the decode GEMV over groups of 16 tokens (each group
// re-streams the weights). The tensor-core GEMM replaces this body.
#include "sg_gemm.cuh"
#include "sg_gemv.cuh"

size_t sg_gemm_scratch_bytes(int64_t m, int64_t n_cols) {
  (void)m;
  (void)n_cols;
  return 0;
}

cudaError_t sg_gemm(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int m, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  (void)scratch;
  (void)scratch_bytes;
  for (int t0 = 0; t0 < m; t0 += 16) {
    const int nb = m - t0 < 16 ? m - t0 : 16;
    SgGemvMat mat = {w, y + (int64_t)t0 * ldy, ldy};
    cudaError_t e = sg_gemv(&mat, 1, x + (int64_t)t0 * ldx, ldx, nb, accumulate, num_sms, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}
