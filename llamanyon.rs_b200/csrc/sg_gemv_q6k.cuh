// sg_gemv_q6k.cuh -- decode GEMV for Q6_K weights (sg_gemv_q6k.cu).
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_Q6K_MAX_BATCH 16  // larger batches of a Q6_K tensor run the prefill GEMM

// y[t][r] (ldy) = sum_k W[r][k] x[t][k] (ldx) for t < batch (1..16), or
// y += W x with accumulate. With several K ranges per row-block the rows of
// y are zeroed first (stream-ordered) and the ranges reduced with red.add.
cudaError_t sg_gemv_q6k(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int batch,
                        bool accumulate, int num_sms, cudaStream_t st);
