// sg_gemm.cuh -- prefill GEMM interface (batch > 16 tokens), see sg_gemm.cu.
#pragma once
#include "sg_layout.cuh"

// Scratch bytes a prefill call of m tokens over K columns needs.
size_t sg_gemm_scratch_bytes(int64_t m, int64_t n_cols);

// y[t][r] (ldy) = sum_k W[r][k] x[t][k] (ldx) for t < m (y += ... when accumulate).
cudaError_t sg_gemm(const SgDevWeight* w, const float* x, int64_t ldx, float* y, int64_t ldy, int m, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st);
