// sg_gemv.cuh -- decode GEMV interface (batch 1..16), see sg_gemv.cu.
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_MAX_MATS 4
#define SG_GEMV_MAX_BATCH 16

// One matrix of a (multi-)GEMV call sharing the same activations.
struct SgGemvMat {
  const SgDevWeight* w;
  float* y;  // device, [batch][ldy]
  int64_t ldy;
};

// Scratch bytes a decode call over n_cols needs (f16 activation parts and
// per-32-block sums for up to 16 tokens).
size_t sg_gemv_scratch_bytes(int64_t n_cols);

// y_m[b][r] = sum_k W_m[r][k] x[b][k] for all matrices m (same K and dtype),
// batch 1..16; accumulate: y += W x. x must be 16-byte aligned with ldx % 4 == 0.
cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st);
