// sg_gemv.cuh -- decode GEMV interface (batch 1..16), see sg_gemv.cu.
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_MAX_MATS 4
#define SG_GEMV_MAX_BATCH 16
#define SG_GEMV_MAX_CTAS 512  // CTAs per launch (one or two per SM)

// One matrix of a (multi-)GEMV call sharing the same activations.
struct SgGemvMat {
  const SgDevWeight* w;
  float* y;  // device, [batch][ldy]
  int64_t ldy;
};

// Bytes of the GEMV workspace for n_cols and batch: the flags through which
// the CTA that zeroes a shared row-block's rows tells the other CTAs
// (per-call epochs; zero them when the workspace is allocated, and keep it
// across calls), then, from 3 tokens on, the activation unit images.
size_t sg_gemv_scratch_bytes(int64_t n_cols, int batch);

// y_m[b][r] = sum_k W_m[r][k] x[b][k] for all matrices m (same K and dtype),
// batch 1..16; accumulate: y += W x. x must be 16-byte aligned with ldx % 4
// == 0. Calls sharing a workspace must not overlap in time.
cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st);
