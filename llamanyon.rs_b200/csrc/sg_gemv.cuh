// sg_gemv.cuh -- decode GEMV interface (see sg_gemv.cu).
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_MAX_MATS 4

struct SgGemvMatP {
  const uint8_t* tiles;
  const uint32_t* dd;
  int n_sb;
  int n_rb;
  int n_rows;
  int rb0;  // first global row-block index of this matrix
  float* y;
  int64_t ldy;
};

struct SgGemvParams {
  SgGemvMatP mats[SG_GEMV_MAX_MATS];
  int n_mats;
  int batch;
  int n_cols;
  int n_ch;
  int split;       // CTAs (one thread-block cluster) per row-block, each a K slice
  int accumulate;  // y += W x
  const float* x;  // [batch][ldx]
  int64_t ldx;
};

// One matrix of a (multi-)GEMV call sharing the same activations.
struct SgGemvMat {
  const SgDevWeight* w;
  float* y;  // device, [batch][ldy]
  int64_t ldy;
};

// y_m[b][r] = sum_k W_m[r][k] x[b][k] for all matrices m (same K), batch 1..16.
// accumulate: y += W x. x must be 8-byte aligned with an even ldx. Needs no
// global scratch.
cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    int num_sms, cudaStream_t st);
