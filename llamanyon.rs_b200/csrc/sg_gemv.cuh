// sg_gemv.cuh -- decode GEMV interface (see sg_gemv.cu).
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_MAX_MATS 4

struct SgGemvMatP {
  const uint32_t* qs;
  const void* sc;
  const uint32_t* dd;
  int64_t n_sb;
  int64_t n_rows;
  int64_t unit0;
  float* y;
  int64_t ldy;
};

struct SgGemvParams {
  SgGemvMatP mats[SG_GEMV_MAX_MATS];
  int n_mats;
  int batch;
  int64_t n_cols;
  int64_t n_ch;
  int64_t n_units;
  uint2* xfrag;      // [n_ch][4][NT][32] f16x2 pairs (scratch)
  float* xsum;       // [n_ch*2][16] (scratch, Q4_K)
  float* inv_scale;  // [16] (scratch)
};
// One matrix of a (multi-)GEMV call sharing the same activations.
struct SgGemvMat {
  const SgDevWeight* w;
  float* y;      // device, [batch][ldy]
  int64_t ldy;
};

size_t sg_gemv_scratch_bytes(int64_t n_cols);
int sg_gemv_max_ctas_per_sm();
// y_m[b][r] = sum_k W_m[r][k] x[b][k] for all matrices m (same K), batch 1..16.
// accumulate: y += W x (outputs are not zeroed first).
cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st);
