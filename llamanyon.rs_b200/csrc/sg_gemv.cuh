// sg_gemv.cuh -- decode GEMV interface (batch 1..32), see sg_gemv_mma.cu.
#pragma once
#include "sg_layout.cuh"

#define SG_GEMV_MAX_MATS 4
#define SG_GEMV_MAX_BATCH 32
#define SG_GEMV_MMA_MAX_CTAS 320  // CTAs per launch (one or two per SM)

// One matrix of a (multi-)GEMV call sharing the same activations.
struct SgGemvMat {
  const SgDevWeight* w;
  float* y;  // device, [batch][ldy]
  int64_t ldy;
};

// Bytes of the GEMV workspace for n_cols and batch: the activation images of
// the call (rebuilt by every call; nothing in it outlives a call).
size_t sg_gemv_scratch_bytes(int64_t n_cols, int batch);

// y_m[b][r] = sum_k W_m[r][k] x[b][k] for all matrices m (same K and dtype,
// Q4_0 or Q4_K), batch 1..32; accumulate: y += W x. x must be 16-byte
// aligned with ldx % 4 == 0 and must not overlap any y. Calls sharing a
// workspace must not overlap in time.
// An operation applied to x on its way into the decode GEMV's activation
// operands (the resulting rows are never written to memory), bit-identical
// to running the operation first:
//   SG_PRO_RMSNORM  x <- RMSNorm(x) * w over the n_cols of a row, with eps
//                   (sg_rmsnorm_device's arithmetic and summation order)
//   SG_PRO_SILU_MUL x <- silu(x) * x2 (sg_silu_mul_device's arithmetic)
enum { SG_PRO_NONE = 0, SG_PRO_RMSNORM = 1, SG_PRO_SILU_MUL = 2 };
struct SgGemvPrologue {
  int kind;
  const float* w;   // RMSNorm weights [n_cols]
  float eps;
  const float* x2;  // the second SiLU-mul operand, [batch][ldx2]
  int64_t ldx2;
};
// RMSNorm's block size in sg_ops.cu, whose summation order the prologue replays
constexpr int kSgNormThreads = 512;

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st,
                    const SgGemvPrologue* pro = nullptr);
