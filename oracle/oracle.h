/*
 * oracle.h -- CPU restatement of the llamanyon.rs quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path
 * (tests/, __graft_entry__.smoke()) and the timed CPU baseline of bench.py.
 * The product library (libswamp_gpu.so) never links, loads or calls it.
 *
 * Every function restates one reference function; the citation names the
 * reference file and lines (paths inside the llamanyon.rs workspace).
 * Arithmetic follows the reference exactly: IEEE binary32, no FMA
 * contraction (rustc does not contract; this file is built with
 * -ffp-contract=off), sequential accumulation order.
 */
#ifndef LLAMANYON_ORACLE_H
#define LLAMANYON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML dtype ids (swamp-gguf/src/dtype.rs:13,21) and block geometry
 * (q4_0.rs:8-9, q4_k.rs:18-19, dtype.rs:103,117). */
#define ORC_DTYPE_Q4_0 2
#define ORC_DTYPE_Q4_K 12
#define ORC_Q4_0_BLOCK 32
#define ORC_Q4_0_BYTES 18
#define ORC_Q4_K_BLOCK 256
#define ORC_Q4_K_BYTES 144
#define ORC_DTYPE_Q6_K 14
#define ORC_Q6_K_BLOCK 256
#define ORC_Q6_K_BYTES 210

/* IEEE binary16 <-> binary32 (crate `half` 2.7.1, Cargo.lock:607-608;
 * call sites q4_0.rs:24, q4_k.rs:281-282, fused_gemv_q4k.rs:708-710). */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f); /* round-to-nearest-even */

/* swamp-gguf/src/quant/q4_0.rs:11-38 (interleaved nibble order). */
int orc_q4_0_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n);

/* swamp-gguf/src/quant/q4_k.rs:37-53 == fused_gemv_q4k.rs:30-43. */
void orc_q4k_unpack_scales(const uint8_t sc[12], uint8_t scales[8], uint8_t mins[8]);

/* swamp-gguf/src/quant/q4_k.rs:21-33,278-322 (the dispatched scalar path). */
int orc_q4k_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n);
/* swamp-gguf/src/quant/q6_k.rs:8-57 */
int orc_q6k_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n);
/* swamp-kernels/src/fused_gemv_q6k.rs:248-291 (exact f16 d) */
void orc_gemv_q6k_scalar(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols);

/* Dispatch like swamp-gguf/src/quant/mod.rs:18-33 for the two dtypes. */
int orc_dequantize(int dtype, const uint8_t *raw, size_t raw_len, float *dst, size_t n);

/* swamp-kernels/src/fused_gemv_q4k.rs:466-508 (scalar path; overwrites out). */
void orc_gemv_q4k_scalar(const uint8_t *w, const float *x, float *out,
                         int64_t n_rows, int64_t n_cols);

/* swamp-kernels/src/fused_gemv_q4k.rs:650-698 (accumulates: out[t][r] += ...). */
void orc_gemv_q4k_batched_scalar(const uint8_t *w, const float *const *x_ptrs,
                                 float *const *out_ptrs, int64_t n_rows,
                                 int64_t n_cols, int64_t batch);

/* swamp-kernels/src/fused_gemv_q4k.rs:401-460 (scalar, zero-fills outputs). */
void orc_gemv_q4k_multi(const uint8_t *const *raws, const float *x,
                        float *const *outputs, const int64_t *row_counts,
                        int64_t n_matrices, int64_t n_cols);

/* swamp-kernels/src/fused_gemv_q4k.rs:799-823 (C ABI: null/shape -> silent
 * return; zeroes out before accumulating). */
void orc_swamp_fused_gemv_q4k(const uint8_t *w, const float *x, float *out,
                              int n_rows, int n_cols);

/* swamp-engine/src/linear.rs:68-87: the engine's Q4_0 route. Dequantize the
 * whole tensor to f32, then a sequential f32 dot per row. deq_scratch may be
 * NULL (then it is malloc'd, as the reference allocates per call). */
int orc_linear_q4_0(const uint8_t *w, const float *x, float *out,
                    int64_t n_rows, int64_t n_cols, float *deq_scratch);

/* swamp-engine/src/linear.rs:14-90 forward_linear, row-partitioned exactly as
 * :31-45 (rpt = ceil(N/n_threads); thread t gets [t*rpt, min(N,(t+1)*rpt))),
 * threads = n_threads pthreads. Q4_K -> orc_gemv_q4k_scalar per chunk,
 * Q4_0 -> full-tensor dequant + row dots. This is the CPU baseline. */
int orc_forward_linear(int dtype, const uint8_t *w, const float *x, float *out,
                       int64_t n_rows, int64_t n_cols, int n_threads);

/* swamp-engine/src/linear.rs:176-239 forward_linear_batch: Q4_K partitions rows
 * over threads and calls the batched kernel (outputs zeroed first); other
 * dtypes go to fallback_gemv (:336-364) which for Q4_0 bytes calls the Q4_K
 * kernel (garbage). Here the Q4_0 arm uses the correct engine route per token
 * instead and the deviation is flagged by the return value 1. */
int orc_forward_linear_batch(int dtype, const uint8_t *w, const float *const *xs,
                             float *const *outs, int64_t batch, int64_t n_rows,
                             int64_t n_cols, int n_threads);

/* oracle_simd.c: the reference's dispatched SIMD Q4_K paths, for CPU timing
 * only (numerically divergent from the reference's dequantizer; see that
 * file). orc_simd_path: 2 = AVX-512 VNNI, 1 = AVX2+FMA, 0 = neither.
 * orc_gemv_q4k_vnni accumulates into out, orc_gemv_q4k_avx2 overwrites;
 * both return -1 when the CPU lacks the path. orc_forward_linear_dispatched
 * zeroes out, partitions rows as linear.rs:31-45 and returns the path used. */
int orc_simd_path(void);
int orc_gemv_q4k_vnni(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols);
int orc_gemv_q4k_avx2(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols);
int orc_forward_linear_dispatched(const uint8_t *w, const float *x, float *out, int64_t n_rows,
                                  int64_t n_cols, int n_threads);
/* forward_linear_batch's non-Q4_K route, fallback_gemv (linear.rs:336-364),
 * over the dispatched kernel: returns the path used, or < 0. */
int orc_fallback_gemv_dispatched(const uint8_t *w, const float *const *xs, float *const *outs, int64_t batch,
                                 int64_t n_rows, int64_t n_cols, int n_threads);

/* The reference's test block packer, fused_gemv_q4k.rs:708-724 (inverse of
 * unpack_scales). d and dmin go through f16 round-to-nearest-even. */
void orc_make_q4k_block(float d, float dmin, const uint8_t scales[8],
                        const uint8_t mins[8], uint8_t nibble_val, uint8_t out[144]);

/* The reference's test fixtures: fused_gemv_q4k.rs:726-736 make_weight and
 * :738-740 make_x. */
void orc_make_weight(int64_t n_rows, uint8_t *out /* n_rows*144 */);
void orc_make_x(int64_t n_cols, float *out);

/* Seeded synthetic generators for the benchmark configurations (no
 * reference counterpart; the reference benchmarks use ad-hoc fills, see
 * swamp-tools/src/bin/benchmark_q4k_batched.rs:19-41). Counter-based:
 * h = splitmix64(seed ^ (tensor_id << 40) ^ index), so any slice can be
 * regenerated independently and threads partition freely. */
uint64_t orc_splitmix64(uint64_t z);
void orc_gen_q4_0(uint64_t seed, uint64_t tensor_id, int64_t n_rows,
                  int64_t n_cols, uint8_t *out, int n_threads);
void orc_gen_q6k(uint64_t seed, uint64_t tensor_id, int64_t n_rows, int64_t n_cols, uint8_t *out, int n_threads);
void orc_gen_q4k(uint64_t seed, uint64_t tensor_id, int64_t n_rows,
                 int64_t n_cols, uint8_t *out, int n_threads);
void orc_gen_x(uint64_t seed, uint64_t tensor_id, int64_t n, float *out);

/* fp64 dot of the dequantized weights (error-analysis truth, not a
 * reference function): out64[r] = sum_k w[r,k]*x[k] in double, and
 * absdot[r] = sum_k |w[r,k]*x[k]|, l2dot[r] = sqrt(sum_k (w x)^2). */
int orc_gemv_f64(int dtype, const uint8_t *w, const float *x, int64_t n_rows,
                 int64_t n_cols, double *out64, double *absdot, double *l2dot);

/* decoder-layer operations (swamp-engine/src/ops.rs, sampler.rs) */
void orc_rmsnorm(const float *x, const float *w, float *out, int64_t n, float eps);
void orc_rope_lut(int head_dim, int64_t max_seq_len, float *lut);
void orc_rope_apply(float *q, float *k, int64_t pos, int n_q_heads, int n_kv_heads, int head_dim,
                    int64_t max_context, const float *lut);
void orc_attention(float *out, const float *q, const float *k_cache, const float *v_cache, int64_t head_stride,
                   int64_t seq_len, int64_t q_pos, int n_heads, int n_kv_heads, int head_dim);
void orc_silu_mul(float *g, const float *u, int64_t n);
void orc_add(float *a, const float *b, int64_t n);
int64_t orc_argmax(const float *logits, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
