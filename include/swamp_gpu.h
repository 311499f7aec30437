/*
 * swamp_gpu.h -- C ABI of libswamp_gpu.so, the B200 (sm_100a) drop-in for
 * llamanyon.rs's quantized-linear hot path.
 *
 * It replaces, for GGUF Q4_0 (dtype 2) and Q4_K (dtype 12) tensors:
 *   swamp-engine/src/linear.rs:14-90    forward_linear        -> sg_linear (batch 1)
 *   swamp-engine/src/linear.rs:96-170   forward_linear_multi  -> sg_linear_multi
 *   swamp-engine/src/linear.rs:176-239  forward_linear_batch  -> sg_linear (batch B)
 *   swamp-engine/src/linear.rs:278-333  forward_gemvs         -> sg_linear_multi / sg_linear
 *   swamp-kernels/src/fused_gemv_q4k.rs:59-82,527-554         -> sg_linear
 *   swamp-kernels/src/fused_gemv_q4k.rs:799-823 swamp_fused_gemv_q4k -> sg_fused_gemv_q4k
 *   swamp-gguf/src/quant/{q4_0.rs:11-38,q4_k.rs:21-33} dequant -> sg_dequant_f32
 * and the swamp-gpu crate's loader/handle conventions
 * (swamp-gpu/src/lib.rs:16-71: dlopen of libswamp_gpu.so, int status codes,
 * opaque void* handles, host- and device-pointer entry points).
 *
 * Conventions
 *  - Every entry returns an int status: SG_OK (0) or a negative SG_ERR_*;
 *    sg_last_error() returns a message for the calling thread. Arguments are
 *    validated on the host before anything is launched.
 *  - Weights are uploaded once (sg_weight_register) and stay resident on the
 *    GPU(s) until sg_weight_free; callers key the handle on the GGUF
 *    TensorInfo.offset as the reference re-reads the mmap on every call
 *    (swamp-engine/src/linear.rs:24).
 *  - Output semantics are overwrite (forward_linear*, swamp_fused_gemv_q4k
 *    zero-fill then accumulate, linear.rs:107,204-207, fused_gemv_q4k.rs:820)
 *    unless SG_FLAG_ACCUMULATE asks for the batched kernel's out += W x
 *    (fused_gemv_q4k.rs:696).
 *  - Numerics: dequantized weights are bit-identical to swamp-gguf's. The
 *    decode GEMV multiplies the raw nibbles by the activations' exact 8-bit
 *    digits in integer arithmetic and applies the block scales in f32; the
 *    prefill GEMM accumulates in f32 with weights and activations split into
 *    bf16 hi + lo parts. The tested bound is
 *    |y - y_ref| <= 1e-3 * max(|y_ref|, ||w.*x||_2) per element against the
 *    reference's f32 result.
 *  - Thread safety: calls are serialised on an internal mutex per library
 *    instance; each device has one stream. Calls may come from any host
 *    thread (the reference calls from rayon workers, linear.rs:35).
 *  - There is no CPU fallback: without a usable sm_100 GPU, sg_init fails.
 */
#ifndef SWAMP_GPU_H
#define SWAMP_GPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SG_API __attribute__((visibility("default")))
#else
#define SG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes (swamp-gpu/src/lib.rs:16-26 maps non-zero to GpuError) */
#define SG_OK 0
#define SG_ERR_INVALID_ARG (-1)
#define SG_ERR_CUDA (-2)
#define SG_ERR_NCCL (-3)
#define SG_ERR_OOM (-4)
#define SG_ERR_UNSUPPORTED (-5)
#define SG_ERR_NOT_INITIALIZED (-6)
#define SG_ERR_DEVICE_FAULT (-7) /* a kernel's bounded wait gave up; see sg_last_error */
#define SG_ERR_FORMAT (-8)       /* malformed GGUF file (swamp-gguf GgufError, error.rs) */
#define SG_ERR_NOT_FOUND (-9)    /* no such GGUF tensor or metadata key */

/* GgmlDType ids (swamp-gguf/src/dtype.rs:13,21) */
#define SG_DTYPE_Q4_0 2
#define SG_DTYPE_Q4_K 12
#define SG_DTYPE_Q6_K 14 /* swamp-gguf/src/quant/q6_k.rs: 210 B per 256 */

/* tensor-parallel placement of a registered weight */
#define SG_TP_REPLICATE 0 /* every rank holds the whole tensor */
#define SG_TP_COLUMN 1    /* split N (output rows): Q/K/V/gate/up; outputs stay local */
#define SG_TP_ROW 2       /* split K (reduction): O/down; outputs all-reduced (sum) */

/* flags */
#define SG_FLAG_DEVICE_PTRS 0x1 /* x/out pointers are device memory on this rank's device */
#define SG_FLAG_ACCUMULATE 0x2  /* out += W x instead of out = W x */

typedef struct sg_weight_s *sg_weight_t;
typedef struct sg_gguf_s *sg_gguf_t;

/* ------------------------------------------------------------------ setup */

/* Single-process mode (the reference engine is one process, one host thread,
 * swamp-engine/src/executor.rs:292): use devices 0..n_gpus-1; for n_gpus > 1
 * build an NCCL communicator over them (ncclCommInitAll). */
SG_API int sg_init(int n_gpus);

/* One-process-per-GPU mode: this process is `rank` of `world`, drives CUDA
 * device `device`, and joins the NCCL communicator identified by the 128-byte
 * id that rank 0 produced with sg_get_unique_id (shipped to the other ranks by
 * the caller, e.g. over torch.distributed). */
SG_API int sg_get_unique_id(void *id128);
SG_API int sg_init_rank(int rank, int world, const void *id128, int device);

SG_API int sg_shutdown(void);
SG_API const char *sg_last_error(void);
/* rank / world size / number of devices driven by this process */
SG_API int sg_topology(int *rank, int *world, int *local_devices);

/* Page-locked host memory for the xs / outs of the host-pointer entry
 * points (copied by DMA without the staging copy). bytes == 0 gives NULL.
 * No sg_init needed. The reference has no counterpart: its buffers are
 * ordinary Vec<f32>. */
SG_API int sg_host_alloc(size_t bytes, void **out);
SG_API int sg_host_free(void *p);

/* ---------------------------------------------------------------- weights */

/* Upload one GGUF tensor (host pointer to its raw block bytes, row-major:
 * n_rows rows of n_cols/32*18 (Q4_0) or n_cols/256*144 (Q4_K) bytes) and
 * repack it into the device tile layout. n_cols % 32 == 0 (Q4_0) or
 * % 256 == 0 (Q4_K). tp_mode splits across the process's ranks/devices on
 * whole blocks (SG_TP_ROW needs n_cols/world to stay a block multiple). */
SG_API int sg_weight_register(const void *host_blocks, int dtype, int64_t n_rows, int64_t n_cols,
                       int tp_mode, sg_weight_t *out);
SG_API int sg_weight_free(sg_weight_t w);
/* The slice rank `rank` of `world` holds under tp_mode, computed on the host
 * (no GPU or init needed): rows [row0, row0+rows) and columns
 * [col0, col0+cols). Column split: rows [rank*N/world, (rank+1)*N/world);
 * row split: whole blocks [rank*nblk/world, (rank+1)*nblk/world) of every
 * row (nblk = n_cols/32 or /256). Same validation as sg_weight_register. */
SG_API int sg_tp_shard(int dtype, int64_t n_rows, int64_t n_cols, int tp_mode, int world, int rank,
                       int64_t *row0, int64_t *rows, int64_t *col0, int64_t *cols);
/* shape of the shard this rank holds: local rows/cols and their offsets */
SG_API int sg_weight_shard(sg_weight_t w, int local_device, int64_t *n_rows, int64_t *n_cols,
                    int64_t *row0, int64_t *col0);

/* -------------------------------------------------------------- compute */

/* forward_linear / forward_linear_batch: outs[b][r] = sum_k W[r][k] xs[b][k]
 * for b < batch. Host pointers (default): xs[b] has n_cols floats, outs[b]
 * n_rows floats (the whole tensor, whatever the TP split; in one-process-per-
 * GPU mode a column-split call fills only this rank's rows of outs[b]). With
 * SG_FLAG_DEVICE_PTRS (single-device or rank mode only) xs/outs point at
 * this rank's device and hold this rank's shard: x of n_cols_local, out of
 * n_rows_local (column split) or n_rows (replicate / row split, all-reduced).
 * Batches of 1..32 run the decode GEMV; larger batches the prefill GEMM.
 * Host rows one fixed stride apart in page-locked memory (sg_host_alloc, or
 * the caller's own cudaHostAlloc) are copied by DMA straight from xs and into
 * outs (one device per process, no SG_FLAG_ACCUMULATE for outs); other host
 * rows pass through the library's page-locked staging buffer with one extra
 * host copy. Either way the call returns with the results in outs. */
SG_API int sg_linear(sg_weight_t w, const float *const *xs, float *const *outs, int batch, int flags);

/* forward_linear_multi (linear.rs:96-170): several tensors, same x (K). */
SG_API int sg_linear_multi(const sg_weight_t *ws, int n_weights, const float *x, float *const *outs,
                    int flags);

/* Device-resident, stream-ordered form for engines that keep activations on
 * the GPU: x is [batch][ldx] (this rank's K-slice starts at x), y is
 * [batch][ldy]. stream is a cudaStream_t; NULL means CUDA's default stream.
 * Returns once the work is enqueued. A row-split tensor's outputs are
 * all-reduced in place; with SG_FLAG_ACCUMULATE every rank passes the same
 * y (e.g. the replicated residual stream) and gets y + W x, the old y counted
 * once. Batches of 1..32 run the decode GEMV, larger ones the prefill GEMM. */
SG_API int sg_linear_device(sg_weight_t w, const float *x, int64_t ldx, float *y, int64_t ldy, int batch,
                     void *stream, int flags);
SG_API int sg_linear_multi_device(const sg_weight_t *ws, int n_weights, const float *x, int64_t ldx,
                           float *const *ys, const int64_t *ldys, int batch, void *stream, int flags);

/* sg_linear_device for callers that must not trigger a device allocation --
 * for example a serving loop with a fixed memory budget, where the implicit
 * device-wide synchronisation of a first-use cudaMalloc would stall other
 * streams. Same arguments and results as sg_linear_device for one tensor at
 * decode batch 1..16 (larger batches are rejected with SG_ERR_UNSUPPORTED:
 * they run the prefill GEMM, whose activation scratch is allocated on first
 * use). The decode kernel's workspace (the call's activations converted to
 * the MMA operand layout) is a fixed 1.65 MB per-device array inside the
 * library, so the call allocates nothing: n_cols up to 174080 at batch 1..2,
 * 64768 at 3..8 and 32768 at 9..16 (wider tensors are rejected with
 * SG_ERR_UNSUPPORTED and a message naming the limit). The first call on a
 * device looks up that workspace's address once; make it before any stream
 * capture begins. All decode calls on a device share the workspace: calls
 * whose work may overlap in time (different streams with no ordering between
 * them) race, so order them. A row-split tensor in one-process-per-GPU mode
 * needs ldy == n_rows and no SG_FLAG_ACCUMULATE; its all-reduce is the peer
 * kernel over the buffers sg_init_rank mapped (batch * n_rows up to 512 Ki
 * floats), which allocates nothing. With that kernel off
 * (SG_PEER_ALLREDUCE=0, or a set-up that failed: sg_allreduce_path) or a
 * longer vector it is ncclAllReduce, and NCCL may set up connections and
 * their buffers on its first collective of a kind.
 * The reference has no counterpart: its CPU path allocates per call. */
SG_API int sg_linear_device_noalloc(sg_weight_t w, const float *x, int64_t ldx, float *y, int64_t ldy, int batch,
                                    void *stream, int flags);

/* Dequantize the whole tensor to f32 [n_rows][n_cols] (host pointer, or this
 * rank's shard into device memory with SG_FLAG_DEVICE_PTRS). Bit-exact with
 * swamp-gguf's dequant. */
SG_API int sg_dequant_f32(sg_weight_t w, float *dst, int flags);

/* swamp_fused_gemv_q4k (fused_gemv_q4k.rs:799-823): raw Q4_K host bytes on
 * every call, x of n_cols, out of n_rows (overwritten). Unlike the Rust
 * symbol it reports errors instead of silently returning. */
SG_API int sg_fused_gemv_q4k(const uint8_t *w_raw, const float *x, float *out, int n_rows, int n_cols);

/* Sum all-reduce of `count` floats in place across the ranks of a
 * one-process-per-GPU job (every rank calls it with the same count; the
 * row-split linears use it for their outputs). Up to 512 Ki floats it runs
 * the library's peer kernel: each rank stores its partial straight into
 * every peer's receive buffer over NVLink (CUDA IPC mappings made at
 * sg_init_rank), every value beside the call's epoch in one 8-byte word,
 * reads the peers' values from its own buffer as their epochs arrive
 * (bounded waits) and sums in rank order, so every rank gets the same bits.
 * Larger vectors, or jobs where any rank could not map its peers, use
 * ncclAllReduce. Stream-ordered and graph-capturable. SG_PEER_ALLREDUCE=0
 * in the environment at sg_init_rank makes every call use NCCL.
 * sg_allreduce_path reports which one this job uses (1: peer kernel). */
SG_API int sg_allreduce_device(float *buf, int64_t count, void *stream);
SG_API int sg_allreduce_path(int *peer);

/* Wait for this process's devices and surface any device-side error flag. */
SG_API int sg_synchronize(void);

/* ------------------------------------------------------------------ GGUF */

/* GGUF reader and upload path, replacing swamp-gguf's GgufFile
 * (swamp-gguf/src/mmap.rs:26-120, metadata.rs:118-236, tensor_info.rs:8-38).
 * Host-only: these calls need no GPU and no sg_init, except
 * sg_gguf_register. The format rules are the reference's: version 1..3;
 * u32 counts and dimensions in version 1, u64 from 2; strings are a u64
 * length and bytes decoded as UTF-8 with invalid sequences replaced by
 * U+FFFD; a repeated metadata key keeps its last value; tensor data starts
 * at the end of the tensor table rounded up to 32 bytes (general.alignment
 * is not consulted, mmap.rs:13,78-89). Malformed files give SG_ERR_FORMAT.
 * Returned strings stay valid until sg_gguf_close. */
SG_API int sg_gguf_open(const char *path, sg_gguf_t *out);   /* mmap.rs:28-32 GgufFile::open */
/* parse a file image the caller keeps alive until sg_gguf_close */
SG_API int sg_gguf_open_memory(const void *data, size_t size, sg_gguf_t *out);
SG_API int sg_gguf_close(sg_gguf_t g);
SG_API int sg_gguf_header(sg_gguf_t g, uint32_t *version, int64_t *n_tensors, int64_t *n_kv, int64_t *data_offset,
                          int64_t *file_size);
/* first tensor with this name (mmap.rs:95-98 GgufFile::tensor); SG_ERR_NOT_FOUND otherwise */
SG_API int sg_gguf_find_tensor(sg_gguf_t g, const char *name, int64_t *index);
/* TensorInfo (tensor_info.rs:8-16): name, ggml type, dims (up to dims_cap of
 * n_dims written; dims[0] is the contiguous one), absolute file offset and
 * byte size (tensor_info.rs:24-26) */
SG_API int sg_gguf_tensor_info(sg_gguf_t g, int64_t index, const char **name, int *dtype, int *n_dims, int64_t *dims,
                               int dims_cap, int64_t *offset, int64_t *nbytes);
/* the tensor's raw bytes in the mapped file, range-checked (mmap.rs:111-118) */
SG_API int sg_gguf_tensor_data(sg_gguf_t g, int64_t index, const void **data, int64_t *nbytes);
/* metadata: index of a key (its last occurrence), then its type (GGUF value
 * type 0..12; 9 = array with elem_type and count elements) and values.
 * Integer and bool types read as int64 (u64 as its bits), f32/f64 as double,
 * strings as UTF-8 bytes; elem is 0 for a scalar. */
SG_API int sg_gguf_find_kv(sg_gguf_t g, const char *key, int64_t *index);
SG_API int sg_gguf_kv_info(sg_gguf_t g, int64_t index, const char **key, int *type, int *elem_type, int64_t *count);
SG_API int sg_gguf_kv_int(sg_gguf_t g, int64_t index, int64_t elem, int64_t *value);
SG_API int sg_gguf_kv_float(sg_gguf_t g, int64_t index, int64_t elem, double *value);
SG_API int sg_gguf_kv_string(sg_gguf_t g, int64_t index, int64_t elem, const char **str, int64_t *len);
/* Upload a Q4_0/Q4_K matrix of the file (shape[0] = n_cols K, shape[1] =
 * n_rows N, as swamp-engine reads it, linear.rs:21-22) through
 * sg_weight_register, straight from the mapped blocks; the handle is
 * independent of the file afterwards. */
SG_API int sg_gguf_register(sg_gguf_t g, int64_t index, int tp_mode, sg_weight_t *out);

/* ------------------------------------------------------- synthetic inputs */

/* Seeded random-init tensors of the benchmark configurations, generated on
 * the device: Q4_0 d uniform in [0.001, 0.01) (f16), nibbles uniform 0..15;
 * Q4_K d and dmin likewise, 6-bit scales and mins uniform, packed as
 * make_q4k_block (swamp-kernels/src/fused_gemv_q4k.rs:708-724); Q6_K int8
 * scales and 6-bit values uniform. Each block's bytes are a function of
 * (seed, tensor_id, block index) through splitmix64, so a tensor-parallel
 * shard generates only its own blocks. sg_synth_weight registers such a
 * tensor like sg_weight_register would; sg_synth_blocks writes its GGUF
 * bytes (host memory, or device memory with SG_FLAG_DEVICE_PTRS). */
SG_API int sg_synth_weight(int dtype, uint64_t seed, uint64_t tensor_id, int64_t n_rows, int64_t n_cols,
                           int tp_mode, sg_weight_t *out);
SG_API int sg_synth_blocks(int dtype, uint64_t seed, uint64_t tensor_id, int64_t n_rows, int64_t n_cols,
                           void *dst, int flags);
/* N(0,1) activations (Box-Muller in double, one f32 rounding), host memory;
 * needs no GPU. */
SG_API int sg_synth_x(uint64_t seed, uint64_t tensor_id, int64_t n, float *dst);

/* ------------------------------------------------------------- layer ops */

/* The non-matmul operations of a decoder layer on device-resident
 * activations, so that an engine keeps x between the linears on the GPU
 * (swamp-engine/src/executor.rs:403-550 decode, :48-190 prefill). All are
 * stream-ordered on the caller's stream (NULL = CUDA's default stream), take
 * device pointers, need one device per process, and return once the work is
 * enqueued. Per-row int32 arrays (pos, seq_len, seq, tokens) live in device
 * memory so that a captured CUDA graph can be replayed with new positions.
 * A device-side index out of range (position outside the cache, token
 * outside the table, sequence outside the cache) skips that row's work and
 * makes the next sg_synchronize return SG_ERR_DEVICE_FAULT. */
typedef struct sg_rope_s *sg_rope_t;
typedef struct sg_kv_cache_s *sg_kv_cache_t;

/* init_rope_lut (swamp-engine/src/ops.rs:20-38): the f32 (cos, sin) table of
 * theta = 10000 for head_dim and positions 0..max_context-1, computed with
 * the host libm as the reference does and kept on the device.
 * sg_rope_table copies it to host memory ([max_context][head_dim/2][2]). */
SG_API int sg_rope_create(int head_dim, int max_context, sg_rope_t *out);
SG_API int sg_rope_free(sg_rope_t rope);
SG_API int sg_rope_table(sg_rope_t rope, float *dst);

/* PagedKVCache::new (swamp-engine/src/cache.rs:55-100): K and V of n_seqs
 * independent sequences, zero-filled, laid out
 * [seq][layer][kv_head][max_seq][head_dim] f32 (the reference's pages of 32
 * positions exist to move them to NVMe; here the cache stays resident).
 * sg_kv_cache_ptr gives the device address of position 0 of one
 * (seq, layer, kv_head); position p is p * head_dim floats further
 * (get_k_unchecked / k_page_ptr, cache.rs:373-410). */
SG_API int sg_kv_cache_create(int n_layers, int n_kv_heads, int head_dim, int max_seq, int n_seqs,
                              sg_kv_cache_t *out);
SG_API int sg_kv_cache_free(sg_kv_cache_t cache);
SG_API int sg_kv_cache_ptr(sg_kv_cache_t cache, int seq, int layer, int kv_head, float **k, float **v);

/* rmsnorm (ops.rs:188-201) of `rows` rows of n: out = x / sqrt(mean(x^2) + eps) * weight.
 * out may equal x. */
SG_API int sg_rmsnorm_device(const float *x, int64_t ldx, const float *weight, float *out, int64_t ldo, int n,
                             int rows, float eps, void *stream);

/* apply_rope_ufc (ops.rs:42-80) on q (n_q_heads heads) and k (the cache's
 * n_kv_heads) of each row at position pos[r] (table row min(pos,
 * max_context - 1)), in place, then PagedKVCache::save_at (cache.rs:412-434):
 * k and v of row r go to position pos[r] of sequence seq[r] (seq NULL: 0) in
 * `layer`. rope NULL stores k and v without rotating (q unused). */
SG_API int sg_rope_kv_device(sg_rope_t rope, sg_kv_cache_t cache, int layer, float *q, int64_t ldq, float *k,
                             int64_t ldk, const float *v, int64_t ldv, const int32_t *pos, const int32_t *seq,
                             int rows, int n_q_heads, void *stream);

/* attention (ops.rs:82-186): row r's n_heads query heads (q [rows][ldq],
 * head h at h*head_dim) attend positions 0..min(pos[r], seq_len[r]-1) of
 * sequence seq[r] (seq_len NULL: pos+1; seq NULL: 0), query head h reading
 * KV head h / (n_heads / n_kv_heads); softmax of q.k / sqrt(head_dim);
 * out [rows][ldo] gets the weighted sum of V. head_dim 64, 128 or 256, at
 * most 8 query heads per KV head. The split partials live in a per-device
 * workspace that grows on first use (make one call with the largest `rows`
 * before capturing a graph) and is shared by all attention calls, so calls
 * on different streams must be ordered. */
SG_API int sg_attention_device(sg_kv_cache_t cache, int layer, const float *q, int64_t ldq, float *out, int64_t ldo,
                               const int32_t *pos, const int32_t *seq_len, const int32_t *seq, int rows, int n_heads,
                               void *stream);

/* The decode form of sg_rope_kv_device followed by sg_attention_device, in
 * one kernel: row r is the next token of sequence seq[r] (one row per
 * sequence, so rows <= the cache's n_seqs) at position pos[r]; it rotates
 * q and k with the table row, stores k and v at pos[r], and attends
 * positions 0..pos[r]. q, k and v are read and left unchanged; out gets the
 * attention output. The results are the same bits as the two-call form.
 * It shares the attention workspace (grows on first use). */
SG_API int sg_rope_attention_device(sg_rope_t rope, sg_kv_cache_t cache, int layer, const float *q, int64_t ldq,
                                    const float *k, int64_t ldk, const float *v, int64_t ldv, float *out,
                                    int64_t ldo, const int32_t *pos, const int32_t *seq, int rows, int n_heads,
                                    void *stream);

/* The batched prefill's attention (executor.rs:113-141): positions
 * 0..n_tokens-1 of sequences 0..n_seqs-1, whose K and V rows the cache
 * already holds (sg_rope_kv_device stored them), each attending positions
 * 0..t of its own sequence. The row of (sequence s, position t) in q and out
 * is s * row_stride_seq + t * row_stride_pos. Same results as
 * sg_attention_device with pos = t and seq = s per row, within the attention
 * tolerance (another summation order); one CTA serves a block of positions
 * of one KV head, so each K/V tile is read once per block instead of once
 * per position. head_dim 64 or 128; q and out 16-byte aligned with
 * ldq, ldo multiples of 4. */
SG_API int sg_attention_prefill_device(sg_kv_cache_t cache, int layer, const float *q, int64_t ldq, float *out,
                                       int64_t ldo, int n_seqs, int n_tokens, int64_t row_stride_seq,
                                       int64_t row_stride_pos, int n_heads, void *stream);

/* silu then mul_in_place (ops.rs:203-214): g = g / (1 + exp(-g)) * u. */
SG_API int sg_silu_mul_device(float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, void *stream);

/* Fused forms of two engine sequences, for decode: the op runs on the way
 * into the decode GEMV's activation operands, so its output rows are never
 * written and one kernel per call is saved. Results are bit-identical to
 * running the op then the linear (the same arithmetic, RMSNorm's summation
 * order included). Batches above the decode range, and Q6_K tensors, run the
 * two steps (the op's rows go to a library buffer allocated on first use).
 * No reference counterparts: the engine calls rmsnorm then
 * forward_linear_multi (executor.rs:436-445 / :493-499), and silu,
 * mul_in_place then forward_linear (:499-505).
 *
 * sg_rmsnorm_linear_multi_device: ys[i] = W_i rmsnorm(x) with weight
 * `norm_weight` [n_cols] and eps, otherwise as sg_linear_multi_device (x is
 * not modified).
 * sg_silu_mul_linear_device: y = W (silu(g) * u), otherwise as
 * sg_linear_device (g and u [batch][n_cols] with strides ldg / ldu; neither
 * is modified). */
SG_API int sg_rmsnorm_linear_multi_device(const sg_weight_t *ws, int n_weights, const float *x, int64_t ldx,
                                          const float *norm_weight, float eps, float *const *ys,
                                          const int64_t *ldys, int batch, void *stream, int flags);
SG_API int sg_silu_mul_linear_device(sg_weight_t w, const float *g, int64_t ldg, const float *u, int64_t ldu,
                                     float *y, int64_t ldy, int batch, void *stream, int flags);
/* add_in_place (ops.rs:216-220): x += y. (A linear's SG_FLAG_ACCUMULATE
 * adds its result into the residual stream in the same kernel.) */
SG_API int sg_add_device(float *x, int64_t ldx, const float *y, int64_t ldy, int n, int rows, void *stream);
/* Greedy decoding: out[r] = index of the largest logit of row r, the last
 * of equal maxima (the sampler's max_by fallback, sampler.rs:94-95); -1 for
 * a row holding a NaN (where the reference panics). */
SG_API int sg_argmax_device(const float *logits, int64_t ld, int n, int rows, int32_t *out, void *stream);
/* Embedding lookup (executor.rs:416-418): out[r] = row tokens[r] of the
 * registered (replicated) table, dequantized bit-exactly; out 16-byte
 * aligned, ldo % 4 == 0. */
SG_API int sg_embed_device(sg_weight_t table, const int32_t *tokens, int rows, float *out, int64_t ldo,
                           void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SWAMP_GPU_H */
