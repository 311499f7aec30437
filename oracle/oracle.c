/*
 * oracle.c -- CPU restatement of the llamanyon.rs Q4_0 / Q4_K linear path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
 * baseline. Nothing in the product library links or calls this file.
 *
 * Built with -O2 -ffp-contract=off (rustc never contracts a*b+c into an FMA),
 * so every expression below rounds exactly where the Rust source rounds.
 * Citations are file:line inside the llamanyon.rs workspace.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* binary16 <-> binary32 (crate half 2.7.1: exact widening; RNE narrowing)   */
/* ------------------------------------------------------------------------- */

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: value = man * 2^-24; renormalise */
            int shifts = 0;
            while (!(man & 0x400u)) {
                man <<= 1;
                shifts++;
            }
            bits = sign | ((uint32_t)(127 - 15 + 1 - shifts) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = man ? (sign | 0x7FC00000u | (man << 13)) : (sign | 0x7F800000u);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man) return (uint16_t)(sign | 0x7E00u | (man >> 13));
        return (uint16_t)(sign | 0x7C00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e; /* 14..24 */
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hbits = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (hbits & 1u))) hbits++;
    return (uint16_t)hbits;
}

static inline float ld_f16(const uint8_t *p) {
    return orc_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

/* ------------------------------------------------------------------------- */
/* Dequantizers                                                              */
/* ------------------------------------------------------------------------- */

/* swamp-gguf/src/quant/q4_0.rs:11-38 */
int orc_q4_0_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n) {
    size_t n_blocks = (n + ORC_Q4_0_BLOCK - 1) / ORC_Q4_0_BLOCK;
    if (raw_len < n_blocks * ORC_Q4_0_BYTES) return -1; /* BufferTooSmall (:15-19) */
    for (size_t b = 0; b < n_blocks; b++) {
        const uint8_t *blk = raw + b * ORC_Q4_0_BYTES;
        float scale = ld_f16(blk);                      /* :24 */
        const uint8_t *nib = blk + 2;                   /* :25 */
        size_t out_start = b * ORC_Q4_0_BLOCK;
        size_t out_end = out_start + ORC_Q4_0_BLOCK;
        if (out_end > n) out_end = n;
        for (size_t i = 0; i < out_end - out_start; i++) {
            uint8_t byte = nib[i / 2];                  /* :31 */
            uint8_t q = (i % 2 == 0) ? (byte & 0x0F) : (byte >> 4); /* :32 */
            int32_t v = (int32_t)q - 8;                 /* :34 */
            dst[out_start + i] = (float)v * scale;      /* :35 */
        }
    }
    return 0;
}

/* swamp-gguf/src/quant/q4_k.rs:37-53 (== fused_gemv_q4k.rs:30-43) */
void orc_q4k_unpack_scales(const uint8_t sc[12], uint8_t scales[8], uint8_t mins[8]) {
    for (int j = 0; j < 4; j++) {
        scales[j] = sc[j] & 63;
        mins[j] = sc[j + 4] & 63;
    }
    for (int j = 4; j < 8; j++) {
        scales[j] = (uint8_t)((sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4));
        mins[j] = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
    }
}

/* swamp-gguf/src/quant/q4_k.rs:21-33 (dispatch) and :278-322 (scalar body) */
int orc_q4k_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n) {
    size_t n_blocks = (n + ORC_Q4_K_BLOCK - 1) / ORC_Q4_K_BLOCK;
    if (raw_len < n_blocks * ORC_Q4_K_BYTES) return -1; /* :25-30 */
    for (size_t b = 0; b < n_blocks; b++) {
        const uint8_t *blk = raw + b * ORC_Q4_K_BYTES;
        float d = ld_f16(blk);          /* :281 */
        float dmin = ld_f16(blk + 2);   /* :282 */
        const uint8_t *sc = blk + 4;    /* :283 */
        const uint8_t *qs = blk + 16;   /* :284 */
        uint8_t scales[8], mins[8];
        orc_q4k_unpack_scales(sc, scales, mins);
        size_t out_start = b * ORC_Q4_K_BLOCK;
        size_t out_end = out_start + ORC_Q4_K_BLOCK;
        if (out_end > n) out_end = n;
        for (int pair = 0; pair < 4; pair++) {       /* :291 */
            const uint8_t *qb = qs + pair * 32;
            int sb_even = pair * 2;
            float scale_even = d * (float)(scales[sb_even] & 0x3F); /* :297 */
            float min_even = dmin * (float)(mins[sb_even] & 0x3F);  /* :298 */
            for (int i = 0; i < 32; i++) {
                size_t g = out_start + (size_t)sb_even * 32 + (size_t)i;
                if (g < out_end) {
                    uint8_t qi = qb[i] & 0x0F;
                    dst[g] = scale_even * (float)qi - min_even;     /* :304 */
                }
            }
            int sb_odd = pair * 2 + 1;
            float scale_odd = d * (float)(scales[sb_odd] & 0x3F);   /* :310 */
            float min_odd = dmin * (float)(mins[sb_odd] & 0x3F);    /* :311 */
            for (int i = 0; i < 32; i++) {
                size_t g = out_start + (size_t)sb_odd * 32 + (size_t)i;
                if (g < out_end) {
                    uint8_t qi = qb[i] >> 4;
                    dst[g] = scale_odd * (float)qi - min_odd;       /* :317 */
                }
            }
        }
    }
    return 0;
}

/* swamp-gguf/src/quant/q6_k.rs:8-57. Per 256-block: ql[128] low nibbles,
 * qh[64] high 2-bit pairs, 16 int8 scales, f16 d. Half h (128 elements),
 * l in 0..32, m in 0..4: element 128h + 32m + l has
 *   q = ((ql[64h + l + 32(m&1)] >> 4(m>>1)) & 0xF) | (((qh[32h + l] >> 2m) & 3) << 4)
 * and w = d * (f32)sc[8h + 2m + l/16] * (f32)(q - 32), left to right (:37-46).
 * Both products are exact in f32 (d: 11 significant bits, sc: at most 7,
 * q - 32: at most 5), as in the reference. */
int orc_q6k_dequant(const uint8_t *raw, size_t raw_len, float *dst, size_t n) {
    size_t n_blocks = (n + ORC_Q6_K_BLOCK - 1) / ORC_Q6_K_BLOCK;
    if (raw_len < n_blocks * ORC_Q6_K_BYTES) return -1; /* :12-17 */
    for (size_t b = 0; b < n_blocks; b++) {
        const uint8_t *blk = raw + b * ORC_Q6_K_BYTES;
        const uint8_t *ql = blk, *qh = blk + 128, *sc = blk + 192;
        float d = ld_f16(blk + 208); /* :28 */
        float y[256];
        for (int h = 0; h < 2; h++) {
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (int)(int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                int q2 = (int)(int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)(int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)(int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[128 * h + l] = d * (float)(int8_t)sc[is] * (float)q1;
                y[128 * h + l + 32] = d * (float)(int8_t)sc[is + 2] * (float)q2;
                y[128 * h + l + 64] = d * (float)(int8_t)sc[is + 4] * (float)q3;
                y[128 * h + l + 96] = d * (float)(int8_t)sc[is + 6] * (float)q4;
            }
            ql += 64;
            qh += 32;
            sc += 8;
        }
        size_t out_start = b * ORC_Q6_K_BLOCK;
        size_t cnt = n - out_start < 256 ? n - out_start : 256;
        memcpy(dst + out_start, y, cnt * sizeof(float));
    }
    return 0;
}

/* swamp-gguf/src/quant/mod.rs:18-33 (the dtypes in scope) */
int orc_dequantize(int dtype, const uint8_t *raw, size_t raw_len, float *dst, size_t n) {
    if (dtype == ORC_DTYPE_Q4_0) return orc_q4_0_dequant(raw, raw_len, dst, n);
    if (dtype == ORC_DTYPE_Q4_K) return orc_q4k_dequant(raw, raw_len, dst, n);
    if (dtype == ORC_DTYPE_Q6_K) return orc_q6k_dequant(raw, raw_len, dst, n);
    return -2;
}

/* swamp-kernels/src/fused_gemv_q6k.rs:248-291, the scalar path of the engine's
 * Q6_K route (swamp-engine/src/linear.rs:48-67): acc += d*sc*q*x in f32, left
 * to right, blocks, halves, then l with the four elements l, l+32, l+64,
 * l+96. d is decoded exactly (the kernel's own f16 decode, :11-20, breaks on
 * subnormal d; the dequantizer's exact one, q6_k.rs:28, is the parity
 * target); for normal d both agree. */
void orc_gemv_q6k_scalar(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols) {
    int64_t n_blocks = n_cols / ORC_Q6_K_BLOCK;
    for (int64_t row = 0; row < n_rows; row++) {
        float acc = 0.0f;
        for (int64_t blk = 0; blk < n_blocks; blk++) {
            const uint8_t *b = w + (size_t)(row * n_blocks + blk) * ORC_Q6_K_BYTES;
            float d = ld_f16(b + 208);
            const float *x_blk = x + blk * ORC_Q6_K_BLOCK;
            for (int half = 0; half < 2; half++) {
                const uint8_t *ql = b + 64 * half, *qh = b + 128 + 32 * half, *sc = b + 192 + 8 * half;
                const float *xh = x_blk + 128 * half;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    float q1 = (float)((int)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32);
                    float q2 = (float)((int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32);
                    float q3 = (float)((int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
                    float q4 = (float)((int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
                    acc += d * (float)(int8_t)sc[is] * q1 * xh[l];
                    acc += d * (float)(int8_t)sc[is + 2] * q2 * xh[l + 32];
                    acc += d * (float)(int8_t)sc[is + 4] * q3 * xh[l + 64];
                    acc += d * (float)(int8_t)sc[is + 6] * q4 * xh[l + 96];
                }
            }
        }
        out[row] = acc;
    }
}

/* ------------------------------------------------------------------------- */
/* Fused Q4_K GEMV, scalar path                                              */
/* ------------------------------------------------------------------------- */

/* Dot of one 256-element Q4_K block with x_blk, in the scalar kernels' exact
 * order: pairs 0..3, even (low nibbles) then odd (high nibbles), i = 0..31,
 * acc += (sv*q - mv) * x. fused_gemv_q4k.rs:486-503 / :672-691. */
static inline float q4k_block_dot(const uint8_t *blk, const float *x_blk, float acc) {
    float d = ld_f16(blk);
    float dmin = ld_f16(blk + 2);
    uint8_t scales[8], mins[8];
    orc_q4k_unpack_scales(blk + 4, scales, mins);
    const uint8_t *qs = blk + 16;
    for (int pair = 0; pair < 4; pair++) {
        const uint8_t *qb = qs + pair * 32;
        int sb_even = pair * 2;
        float sv_even = d * (float)(scales[sb_even] & 0x3F);
        float mv_even = dmin * (float)(mins[sb_even] & 0x3F);
        for (int i = 0; i < 32; i++) {
            uint8_t qi = qb[i] & 0x0F;
            float w_f = sv_even * (float)qi - mv_even;
            acc += w_f * x_blk[sb_even * 32 + i];
        }
        int sb_odd = pair * 2 + 1;
        float sv_odd = d * (float)(scales[sb_odd] & 0x3F);
        float mv_odd = dmin * (float)(mins[sb_odd] & 0x3F);
        for (int i = 0; i < 32; i++) {
            uint8_t qi = qb[i] >> 4;
            float w_f = sv_odd * (float)qi - mv_odd;
            acc += w_f * x_blk[sb_odd * 32 + i];
        }
    }
    return acc;
}

/* swamp-kernels/src/fused_gemv_q4k.rs:466-508 */
void orc_gemv_q4k_scalar(const uint8_t *w, const float *x, float *out,
                         int64_t n_rows, int64_t n_cols) {
    int64_t n_blocks = n_cols / ORC_Q4_K_BLOCK;
    for (int64_t row = 0; row < n_rows; row++) {
        float acc = 0.0f;
        for (int64_t blk = 0; blk < n_blocks; blk++) {
            const uint8_t *b = w + (size_t)(row * n_blocks + blk) * ORC_Q4_K_BYTES;
            acc = q4k_block_dot(b, x + blk * ORC_Q4_K_BLOCK, acc);
        }
        out[row] = acc; /* :506 overwrite */
    }
}

/* swamp-kernels/src/fused_gemv_q4k.rs:650-698: block-outer, row, token; a
 * fresh acc per (blk,row,token), then out += acc. */
void orc_gemv_q4k_batched_scalar(const uint8_t *w, const float *const *x_ptrs,
                                 float *const *out_ptrs, int64_t n_rows,
                                 int64_t n_cols, int64_t batch) {
    int64_t n_blocks = n_cols / ORC_Q4_K_BLOCK;
    for (int64_t blk = 0; blk < n_blocks; blk++) {
        int64_t off = blk * ORC_Q4_K_BLOCK;
        for (int64_t row = 0; row < n_rows; row++) {
            const uint8_t *b = w + (size_t)(row * n_blocks + blk) * ORC_Q4_K_BYTES;
            for (int64_t t = 0; t < batch; t++) {
                float acc = q4k_block_dot(b, x_ptrs[t] + off, 0.0f);
                out_ptrs[t][row] += acc;
            }
        }
    }
}

/* swamp-kernels/src/fused_gemv_q4k.rs:401-460 */
void orc_gemv_q4k_multi(const uint8_t *const *raws, const float *x,
                        float *const *outputs, const int64_t *row_counts,
                        int64_t n_matrices, int64_t n_cols) {
    int64_t n_blocks = n_cols / ORC_Q4_K_BLOCK;
    for (int64_t m = 0; m < n_matrices; m++)
        memset(outputs[m], 0, (size_t)row_counts[m] * sizeof(float));
    for (int64_t blk = 0; blk < n_blocks; blk++) {
        for (int64_t m = 0; m < n_matrices; m++) {
            for (int64_t row = 0; row < row_counts[m]; row++) {
                const uint8_t *b = raws[m] + (size_t)(row * n_blocks + blk) * ORC_Q4_K_BYTES;
                float acc = outputs[m][row];            /* :436 */
                acc = q4k_block_dot(b, x + blk * ORC_Q4_K_BLOCK, acc);
                outputs[m][row] = acc;                  /* :456 */
            }
        }
    }
}

/* swamp-kernels/src/fused_gemv_q4k.rs:799-823 (the C ABI precedent). On this
 * restatement the dispatched body is the scalar path, see the header note. */
void orc_swamp_fused_gemv_q4k(const uint8_t *w, const float *x, float *out,
                              int n_rows, int n_cols) {
    if (!w || !x || !out) return;
    if (n_cols % ORC_Q4_K_BLOCK != 0) return;
    memset(out, 0, (size_t)n_rows * sizeof(float));
    orc_gemv_q4k_scalar(w, x, out, n_rows, n_cols);
}

/* ------------------------------------------------------------------------- */
/* Engine routes (swamp-engine/src/linear.rs)                                */
/* ------------------------------------------------------------------------- */

static void dot_rows(const float *deq, const float *x, float *out, int64_t r0,
                     int64_t r1, int64_t nc) {
    for (int64_t i = r0; i < r1; i++) {
        const float *row = deq + (size_t)i * (size_t)nc;
        float s = 0.0f;
        for (int64_t j = 0; j < nc; j++) s += row[j] * x[j]; /* linear.rs:81 */
        out[i] = s;
    }
}

/* swamp-engine/src/linear.rs:68-87 */
int orc_linear_q4_0(const uint8_t *w, const float *x, float *out,
                    int64_t n_rows, int64_t n_cols, float *deq_scratch) {
    size_t n = (size_t)n_rows * (size_t)n_cols;
    float *deq = deq_scratch ? deq_scratch : (float *)malloc(n * sizeof(float));
    if (!deq) return -3;
    size_t raw_len = (size_t)n_rows * (size_t)(n_cols / ORC_Q4_0_BLOCK) * ORC_Q4_0_BYTES;
    int rc = orc_q4_0_dequant(w, raw_len, deq, n);
    if (rc == 0) dot_rows(deq, x, out, 0, n_rows, n_cols);
    if (!deq_scratch) free(deq);
    return rc;
}

typedef struct {
    int kind; /* 0 q4k gemv, 1 dot rows, 2 q4k batched, 3 q6k gemv */
    const uint8_t *w;
    const float *x;
    const float *const *xs;
    float *const *outs;
    float *out;
    const float *deq;
    int64_t r0, r1, nc, batch;
} orc_task;

static void *orc_worker(void *arg) {
    orc_task *t = (orc_task *)arg;
    if (t->r0 >= t->r1) return NULL;
    int64_t rc = t->r1 - t->r0;
    if (t->kind == 0) {
        size_t row_bytes = (size_t)(t->nc / ORC_Q4_K_BLOCK) * ORC_Q4_K_BYTES;
        orc_gemv_q4k_scalar(t->w + (size_t)t->r0 * row_bytes, t->x, t->out + t->r0, rc, t->nc);
    } else if (t->kind == 1) {
        for (int64_t b = 0; b < t->batch; b++)
            dot_rows(t->deq, t->xs[b], t->outs[b], t->r0, t->r1, t->nc);
    } else if (t->kind == 3) {
        size_t row_bytes = (size_t)(t->nc / ORC_Q6_K_BLOCK) * ORC_Q6_K_BYTES;
        orc_gemv_q6k_scalar(t->w + (size_t)t->r0 * row_bytes, t->x, t->out + t->r0, rc, t->nc);
    } else {
        size_t row_bytes = (size_t)(t->nc / ORC_Q4_K_BLOCK) * ORC_Q4_K_BYTES;
        float *local_outs[1024];
        int64_t bs = t->batch > 1024 ? 1024 : t->batch;
        for (int64_t b = 0; b < bs; b++) local_outs[b] = t->outs[b] + t->r0;
        orc_gemv_q4k_batched_scalar(t->w + (size_t)t->r0 * row_bytes, t->xs,
                                    local_outs, rc, t->nc, bs);
    }
    return NULL;
}

static void run_partitioned(orc_task proto, int64_t nr, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    orc_task tasks[256];
    int64_t rpt = (nr + n_threads - 1) / n_threads; /* linear.rs:29 */
    for (int t = 0; t < n_threads; t++) {
        tasks[t] = proto;
        tasks[t].r0 = (int64_t)t * rpt;              /* :36 */
        tasks[t].r1 = tasks[t].r0 + rpt < nr ? tasks[t].r0 + rpt : nr; /* :37 */
        if (tasks[t].r0 > nr) tasks[t].r0 = nr;
    }
    if (n_threads == 1) {
        orc_worker(&tasks[0]);
        return;
    }
    for (int t = 0; t < n_threads; t++) pthread_create(&th[t], NULL, orc_worker, &tasks[t]);
    for (int t = 0; t < n_threads; t++) pthread_join(th[t], NULL);
}

/* swamp-engine/src/linear.rs:14-90 */
int orc_forward_linear(int dtype, const uint8_t *w, const float *x, float *out,
                       int64_t n_rows, int64_t n_cols, int n_threads) {
    orc_task proto;
    memset(&proto, 0, sizeof proto);
    proto.w = w;
    proto.x = x;
    proto.out = out;
    proto.nc = n_cols;
    if (dtype == ORC_DTYPE_Q4_K) {
        if (n_cols % ORC_Q4_K_BLOCK) return -1;
        proto.kind = 0;
        run_partitioned(proto, n_rows, n_threads);
        return 0;
    }
    if (dtype == ORC_DTYPE_Q6_K) {  /* linear.rs:48-67 */
        if (n_cols % ORC_Q6_K_BLOCK) return -1;
        proto.kind = 3;
        run_partitioned(proto, n_rows, n_threads);
        return 0;
    }
    if (dtype == ORC_DTYPE_Q4_0) {
        if (n_cols % ORC_Q4_0_BLOCK) return -1;
        size_t n = (size_t)n_rows * (size_t)n_cols;
        float *deq = (float *)malloc(n * sizeof(float)); /* :69 vec! per call */
        if (!deq) return -3;
        size_t raw_len = (size_t)n_rows * (size_t)(n_cols / ORC_Q4_0_BLOCK) * ORC_Q4_0_BYTES;
        orc_q4_0_dequant(w, raw_len, deq, n);            /* :70 single-threaded */
        const float *xs[1] = {x};
        float *outs[1] = {out};
        proto.kind = 1;
        proto.deq = deq;
        proto.xs = xs;
        proto.outs = outs;
        proto.batch = 1;
        run_partitioned(proto, n_rows, n_threads);
        free(deq);
        return 0;
    }
    return -2;
}

/* swamp-engine/src/linear.rs:176-239 */
int orc_forward_linear_batch(int dtype, const uint8_t *w, const float *const *xs,
                             float *const *outs, int64_t batch, int64_t n_rows,
                             int64_t n_cols, int n_threads) {
    if (batch == 0) return 0;
    orc_task proto;
    memset(&proto, 0, sizeof proto);
    proto.w = w;
    proto.xs = xs;
    proto.outs = outs;
    proto.nc = n_cols;
    proto.batch = batch;
    if (dtype == ORC_DTYPE_Q4_K) {
        if (n_cols % ORC_Q4_K_BLOCK) return -1;
        for (int64_t b = 0; b < batch; b++) memset(outs[b], 0, (size_t)n_rows * sizeof(float)); /* :204-207 */
        proto.kind = 2;
        run_partitioned(proto, n_rows, n_threads);
        return 0;
    }
    if (dtype == ORC_DTYPE_Q4_0) {
        if (n_cols % ORC_Q4_0_BLOCK) return -1;
        size_t n = (size_t)n_rows * (size_t)n_cols;
        float *deq = (float *)malloc(n * sizeof(float));
        if (!deq) return -3;
        size_t raw_len = (size_t)n_rows * (size_t)(n_cols / ORC_Q4_0_BLOCK) * ORC_Q4_0_BYTES;
        orc_q4_0_dequant(w, raw_len, deq, n);
        proto.kind = 1;
        proto.deq = deq;
        run_partitioned(proto, n_rows, n_threads);
        free(deq);
        return 1; /* deviation: reference routes Q4_0 batches to fallback_gemv (:336-364) */
    }
    return -2;
}

/* ------------------------------------------------------------------------- */
/* Reference test fixtures (fused_gemv_q4k.rs:708-740)                       */
/* ------------------------------------------------------------------------- */

void orc_make_q4k_block(float d, float dmin, const uint8_t scales[8],
                        const uint8_t mins[8], uint8_t nibble_val, uint8_t out[144]) {
    memset(out, 0, 144);
    uint16_t hd = orc_f32_to_f16(d), hm = orc_f32_to_f16(dmin);
    out[0] = (uint8_t)(hd & 0xFF);
    out[1] = (uint8_t)(hd >> 8);
    out[2] = (uint8_t)(hm & 0xFF);
    out[3] = (uint8_t)(hm >> 8);
    for (int j = 0; j < 4; j++) {
        out[4 + j] = (uint8_t)((scales[j] & 0x3F) | ((scales[4 + j] >> 4) << 6)); /* :714 */
        out[8 + j] = (uint8_t)((mins[j] & 0x3F) | ((mins[4 + j] >> 4) << 6));     /* :715 */
    }
    out[12] = (uint8_t)((scales[4] & 0x0F) | ((mins[4] & 0x0F) << 4));            /* :717 */
    out[13] = (uint8_t)((scales[5] & 0x0F) | ((mins[5] & 0x0F) << 4));
    out[14] = (uint8_t)((scales[6] & 0x0F) | ((mins[6] & 0x0F) << 4));
    out[15] = (uint8_t)((scales[7] & 0x0F) | ((mins[7] & 0x0F) << 4));
    for (int i = 0; i < 128; i++) out[16 + i] = (uint8_t)(nibble_val | (nibble_val << 4)); /* :721 */
}

/* :726-736; note `r as f32 * 0.1` is one f32 multiply, then an f32 add. */
void orc_make_weight(int64_t n_rows, uint8_t *out) {
    for (int64_t r = 0; r < n_rows; r++) {
        float d = 0.5f + (float)r * 0.1f;
        float dm = 0.1f + (float)r * 0.05f;
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)(((uint8_t)r + 1) & 0x3F);
            mn[j] = (uint8_t)(((uint8_t)r + 2) & 0x3F);
        }
        orc_make_q4k_block(d, dm, sc, mn, 8, out + (size_t)r * 144);
    }
}

/* :738-740 */
void orc_make_x(int64_t n_cols, float *out) {
    for (int64_t i = 0; i < n_cols; i++) out[i] = (float)(i % 100) / 50.0f - 1.0f;
}

/* ------------------------------------------------------------------------- */
/* Seeded synthetic generators                                               */
/* ------------------------------------------------------------------------- */

uint64_t orc_splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t hh(uint64_t seed, uint64_t id, uint64_t i) {
    return orc_splitmix64(seed ^ (id << 40) ^ i);
}

/* uniform [0.001, 0.01): 24 random bits, f32 multiply then f32 add, then f16 RNE */
static inline uint16_t gen_scale(uint64_t bits24) {
    float u = (float)bits24 * (1.0f / 16777216.0f);
    float v = 0.001f + 0.009f * u;
    return orc_f32_to_f16(v);
}

typedef struct {
    int kind; /* 0 q4_0, 1 q4k */
    uint64_t seed, id;
    int64_t b0, b1; /* block range */
    uint8_t *out;
} gen_task;

static void gen_q4_0_blocks(uint64_t seed, uint64_t id, int64_t b0, int64_t b1, uint8_t *out) {
    for (int64_t b = b0; b < b1; b++) {
        uint8_t *blk = out + (size_t)b * ORC_Q4_0_BYTES;
        uint64_t r0 = hh(seed, id, 4 * (uint64_t)b);
        uint64_t r1 = hh(seed, id, 4 * (uint64_t)b + 1);
        uint64_t r2 = hh(seed, id, 4 * (uint64_t)b + 2);
        uint16_t d = gen_scale(r0 >> 40);
        blk[0] = (uint8_t)(d & 0xFF);
        blk[1] = (uint8_t)(d >> 8);
        uint8_t q[32];
        for (int i = 0; i < 16; i++) q[i] = (uint8_t)((r1 >> (4 * i)) & 15);
        for (int i = 0; i < 16; i++) q[16 + i] = (uint8_t)((r2 >> (4 * i)) & 15);
        /* swamp-gguf interleaved order (q4_0.rs:31-32): byte j = q[2j] | q[2j+1]<<4 */
        for (int j = 0; j < 16; j++) blk[2 + j] = (uint8_t)(q[2 * j] | (q[2 * j + 1] << 4));
    }
}

static void gen_q4k_blocks(uint64_t seed, uint64_t id, int64_t b0, int64_t b1, uint8_t *out) {
    for (int64_t b = b0; b < b1; b++) {
        uint8_t *blk = out + (size_t)b * ORC_Q4_K_BYTES;
        uint64_t base = 32 * (uint64_t)b;
        uint64_t r0 = hh(seed, id, base);
        uint64_t r1 = hh(seed, id, base + 1);
        uint64_t r2 = hh(seed, id, base + 2);
        uint16_t d = gen_scale(r0 >> 40);
        uint16_t dm = gen_scale((r0 >> 16) & 0xFFFFFFull);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)((r1 >> (6 * j)) & 63);
            mn[j] = (uint8_t)((r2 >> (6 * j)) & 63);
        }
        /* pack scales/mins exactly as make_q4k_block (fused_gemv_q4k.rs:713-719) */
        blk[0] = (uint8_t)(d & 0xFF);
        blk[1] = (uint8_t)(d >> 8);
        blk[2] = (uint8_t)(dm & 0xFF);
        blk[3] = (uint8_t)(dm >> 8);
        for (int j = 0; j < 4; j++) {
            blk[4 + j] = (uint8_t)((sc[j] & 0x3F) | ((sc[4 + j] >> 4) << 6));
            blk[8 + j] = (uint8_t)((mn[j] & 0x3F) | ((mn[4 + j] >> 4) << 6));
        }
        for (int j = 0; j < 4; j++)
            blk[12 + j] = (uint8_t)((sc[4 + j] & 0x0F) | ((mn[4 + j] & 0x0F) << 4));
        uint8_t q[256];
        for (int h = 0; h < 16; h++) {
            uint64_t r = hh(seed, id, base + 3 + (uint64_t)h);
            for (int i = 0; i < 16; i++) q[16 * h + i] = (uint8_t)((r >> (4 * i)) & 15);
        }
        /* q4_k.rs:291-319 order: element 64p+i <- low nibble of qs[32p+i],
         * element 64p+32+i <- high nibble of qs[32p+i] */
        for (int p = 0; p < 4; p++)
            for (int i = 0; i < 32; i++)
                blk[16 + 32 * p + i] = (uint8_t)(q[64 * p + i] | (q[64 * p + 32 + i] << 4));
    }
}

/* Q6_K: d as the other types; 16 int8 scales uniform over -128..127; 256
 * 6-bit values uniform over 0..63, packed as q6_k.rs reads them (:33-46). */
static void gen_q6k_blocks(uint64_t seed, uint64_t id, int64_t b0, int64_t b1, uint8_t *out) {
    for (int64_t b = b0; b < b1; b++) {
        uint8_t *blk = out + (size_t)b * ORC_Q6_K_BYTES;
        uint64_t base = 40 * (uint64_t)b;
        uint64_t r0 = hh(seed, id, base), r1 = hh(seed, id, base + 1), r2 = hh(seed, id, base + 2);
        uint16_t d = gen_scale(r0 >> 40);
        for (int j = 0; j < 8; j++) {
            blk[192 + j] = (uint8_t)(r1 >> (8 * j));
            blk[200 + j] = (uint8_t)(r2 >> (8 * j));
        }
        blk[208] = (uint8_t)(d & 0xFF);
        blk[209] = (uint8_t)(d >> 8);
        uint8_t q[256];
        for (int g = 0; g < 32; g++) {  /* 8 values of 6 bits per draw */
            uint64_t r = hh(seed, id, base + 3 + (uint64_t)g);
            for (int i = 0; i < 8; i++) q[8 * g + i] = (uint8_t)((r >> (6 * i)) & 63);
        }
        memset(blk, 0, 192);
        for (int h = 0; h < 2; h++)
            for (int m = 0; m < 4; m++)
                for (int l = 0; l < 32; l++) {
                    uint8_t v = q[128 * h + 32 * m + l];
                    blk[64 * h + l + 32 * (m & 1)] |= (uint8_t)((v & 0xF) << (4 * (m >> 1)));
                    blk[128 + 32 * h + l] |= (uint8_t)((v >> 4) << (2 * m));
                }
    }
}

static void *gen_worker(void *arg) {
    gen_task *t = (gen_task *)arg;
    if (t->kind == 0) gen_q4_0_blocks(t->seed, t->id, t->b0, t->b1, t->out);
    else if (t->kind == 1) gen_q4k_blocks(t->seed, t->id, t->b0, t->b1, t->out);
    else gen_q6k_blocks(t->seed, t->id, t->b0, t->b1, t->out);
    return NULL;
}

static void gen_parallel(int kind, uint64_t seed, uint64_t id, int64_t n_blocks,
                         uint8_t *out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    gen_task tasks[256];
    pthread_t th[256];
    int64_t per = (n_blocks + n_threads - 1) / n_threads;
    for (int t = 0; t < n_threads; t++) {
        tasks[t].kind = kind;
        tasks[t].seed = seed;
        tasks[t].id = id;
        tasks[t].b0 = (int64_t)t * per < n_blocks ? (int64_t)t * per : n_blocks;
        tasks[t].b1 = tasks[t].b0 + per < n_blocks ? tasks[t].b0 + per : n_blocks;
        tasks[t].out = out;
    }
    if (n_threads == 1) {
        gen_worker(&tasks[0]);
        return;
    }
    for (int t = 0; t < n_threads; t++) pthread_create(&th[t], NULL, gen_worker, &tasks[t]);
    for (int t = 0; t < n_threads; t++) pthread_join(th[t], NULL);
}

void orc_gen_q4_0(uint64_t seed, uint64_t tensor_id, int64_t n_rows,
                  int64_t n_cols, uint8_t *out, int n_threads) {
    gen_parallel(0, seed, tensor_id, n_rows * (n_cols / ORC_Q4_0_BLOCK), out, n_threads);
}

void orc_gen_q4k(uint64_t seed, uint64_t tensor_id, int64_t n_rows,
                 int64_t n_cols, uint8_t *out, int n_threads) {
    gen_parallel(1, seed, tensor_id, n_rows * (n_cols / ORC_Q4_K_BLOCK), out, n_threads);
}

void orc_gen_q6k(uint64_t seed, uint64_t tensor_id, int64_t n_rows,
                 int64_t n_cols, uint8_t *out, int n_threads) {
    gen_parallel(2, seed, tensor_id, n_rows * (n_cols / ORC_Q6_K_BLOCK), out, n_threads);
}

/* N(0,1) by Box-Muller in double, rounded once to f32. */
void orc_gen_x(uint64_t seed, uint64_t tensor_id, int64_t n, float *out) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t j = 0; 2 * j < n; j++) {
        uint64_t ra = hh(seed, tensor_id, 2 * (uint64_t)j);
        uint64_t rb = hh(seed, tensor_id, 2 * (uint64_t)j + 1);
        double u1 = ((double)(ra >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        double u2 = (double)(rb >> 11) * (1.0 / 9007199254740992.0);
        double rad = sqrt(-2.0 * log(u1));
        out[2 * j] = (float)(rad * cos(two_pi * u2));
        if (2 * j + 1 < n) out[2 * j + 1] = (float)(rad * sin(two_pi * u2));
    }
}

/* ------------------------------------------------------------------------- */
/* fp64 truth                                                                */
/* ------------------------------------------------------------------------- */

int orc_gemv_f64(int dtype, const uint8_t *w, const float *x, int64_t n_rows,
                 int64_t n_cols, double *out64, double *absdot, double *l2dot) {
    size_t row_bytes;
    if (dtype == ORC_DTYPE_Q4_0) row_bytes = (size_t)(n_cols / ORC_Q4_0_BLOCK) * ORC_Q4_0_BYTES;
    else if (dtype == ORC_DTYPE_Q4_K) row_bytes = (size_t)(n_cols / ORC_Q4_K_BLOCK) * ORC_Q4_K_BYTES;
    else if (dtype == ORC_DTYPE_Q6_K) row_bytes = (size_t)(n_cols / ORC_Q6_K_BLOCK) * ORC_Q6_K_BYTES;
    else return -2;
    float *row = (float *)malloc((size_t)n_cols * sizeof(float));
    if (!row) return -3;
    for (int64_t r = 0; r < n_rows; r++) {
        int rc = orc_dequantize(dtype, w + (size_t)r * row_bytes, row_bytes, row, (size_t)n_cols);
        if (rc) {
            free(row);
            return rc;
        }
        double s = 0.0, a = 0.0, q = 0.0;
        for (int64_t k = 0; k < n_cols; k++) {
            double p = (double)row[k] * (double)x[k];
            s += p;
            a += fabs(p);
            q += p * p;
        }
        if (out64) out64[r] = s;
        if (absdot) absdot[r] = a;
        if (l2dot) l2dot[r] = sqrt(q);
    }
    free(row);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Decoder-layer operations (swamp-engine/src/ops.rs, sampler.rs)            */
/* ------------------------------------------------------------------------- */

/* rmsnorm, ops.rs:188-201: a running f32 sum of x*x, then mean, + eps,
 * 1 / sqrt, and out = x * inv * w left to right. */
void orc_rmsnorm(const float *x, const float *w, float *out, int64_t n, float eps) {
    float ss = 0.0f;
    for (int64_t i = 0; i < n; i++) ss += x[i] * x[i];
    ss /= (float)n;
    ss += eps;
    float inv = 1.0f / sqrtf(ss);
    for (int64_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* init_rope_lut, ops.rs:20-38 (theta = 10000, ops.rs:11): lut[m][k] =
 * (cos, sin) of m * (1 / 10000^(2k / head_dim)), all f32 with the libm
 * powf / cosf / sinf that Rust's f32::powf / cos / sin call. */
void orc_rope_lut(int head_dim, int64_t max_seq_len, float *lut) {
    int half = head_dim / 2;
    for (int64_t m = 0; m < max_seq_len; m++)
        for (int k = 0; k < half; k++) {
            float freq = 1.0f / powf(10000.0f, (float)(2 * k) / (float)head_dim);
            float angle = (float)m * freq;
            lut[2 * (m * half + k)] = cosf(angle);
            lut[2 * (m * half + k) + 1] = sinf(angle);
        }
}

/* apply_rope_ufc + apply_rotation_pair, ops.rs:42-80. */
void orc_rope_apply(float *q, float *k, int64_t pos, int n_q_heads, int n_kv_heads, int head_dim,
                    int64_t max_context, const float *lut) {
    int half = head_dim / 2;
    if (pos > max_context - 1) pos = max_context - 1;
    const float *cs = lut + 2 * pos * half;
    for (int pass = 0; pass < 2; pass++) {
        float *v = pass ? k : q;
        int nh = pass ? n_kv_heads : n_q_heads;
        for (int h = 0; h < nh; h++)
            for (int j = 0; j < half; j++) {
                float *e = v + (int64_t)h * head_dim + 2 * j;
                float x = e[0], y = e[1], c = cs[2 * j], s = cs[2 * j + 1];
                e[0] = x * c - y * s;
                e[1] = x * s + y * c;
            }
    }
}

/* attention, ops.rs:82-186 with the scalar dot_product_raw / weighted_sum_raw
 * (swamp-kernels/src/simd.rs:155-161,175-179): per query head h, KV head
 * h / n_rep; scores dot * scale over 0..=valid_end (valid_end = min(q_pos,
 * seq_len - 1)), -inf past it; softmax with a running max; out = sum p v.
 * k_cache / v_cache hold this sequence and layer as [kv_head][head_stride],
 * position t at t * head_dim (the reference's pages only change addressing). */
void orc_attention(float *out, const float *q, const float *k_cache, const float *v_cache, int64_t head_stride,
                   int64_t seq_len, int64_t q_pos, int n_heads, int n_kv_heads, int head_dim) {
    float scale = 1.0f / sqrtf((float)head_dim);
    int n_rep = n_heads / n_kv_heads;
    int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
    float *scores = (float *)malloc((size_t)seq_len * sizeof(float));
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + (int64_t)h * head_dim;
        const float *kb = k_cache + (int64_t)(h / n_rep) * head_stride;
        const float *vb = v_cache + (int64_t)(h / n_rep) * head_stride;
        float max_score = -INFINITY;
        for (int64_t t = 0; t <= valid_end; t++) {
            float sum = 0.0f;
            for (int d = 0; d < head_dim; d++) sum += qh[d] * kb[t * head_dim + d];
            float score = sum * scale;
            scores[t] = score;
            if (score > max_score) max_score = score;
        }
        for (int64_t t = valid_end + 1; t < seq_len; t++) scores[t] = -INFINITY;
        float sum_exp = 0.0f;
        for (int64_t t = 0; t < seq_len; t++) {
            float e = expf(scores[t] - max_score);
            scores[t] = e;
            sum_exp += e;
        }
        float inv_sum = 1.0f / sum_exp;
        for (int64_t t = 0; t < seq_len; t++) scores[t] *= inv_sum;
        float *o = out + (int64_t)h * head_dim;
        for (int d = 0; d < head_dim; d++) o[d] = 0.0f;
        for (int64_t t = 0; t <= valid_end; t++)
            for (int d = 0; d < head_dim; d++) o[d] += scores[t] * vb[t * head_dim + d];
    }
    free(scores);
}

/* silu then mul_in_place, ops.rs:203-214 */
void orc_silu_mul(float *g, const float *u, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        float val = g[i];
        g[i] = val / (1.0f + expf(-val));
    }
    for (int64_t i = 0; i < n; i++) g[i] *= u[i];
}

/* add_in_place, ops.rs:216-220 */
void orc_add(float *a, const float *b, int64_t n) {
    for (int64_t i = 0; i < n; i++) a[i] += b[i];
}

/* Greedy pick, sampler.rs:94-95: Iterator::max_by over partial_cmp keeps the
 * last of equal maxima; a NaN makes partial_cmp return None and the unwrap
 * panic, reported here as -1. */
int64_t orc_argmax(const float *logits, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 0; i < n; i++)
        if (logits[i] != logits[i]) return -1;
    for (int64_t i = 1; i < n; i++)
        if (!(logits[i] < logits[best])) best = i;
    return best;
}
