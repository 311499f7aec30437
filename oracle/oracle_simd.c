/*
 * oracle_simd.c -- TEST INFRASTRUCTURE ONLY (CPU timing baseline): the
 * reference's dispatched SIMD Q4_K GEMV paths, restated in C with the same
 * intrinsics, for timing the reference's CPU speed on this host. They are
 * NOT parity targets: both disagree with the reference's own dequantizer
 * (q4_k.rs), so their outputs are numerically divergent and only their
 * speed is used. Nothing in the product links or calls this file.
 *
 *  - orc_gemv_q4k_avx2: fused_gemv_q4k_avx2 (swamp-kernels/src/fused_gemv_q4k.rs:325-392):
 *    per row and 256-block, per sub-block sb the 16 bytes qs[16sb..16sb+16];
 *    low nibbles against x[32sb .. 32sb+16), high nibbles against
 *    x[32sb+16 .. 32sb+32), each term (sv*q - mv)*x by two FMAs, 8 lanes
 *    summed per sub-block; overwrites out.
 *  - orc_gemv_q4k_vnni: fused_gemv_q4k_vnni (:101-317): per 256-block of x,
 *    x quantized to int8 by max|x|/127 (round to nearest), then per row and
 *    sub-block one 64-byte dpbusd of the weights (q-8)^0x80 laid out
 *    [lo, hi, lo, hi] against [x[32sb..+32), x[32sb+16..+48)], four rows at
 *    a time; out[row] += quire*scale_x - sum_sb(mv*sum_x + 136*sum_x*sv).
 *    The reference reads 16 bytes past its 256-byte x buffer at sb = 7; here
 *    the buffer is padded with zeros so the same lanes read zeros instead.
 *  - orc_forward_linear_dispatched: forward_linear's row partition
 *    (swamp-engine/src/linear.rs:31-45) over the dispatcher of
 *    fused_gemv_q4k (:59-82): VNNI where the CPU has it, else AVX2. out is
 *    zeroed first (the VNNI path accumulates).
 *  - orc_fallback_gemv_dispatched: forward_linear_batch for a tensor that
 *    is not Q4_K (swamp-engine/src/linear.rs:233-236), i.e. fallback_gemv
 *    (:336-364): tokens split over threads in runs of ceil(batch/threads),
 *    each token a whole-tensor fused_gemv_q4k on one thread into a zeroed
 *    row buffer that is then copied to its output. For a Q4_0 tensor this
 *    runs the Q4_K kernel over Q4_0 bytes (both are 0.5625 B per weight,
 *    so the kernel's length check passes): the reference's batched Q4_0
 *    route, timed here as it runs.
 */
#include <immintrin.h>
#include <stdlib.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#include "oracle.h"

#define Q4K_BS 256
#define Q4K_BB 144

static inline void unpack_sc(const uint8_t *sc, uint8_t scales[8], uint8_t mins[8]) {
  orc_q4k_unpack_scales(sc, scales, mins);
}

__attribute__((target("avx2,fma"))) static void gemv_q4k_avx2(const uint8_t *w, const float *x, float *out,
                                                               int64_t n_rows, int64_t n_blocks) {
  const __m128i mask = _mm_set1_epi8(0x0F);
  for (int64_t row = 0; row < n_rows; ++row) {
    float acc = 0.f;
    for (int64_t blk = 0; blk < n_blocks; ++blk) {
      const uint8_t *b = w + (row * n_blocks + blk) * Q4K_BB;
      const float d = orc_f16_to_f32((uint16_t)(b[0] | b[1] << 8));
      const float dmin = orc_f16_to_f32((uint16_t)(b[2] | b[3] << 8));
      uint8_t scales[8], mins[8];
      unpack_sc(b + 4, scales, mins);
      const uint8_t *qs = b + 16;
      const float *xb = x + blk * Q4K_BS;
      for (int sb = 0; sb < 8; ++sb) {
        const float sv = d * (float)(scales[sb] & 0x3F);
        const float mv = dmin * (float)(mins[sb] & 0x3F);
        __m256 v_acc = _mm256_setzero_ps();
        const __m256 v_mv = _mm256_set1_ps(-mv);
        const __m256 vw = _mm256_set1_ps(sv);
        const __m128i src = _mm_loadu_si128((const __m128i *)(qs + sb * 16));
        for (int half = 0; half < 2; ++half) {
          const __m128i nib = half == 0 ? _mm_and_si128(src, mask) : _mm_and_si128(_mm_srli_epi16(src, 4), mask);
          uint8_t nb[16];
          _mm_storeu_si128((__m128i *)nb, nib);
          for (int chunk = 0; chunk < 2; ++chunk) {
            const __m128i s64 = _mm_loadl_epi64((const __m128i *)(nb + chunk * 8));
            const __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(s64));
            const __m256 vx = _mm256_loadu_ps(xb + sb * 32 + half * 16 + chunk * 8);
            v_acc = _mm256_add_ps(v_acc, _mm256_fmadd_ps(_mm256_fmadd_ps(vw, qf, v_mv), vx, _mm256_setzero_ps()));
          }
        }
        float buf[8];
        _mm256_storeu_ps(buf, v_acc);
        float s = 0.f;
        for (int i = 0; i < 8; ++i) s += buf[i];
        acc += s;
      }
    }
    out[row] = acc;
  }
}

__attribute__((target("avx512f,avx512bw,avx512vnni,avx512vl"))) static int32_t collapse(__m512i q) {
  return _mm512_reduce_add_epi32(q);
}

__attribute__((target("avx512f,avx512bw,avx512vnni,avx512vl"))) static void gemv_q4k_vnni(const uint8_t *w,
                                                                                           const float *x, float *out,
                                                                                           int64_t n_rows,
                                                                                           int64_t n_blocks) {
  const __m512i xor_mask = _mm512_set1_epi8((char)0x80);
  const __m128i mask = _mm_set1_epi8(0x0F);
  const __m128i eight = _mm_set1_epi8(8);
  int8_t x_i8[256 + 64];  // zero padding past 256 (the reference reads beyond its buffer)
  memset(x_i8, 0, sizeof x_i8);
  int32_t sum_x[8];
  __m512i va[8];
  for (int64_t blk = 0; blk < n_blocks; ++blk) {
    const float *xb = x + blk * Q4K_BS;
    __m512 mx = _mm512_setzero_ps();
    for (int j = 0; j < 256; j += 16) mx = _mm512_max_ps(mx, _mm512_abs_ps(_mm512_loadu_ps(xb + j)));
    float b16[16];
    _mm512_storeu_ps(b16, mx);
    float x_max = 0.f;
    for (int i = 0; i < 16; ++i) x_max = b16[i] > x_max ? b16[i] : x_max;
    const float inv_scale = x_max > 1e-6f ? 127.f / x_max : 0.f;
    const float scale_x = x_max > 1e-6f ? x_max / 127.f : 1.f;
    for (int j = 0; j < 256; j += 16) {
      const __m512i vi = _mm512_cvtps_epi32(_mm512_mul_ps(_mm512_loadu_ps(xb + j), _mm512_set1_ps(inv_scale)));
      _mm_storeu_si128((__m128i *)(x_i8 + j), _mm512_cvtepi32_epi8(vi));
    }
    for (int sb = 0; sb < 8; ++sb) {
      int32_t s = 0;
      for (int k = 0; k < 32; ++k) s += x_i8[sb * 32 + k];
      sum_x[sb] = s;
      const __m256i lo = _mm256_loadu_si256((const __m256i *)(x_i8 + sb * 32));
      const __m256i hi = _mm256_loadu_si256((const __m256i *)(x_i8 + sb * 32 + 16));
      va[sb] = _mm512_inserti64x4(_mm512_castsi256_si512(lo), hi, 1);
    }
    // four rows per pass with a prefetch of each row's next block, then the
    // remainder one row at a time (the reference's loop structure)
    int64_t row = 0;
    for (; row < n_rows; row += 4) {
      const int nr = n_rows - row < 4 ? (int)(n_rows - row) : 4;
      const uint8_t *qs[4];
      float d[4], dmin[4], corr[4] = {0.f, 0.f, 0.f, 0.f};
      uint8_t scales[4][8], mins[4][8];
      __m512i quire[4];
      for (int i = 0; i < nr; ++i) {
        const uint8_t *b = w + ((row + i) * n_blocks + blk) * Q4K_BB;
        if (nr == 4 && blk + 1 < n_blocks) _mm_prefetch((const char *)(b + Q4K_BB), _MM_HINT_T0);
        d[i] = orc_f16_to_f32((uint16_t)(b[0] | b[1] << 8));
        dmin[i] = orc_f16_to_f32((uint16_t)(b[2] | b[3] << 8));
        unpack_sc(b + 4, scales[i], mins[i]);
        qs[i] = b + 16;
        quire[i] = _mm512_setzero_si512();
      }
      for (int sb = 0; sb < 8; ++sb) {
        const float sx = (float)sum_x[sb] * scale_x;
        for (int i = 0; i < nr; ++i) {
          const float sv = d[i] * (float)(scales[i][sb] & 0x3F);
          const float mv = dmin[i] * (float)(mins[i][sb] & 0x3F);
          corr[i] += mv * sx + (128.0f + 8.0f) * sx * sv;
          const __m128i packed = _mm_loadu_si128((const __m128i *)(qs[i] + sb * 16));
          const __m128i lo = _mm_sub_epi8(_mm_and_si128(packed, mask), eight);
          const __m128i hi = _mm_sub_epi8(_mm_and_si128(_mm_srli_epi16(packed, 4), mask), eight);
          const __m256i w256 = _mm256_set_m128i(hi, lo);
          const __m512i w512 = _mm512_inserti64x4(_mm512_castsi256_si512(w256), w256, 1);
          quire[i] = _mm512_dpbusd_epi32(quire[i], _mm512_xor_si512(w512, xor_mask), va[sb]);
        }
      }
      for (int i = 0; i < nr; ++i) out[row + i] += (float)collapse(quire[i]) * scale_x - corr[i];
    }
  }
}

int orc_simd_path(void) {
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
      __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl"))
    return 2;  // VNNI
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return 1;  // AVX2
  return 0;
}

int orc_gemv_q4k_avx2(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols) {
  if (n_cols % Q4K_BS || orc_simd_path() < 1) return -1;
  gemv_q4k_avx2(w, x, out, n_rows, n_cols / Q4K_BS);
  return 0;
}

int orc_gemv_q4k_vnni(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols) {
  if (n_cols % Q4K_BS || orc_simd_path() < 2) return -1;
  gemv_q4k_vnni(w, x, out, n_rows, n_cols / Q4K_BS);
  return 0;
}

struct simd_job {
  const uint8_t *w;
  const float *x;
  float *out;
  int64_t r0, r1, n_blocks;
  int path;
};

static void *simd_worker(void *arg) {
  struct simd_job *j = (struct simd_job *)arg;
  if (j->r1 <= j->r0) return NULL;
  const uint8_t *w = j->w + j->r0 * j->n_blocks * Q4K_BB;
  if (j->path == 2)
    gemv_q4k_vnni(w, j->x, j->out + j->r0, j->r1 - j->r0, j->n_blocks);
  else
    gemv_q4k_avx2(w, j->x, j->out + j->r0, j->r1 - j->r0, j->n_blocks);
  return NULL;
}

int orc_forward_linear_dispatched(const uint8_t *w, const float *x, float *out, int64_t n_rows, int64_t n_cols,
                                  int n_threads) {
  const int path = orc_simd_path();
  if (n_cols % Q4K_BS || path < 1 || n_threads < 1 || n_threads > 1024) return -1;
  memset(out, 0, (size_t)n_rows * sizeof(float));
  const int64_t rpt = (n_rows + n_threads - 1) / n_threads;  // linear.rs:31-45
  pthread_t th[1024];
  struct simd_job jobs[1024];
  int started = 0;
  for (int t = 0; t < n_threads; ++t) {
    const int64_t r0 = t * rpt, r1 = r0 + rpt < n_rows ? r0 + rpt : n_rows;
    jobs[t] = (struct simd_job){w, x, out, r0, r1, n_cols / Q4K_BS, path};
    if (pthread_create(&th[t], NULL, simd_worker, &jobs[t]) == 0) {
      ++started;
    } else {
      simd_worker(&jobs[t]);
      th[t] = 0;
    }
  }
  for (int t = 0; t < n_threads; ++t)
    if (th[t]) pthread_join(th[t], NULL);
  (void)started;
  return path;
}

struct fallback_job {
  const uint8_t *w;
  const float *const *xs;
  float *const *outs;
  int64_t b0, b1, n_rows, n_blocks;
  int path, rc;
};

static void *fallback_worker(void *arg) {
  struct fallback_job *j = (struct fallback_job *)arg;
  if (j->b1 <= j->b0) return NULL;
  float *lo = (float *)malloc((size_t)j->n_rows * sizeof(float));
  if (!lo) {
    j->rc = -3;
    return NULL;
  }
  for (int64_t b = j->b0; b < j->b1; ++b) {
    memset(lo, 0, (size_t)j->n_rows * sizeof(float));
    if (j->path == 2)
      gemv_q4k_vnni(j->w, j->xs[b], lo, j->n_rows, j->n_blocks);
    else
      gemv_q4k_avx2(j->w, j->xs[b], lo, j->n_rows, j->n_blocks);
    memcpy(j->outs[b], lo, (size_t)j->n_rows * sizeof(float));
  }
  free(lo);
  return NULL;
}

int orc_fallback_gemv_dispatched(const uint8_t *w, const float *const *xs, float *const *outs, int64_t batch,
                                 int64_t n_rows, int64_t n_cols, int n_threads) {
  const int path = orc_simd_path();
  if (n_cols % Q4K_BS || path < 1 || n_threads < 1 || n_threads > 1024 || batch < 0) return -1;
  if (batch == 0) return path;
  const int64_t cs = (batch + n_threads - 1) / n_threads;  // linear.rs:340
  pthread_t th[1024];
  struct fallback_job jobs[1024];
  for (int t = 0; t < n_threads; ++t) {
    const int64_t b0 = t * cs, b1 = b0 + cs < batch ? b0 + cs : batch;
    jobs[t] = (struct fallback_job){w, xs, outs, b0, b1, n_rows, n_cols / Q4K_BS, path, 0};
    if (b1 <= b0 || pthread_create(&th[t], NULL, fallback_worker, &jobs[t]) != 0) {
      fallback_worker(&jobs[t]);
      th[t] = 0;
    }
  }
  int rc = path;
  for (int t = 0; t < n_threads; ++t) {
    if (th[t]) pthread_join(th[t], NULL);
    if (jobs[t].rc) rc = jobs[t].rc;
  }
  return rc;
}
