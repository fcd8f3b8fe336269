/*
 * wattn_oracle.c -- CPU restatement of whisper.rs's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA path and the
 * timed CPU baseline ("kind": "port") of bench.py. The product never links it.
 *
 * The algorithms follow the reference line by line (citations per function,
 * paths relative to the whisper.rs project root). The reference's matrix
 * products are matrixmultiply 0.3.11 `sgemm` calls (a third-party crate that
 * is not vendored with the reference; call sites attention.rs:141 and :207).
 * They are restated here as register-blocked f32 FMA micro-kernels with the
 * same operands, alpha and beta; their summation order differs from
 * matrixmultiply's, so parity with the reference is pinned by tolerance
 * (1e-5 max-abs, the bar of crates/tensor/tests/test_flash_attention_tiled.rs),
 * not bitwise.
 */
#include "wattn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define ORA_AVX2 1
#endif

/* attention.rs:13,26 */
#define Q_TILE 128
#define KV_TILE 128

/* ---------------------------------------------------------------- softmax */

/* crates/tensor/src/ops/softmax.rs:1-24: max, exp(x - max), sum, x * (1/sum). */
void ora_softmax_inplace(float *x, size_t n) {
  if (n == 0) return;
  float max_val = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > max_val) max_val = x[i];
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf(x[i] - max_val);
    sum += x[i];
  }
  float inv_sum = 1.0f / sum;
  for (size_t i = 0; i < n; i++) x[i] *= inv_sum;
}

/* ------------------------------------------------------------------- dots */

/* crates/tensor/src/simd.rs:24-45: four partial sums, then the tail. */
float ora_dot_f32_scalar(const float *a, const float *b, size_t len) {
  size_t chunks = len / 4;
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  for (size_t i = 0; i < chunks; i++) {
    size_t base = i * 4;
    acc0 += a[base] * b[base];
    acc1 += a[base + 1] * b[base + 1];
    acc2 += a[base + 2] * b[base + 2];
    acc3 += a[base + 3] * b[base + 3];
  }
  float sum = (acc0 + acc1) + (acc2 + acc3);
  for (size_t i = chunks * 4; i < len; i++) sum += a[i] * b[i];
  return sum;
}

/* 8-lane horizontal sum in the order of attention.rs:278-288 / simd.rs
 * hsum256_ps: (lo+hi) -> movehl -> shuffle. */
static float hsum8(const float d[8]) {
  float s0 = d[0] + d[4], s1 = d[1] + d[5], s2 = d[2] + d[6], s3 = d[3] + d[7];
  float t0 = s0 + s2, t1 = s1 + s3;
  return t0 + t1;
}

/* crates/tensor/src/simd.rs:49-108 (AVX2+FMA dot_f32), emulated lane by lane:
 * four 8-lane FMA accumulators over 32-element blocks, pairwise combine,
 * leftover 8-element chunks, horizontal sum, scalar tail. */
static float dot_f32_avx2order(const float *a, const float *b, size_t len) {
  float acc[4][8] = {{0}};
  size_t n_blocks = len / 32, p = 0;
  for (size_t blk = 0; blk < n_blocks; blk++, p += 32)
    for (int u = 0; u < 4; u++)
      for (int l = 0; l < 8; l++)
        acc[u][l] = fmaf(a[p + 8 * u + l], b[p + 8 * u + l], acc[u][l]);
  float s[8];
  for (int l = 0; l < 8; l++)
    s[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  size_t rem = (len % 32) / 8;
  for (size_t c = 0; c < rem; c++, p += 8)
    for (int l = 0; l < 8; l++) s[l] = fmaf(a[p + l], b[p + l], s[l]);
  float result = hsum8(s);
  for (size_t i = len - (len % 8); i < len; i++) result += a[i] * b[i];
  return result;
}

/* -------------------------------------------------- sgemm micro-kernels */

/* S[r][c] = alpha * sum_d A[r][d] * Bt[d][c] for r < tr, c < 128 (Bt is the
 * transposed key tile, zero-padded to 128 columns). Stands in for
 * attention.rs:141-156 (matrixmultiply::sgemm with beta = 0). */
static void gemm_qkt(size_t tr, size_t d_head, float alpha, const float *q,
                     size_t q_stride, const float *kt, float *s) {
  for (size_t r0 = 0; r0 < tr; r0 += 4) {
    size_t nr = tr - r0 < 4 ? tr - r0 : 4;
    for (size_t c0 = 0; c0 < KV_TILE; c0 += 16) {
#ifdef ORA_AVX2
      __m256 acc[4][2];
      for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = _mm256_setzero_ps();
      for (size_t d = 0; d < d_head; d++) {
        __m256 b0 = _mm256_loadu_ps(kt + d * KV_TILE + c0);
        __m256 b1 = _mm256_loadu_ps(kt + d * KV_TILE + c0 + 8);
        for (size_t r = 0; r < nr; r++) {
          __m256 a = _mm256_set1_ps(q[(r0 + r) * q_stride + d]);
          acc[r][0] = _mm256_fmadd_ps(a, b0, acc[r][0]);
          acc[r][1] = _mm256_fmadd_ps(a, b1, acc[r][1]);
        }
      }
      __m256 va = _mm256_set1_ps(alpha);
      for (size_t r = 0; r < nr; r++) {
        _mm256_storeu_ps(s + (r0 + r) * KV_TILE + c0, _mm256_mul_ps(va, acc[r][0]));
        _mm256_storeu_ps(s + (r0 + r) * KV_TILE + c0 + 8, _mm256_mul_ps(va, acc[r][1]));
      }
#else
      for (size_t r = 0; r < nr; r++)
        for (size_t c = c0; c < c0 + 16; c++) {
          float acc = 0.f;
          for (size_t d = 0; d < d_head; d++)
            acc = fmaf(q[(r0 + r) * q_stride + d], kt[d * KV_TILE + c], acc);
          s[(r0 + r) * KV_TILE + c] = alpha * acc;
        }
#endif
    }
  }
}

/* ACC[r][d] += sum_c P[r][c] * V[c][d] for r < tr, c < tc, d < d_head.
 * Stands in for attention.rs:207-222 (matrixmultiply::sgemm, alpha = beta = 1). */
static void gemm_pv(size_t tr, size_t tc, size_t d_head, const float *p,
                    const float *v, size_t v_stride, float *acc_out) {
  for (size_t r0 = 0; r0 < tr; r0 += 4) {
    size_t nr = tr - r0 < 4 ? tr - r0 : 4;
    size_t d0 = 0;
#ifdef ORA_AVX2
    for (; d0 + 16 <= d_head; d0 += 16) {
      __m256 acc[4][2];
      for (size_t r = 0; r < nr; r++) {
        acc[r][0] = _mm256_loadu_ps(acc_out + (r0 + r) * d_head + d0);
        acc[r][1] = _mm256_loadu_ps(acc_out + (r0 + r) * d_head + d0 + 8);
      }
      for (size_t c = 0; c < tc; c++) {
        __m256 b0 = _mm256_loadu_ps(v + c * v_stride + d0);
        __m256 b1 = _mm256_loadu_ps(v + c * v_stride + d0 + 8);
        for (size_t r = 0; r < nr; r++) {
          __m256 a = _mm256_set1_ps(p[(r0 + r) * KV_TILE + c]);
          acc[r][0] = _mm256_fmadd_ps(a, b0, acc[r][0]);
          acc[r][1] = _mm256_fmadd_ps(a, b1, acc[r][1]);
        }
      }
      for (size_t r = 0; r < nr; r++) {
        _mm256_storeu_ps(acc_out + (r0 + r) * d_head + d0, acc[r][0]);
        _mm256_storeu_ps(acc_out + (r0 + r) * d_head + d0 + 8, acc[r][1]);
      }
    }
#endif
    for (; d0 < d_head; d0++)
      for (size_t r = 0; r < nr; r++) {
        float a = acc_out[(r0 + r) * d_head + d0];
        for (size_t c = 0; c < tc; c++)
          a = fmaf(p[(r0 + r) * KV_TILE + c], v[c * v_stride + d0], a);
        acc_out[(r0 + r) * d_head + d0] = a;
      }
  }
}

/* ------------------------------------------------------ flash_attention_2 */

typedef struct {
  const float *q, *k, *v;
  float *out;
  size_t batch, t_q, t_kv, n_heads, d_model, d_head, n_q_tiles;
  int causal;
  size_t n_tasks;
  volatile size_t next; /* shared task counter (atomic fetch-add) */
} fa2_job;

/* One (head, query tile) task of attention.rs:111-242. */
static void fa2_task(const fa2_job *job, size_t task, float *scores, float *acc,
                     float *kt) {
  size_t per_batch = job->n_heads * job->n_q_tiles;
  size_t b = task / per_batch;
  size_t t = task % per_batch;
  size_t h = t / job->n_q_tiles;
  size_t i0 = (t % job->n_q_tiles) * Q_TILE;
  size_t t_q = job->t_q, t_kv = job->t_kv, d_model = job->d_model;
  size_t d_head = job->d_head;
  size_t tr = t_q - i0 < Q_TILE ? t_q - i0 : Q_TILE;
  size_t head_offset = h * d_head;
  const float *q = job->q + b * t_q * d_model;
  const float *k = job->k + b * t_kv * d_model;
  const float *v = job->v + b * t_kv * d_model;
  float *out = job->out + b * t_q * d_model;
  int causal = job->causal;
  float scale = 1.0f / sqrtf((float)d_head); /* attention.rs:107 */
  float row_max[Q_TILE], row_sum[Q_TILE];

  memset(acc, 0, sizeof(float) * tr * d_head);
  for (size_t r = 0; r < tr; r++) {
    row_max[r] = -INFINITY;
    row_sum[r] = 0.0f;
  }
  const float *p_q = q + i0 * d_model + head_offset;

  for (size_t j0 = 0; j0 < t_kv; j0 += KV_TILE) {
    if (causal && j0 > i0 + tr - 1) break; /* attention.rs:132-134 */
    size_t tc = t_kv - j0 < KV_TILE ? t_kv - j0 : KV_TILE;

    /* transpose + zero-pad the key tile for the micro-kernel */
    for (size_t d = 0; d < d_head; d++) {
      for (size_t c = 0; c < tc; c++)
        kt[d * KV_TILE + c] = k[(j0 + c) * d_model + head_offset + d];
      for (size_t c = tc; c < KV_TILE; c++) kt[d * KV_TILE + c] = 0.0f;
    }
    gemm_qkt(tr, d_head, scale, p_q, d_model, kt, scores); /* :141-156 */

    for (size_t r = 0; r < tr; r++) { /* :159-202 */
      float *row = scores + r * KV_TILE;
      size_t end;
      if (causal) {
        size_t lim = i0 + r + 1;
        end = lim > j0 ? lim - j0 : 0;
        if (end > tc) end = tc;
      } else {
        end = tc;
      }
      if (end == 0) {
        for (size_t c = 0; c < tc; c++) row[c] = 0.0f;
        continue;
      }
      float m_tile = -INFINITY;
      for (size_t c = 0; c < end; c++) m_tile = fmaxf(m_tile, row[c]);
      float m_prev = row_max[r];
      float m_new = fmaxf(m_prev, m_tile);
      float alpha = (m_prev == -INFINITY) ? 0.0f : expf(m_prev - m_new);
      float l_tile = 0.0f;
      for (size_t c = 0; c < end; c++) {
        float p = expf(row[c] - m_new);
        row[c] = p;
        l_tile += p;
      }
      for (size_t c = end; c < tc; c++) row[c] = 0.0f; /* :192 */
      row_max[r] = m_new;
      row_sum[r] = row_sum[r] * alpha + l_tile;
      if (alpha != 1.0f) {
        float *acc_row = acc + r * d_head;
        for (size_t d = 0; d < d_head; d++) acc_row[d] *= alpha;
      }
    }
    gemm_pv(tr, tc, d_head, scores, v + j0 * d_model + head_offset, d_model,
            acc); /* :207-222 */
  }

  for (size_t r = 0; r < tr; r++) { /* :228-241 */
    float inv_sum = row_sum[r] > 0.0f ? 1.0f / row_sum[r] : 0.0f;
    float *dst = out + (i0 + r) * d_model + head_offset;
    for (size_t d = 0; d < d_head; d++) dst[d] = acc[r * d_head + d] * inv_sum;
  }
}

static void *fa2_worker(void *arg) {
  fa2_job *job = (fa2_job *)arg;
  float *scores = (float *)malloc(sizeof(float) * Q_TILE * KV_TILE);
  float *acc = (float *)malloc(sizeof(float) * Q_TILE * job->d_head);
  float *kt = (float *)malloc(sizeof(float) * KV_TILE * job->d_head);
  for (;;) {
    size_t task = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (task >= job->n_tasks) break;
    fa2_task(job, task, scores, acc, kt);
  }
  free(scores);
  free(acc);
  free(kt);
  return NULL;
}

static int resolve_threads(int n_threads) {
  if (n_threads > 0) return n_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void run_pool(void *(*fn)(void *), void *job, int n_threads,
                     size_t n_tasks) {
  int nt = resolve_threads(n_threads);
  if ((size_t)nt > n_tasks) nt = (int)n_tasks;
  if (nt <= 1) {
    fn(job);
    return;
  }
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nt);
  for (int i = 0; i < nt; i++) pthread_create(&th[i], NULL, fn, job);
  for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
  free(th);
}

int ora_flash_attention_2_batched(const float *q, const float *k,
                                  const float *v, size_t batch, size_t t_q,
                                  size_t t_kv, size_t n_heads, size_t d_model,
                                  int causal, float *out, int n_threads) {
  /* attention.rs:79-88 (asserts become an error return) */
  if (n_heads == 0 || d_model % n_heads != 0) return -1;
  size_t d_head = d_model / n_heads;
  if (t_q == 0 || batch == 0) return 0; /* :90-92 */
  if (t_kv == 0) {                      /* :93-96 */
    memset(out, 0, sizeof(float) * batch * t_q * d_model);
    return 0;
  }
  /* :102-104: one non-causal query with 64-wide heads takes the decode kernel */
  if (t_q == 1 && d_head == 64 && !causal) {
    for (size_t b = 0; b < batch; b++)
      ora_single_token_mha_d64(q + b * d_model, k + b * t_kv * d_model,
                               v + b * t_kv * d_model, t_kv, n_heads, d_model,
                               out + b * d_model);
    return 0;
  }
  fa2_job job;
  job.q = q;
  job.k = k;
  job.v = v;
  job.out = out;
  job.batch = batch;
  job.t_q = t_q;
  job.t_kv = t_kv;
  job.n_heads = n_heads;
  job.d_model = d_model;
  job.d_head = d_head;
  job.n_q_tiles = (t_q + Q_TILE - 1) / Q_TILE;
  job.causal = causal;
  job.n_tasks = batch * n_heads * job.n_q_tiles;
  job.next = 0;
  run_pool(fa2_worker, &job, n_threads, job.n_tasks);
  return 0;
}

int ora_flash_attention_2(const float *q, const float *k, const float *v,
                          size_t t_q, size_t t_kv, size_t n_heads,
                          size_t d_model, int causal, float *out,
                          int n_threads) {
  return ora_flash_attention_2_batched(q, k, v, 1, t_q, t_kv, n_heads, d_model,
                                       causal, out, n_threads);
}

/* -------------------------------------------------- single-query decode */

/* crates/tensor/src/ops/attention.rs:293-390, the AVX2+FMA kernel, emulated
 * lane by lane so that its rounding is reproduced: q is pre-scaled by 0.125
 * (:329-336), the dot uses two interleaved 8-lane FMA chains (:340-350), the
 * softmax is softmax.rs, and values with weight < 1e-7 are skipped (:366). */
int ora_single_token_mha_d64(const float *q, const float *k, const float *v,
                             size_t t_kv, size_t n_heads, size_t d_model,
                             float *out) {
  if (n_heads * 64 > d_model) return -1;
  const float scale = 0.125f;
  float stack_scores[1500];
  float *scores = t_kv <= 1500 ? stack_scores
                               : (float *)malloc(sizeof(float) * t_kv);
  for (size_t h = 0; h < n_heads; h++) {
    size_t ho = h * 64;
    float vq[64];
    for (int i = 0; i < 64; i++) vq[i] = q[ho + i] * scale;
    for (size_t j = 0; j < t_kv; j++) {
      const float *kj = k + j * d_model + ho;
      float d0[8], d1[8], d[8];
      for (int l = 0; l < 8; l++) {
        d0[l] = vq[l] * kj[l];
        d1[l] = vq[8 + l] * kj[8 + l];
        d0[l] = fmaf(vq[16 + l], kj[16 + l], d0[l]);
        d1[l] = fmaf(vq[24 + l], kj[24 + l], d1[l]);
        d0[l] = fmaf(vq[32 + l], kj[32 + l], d0[l]);
        d1[l] = fmaf(vq[40 + l], kj[40 + l], d1[l]);
        d0[l] = fmaf(vq[48 + l], kj[48 + l], d0[l]);
        d1[l] = fmaf(vq[56 + l], kj[56 + l], d1[l]);
        d[l] = d0[l] + d1[l];
      }
      scores[j] = hsum8(d);
    }
    ora_softmax_inplace(scores, t_kv);
    float acc[64] = {0};
    for (size_t j = 0; j < t_kv; j++) {
      float w = scores[j];
      if (w < 1e-7f) continue;
      const float *vj = v + j * d_model + ho;
      for (int i = 0; i < 64; i++) acc[i] = fmaf(w, vj[i], acc[i]);
    }
    memcpy(out + ho, acc, sizeof(acc));
  }
  if (scores != stack_scores) free(scores);
  return 0;
}

/* crates/tensor/src/ops/attention.rs:393-434 (portable scalar twin). */
int ora_single_token_mha_d64_scalar(const float *q, const float *k,
                                    const float *v, size_t t_kv,
                                    size_t n_heads, size_t d_model,
                                    float *out) {
  if (n_heads * 64 > d_model) return -1;
  const float scale = 0.125f;
  float *scores = (float *)malloc(sizeof(float) * (t_kv ? t_kv : 1));
  for (size_t h = 0; h < n_heads; h++) {
    size_t ho = h * 64;
    for (size_t j = 0; j < t_kv; j++) {
      float dot = 0.0f;
      for (int d = 0; d < 64; d++) dot += q[ho + d] * k[j * d_model + ho + d];
      scores[j] = dot * scale;
    }
    ora_softmax_inplace(scores, t_kv);
    float *o = out + ho;
    for (int d = 0; d < 64; d++) o[d] = 0.0f;
    for (size_t j = 0; j < t_kv; j++) {
      float w = scores[j];
      if (w < 1e-7f) continue;
      for (int d = 0; d < 64; d++) o[d] += w * v[j * d_model + ho + d];
    }
  }
  free(scores);
  return 0;
}

/* ------------------------------------------- causal attention with cache */

/* crates/whisper/src/decoder.rs:835-892: query i of n_tokens sits at position
 * t_past + i and attends keys 0..=t_past+i (:864); n_tokens == 1 with 64-wide
 * heads goes to single_token_mha_d64 over t_past + 1 keys (:852-854). */
int ora_mha_with_cache(const float *q, const float *k, const float *v,
                       size_t n_tokens, size_t total_tokens, size_t t_past,
                       size_t n_heads, size_t d_model, float *out) {
  if (n_heads == 0 || d_model % n_heads != 0) return -1;
  if (t_past + n_tokens > total_tokens) return -1;
  size_t d_head = d_model / n_heads;
  if (n_tokens == 1 && d_head == 64)
    return ora_single_token_mha_d64(q, k, v, t_past + 1, n_heads, d_model, out);
  float scale = 1.0f / sqrtf((float)d_head);
  float *scores = (float *)malloc(sizeof(float) * (total_tokens ? total_tokens : 1));
  for (size_t h = 0; h < n_heads; h++) {
    size_t ho = h * d_head;
    for (size_t i = 0; i < n_tokens; i++) {
      const float *qv = q + i * d_model + ho;
      size_t max_j = t_past + i + 1;
      for (size_t j = 0; j < max_j; j++)
        scores[j] = dot_f32_avx2order(qv, k + j * d_model + ho, d_head) * scale;
      ora_softmax_inplace(scores, max_j);
      float *o = out + i * d_model + ho;
      for (size_t d = 0; d < d_head; d++) o[d] = 0.0f;
      for (size_t j = 0; j < max_j; j++) {
        float w = scores[j];
        if (w < 1e-7f) continue;
        const float *vv = v + j * d_model + ho;
        for (size_t d = 0; d < d_head; d++) o[d] += w * vv[d];
      }
    }
  }
  free(scores);
  return 0;
}

/* ------------------------------------------------------------ linear */

/* crates/tensor/src/ops/matmul.rs:4-110 (linear / linear_parallel):
 * output[t][r] = sum_c input[t][c] * weight[r][c] (+ bias[r]), in_features
 * = k, out_features = n, num_tokens = m. The reference hands the m >= 16
 * case to matrixmultiply::sgemm (third-party, not vendored); its summation
 * order is restated as one f32 FMA chain per output. Rows spread over
 * n_threads. */
typedef struct {
  const float *x, *w, *bias;
  float *y;
  size_t m, n, k, r0, r1;
} LinJob;

static void *linear_rows(void *arg) {
  LinJob *j = (LinJob *)arg;
  for (size_t t = j->r0; t < j->r1; t++)
    for (size_t r = 0; r < j->n; r++) {
      const float *xr = j->x + t * j->k, *wr = j->w + r * j->k;
      float acc = 0.f;
      for (size_t c = 0; c < j->k; c++) acc = fmaf(xr[c], wr[c], acc);
      j->y[t * j->n + r] = acc + (j->bias ? j->bias[r] : 0.f);
    }
  return NULL;
}

int ora_linear(const float *x, const float *w, const float *bias, size_t m, size_t n, size_t k,
               float *y, int n_threads) {
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 64) n_threads = 64;
  pthread_t th[64];
  LinJob jobs[64];
  size_t per = (m + n_threads - 1) / n_threads;
  int started = 0;
  for (int i = 0; i < n_threads; i++) {
    size_t r0 = i * per, r1 = r0 + per > m ? m : r0 + per;
    if (r0 >= r1) break;
    jobs[i] = (LinJob){x, w, bias, y, m, n, k, r0, r1};
    if (pthread_create(&th[i], NULL, linear_rows, &jobs[i]) != 0) {
      linear_rows(&jobs[i]);
      jobs[i].r0 = jobs[i].r1;
      th[i] = 0;
    }
    started = i + 1;
  }
  for (int i = 0; i < started; i++)
    if (th[i]) pthread_join(th[i], NULL);
  return 0;
}

/* crates/tensor/src/ops/norm.rs:67-98 (layer_norm_row_scalar) over
 * num_tokens rows (:116-142): mean, population variance, then
 * (x - mean) / sqrt(var + eps) * gamma + beta. */
int ora_layer_norm(const float *x, const float *gamma, const float *beta, float eps, size_t rows,
                   size_t d, float *y) {
  for (size_t r = 0; r < rows; r++) {
    const float *xr = x + r * d;
    float sum = 0.f;
    for (size_t i = 0; i < d; i++) sum += xr[i];
    float mean = sum / (float)d;
    float sq = 0.f;
    for (size_t i = 0; i < d; i++) {
      float t = xr[i] - mean;
      sq += t * t;
    }
    float inv_std = 1.0f / sqrtf(sq / (float)d + eps);
    for (size_t i = 0; i < d; i++) y[r * d + i] = (xr[i] - mean) * inv_std * gamma[i] + beta[i];
  }
  return 0;
}

/* ------------------------------------------- alignment-head capture */

/* crates/whisper/src/decoder.rs:796-828 (capture_cross_attention_heads): for
 * every token row i and selected (slot, head): score_j = dot_f32(q_i, k_j)
 * over the head's dims (simd.rs lane order) * 1/sqrt(d_head), softmax_inplace
 * over the n_audio scores, copied to out[((row_offset + i) * n_selected +
 * slot) * n_audio ..]. Other slots are not touched. */
int ora_capture_heads(const float *q, const float *k, size_t n_tokens, size_t n_audio,
                      size_t n_heads, size_t d_model, const int *sel_slot,
                      const int *sel_head, size_t n_sel, size_t n_selected,
                      size_t row_offset, float *out) {
  if (n_heads == 0 || d_model % n_heads != 0) return -1;
  size_t d_head = d_model / n_heads;
  float scale = 1.0f / sqrtf((float)d_head);
  float *scores = (float *)malloc(sizeof(float) * (n_audio ? n_audio : 1));
  for (size_t i = 0; i < n_tokens; i++) {
    for (size_t s = 0; s < n_sel; s++) {
      if (sel_slot[s] < 0 || (size_t)sel_slot[s] >= n_selected || sel_head[s] < 0 ||
          (size_t)sel_head[s] >= n_heads) {
        free(scores);
        return -1;
      }
      size_t ho = (size_t)sel_head[s] * d_head;
      const float *qv = q + i * d_model + ho;
      for (size_t j = 0; j < n_audio; j++)
        scores[j] = dot_f32_avx2order(qv, k + j * d_model + ho, d_head) * scale;
      ora_softmax_inplace(scores, n_audio);
      float *dst = out + ((row_offset + i) * n_selected + (size_t)sel_slot[s]) * n_audio;
      memcpy(dst, scores, sizeof(float) * n_audio);
    }
  }
  free(scores);
  return 0;
}

/* ------------------------------------------------- materialized reference */

/* crates/tensor/tests/test_flash_attention_tiled.rs:41-89: full score matrix
 * per head, row softmax (causal rows keep min(i+1, t_kv) keys), then S.V. */
int ora_materialized(const float *q, const float *k, const float *v,
                     size_t t_q, size_t t_kv, size_t n_heads, size_t d_model,
                     int causal, float *out) {
  if (n_heads == 0 || d_model % n_heads != 0) return -1;
  size_t d_head = d_model / n_heads;
  float scale = 1.0f / sqrtf((float)d_head);
  size_t n_scores = t_q * t_kv;
  float *scores = (float *)malloc(sizeof(float) * (n_scores > 0 ? n_scores : 1));
  for (size_t h = 0; h < n_heads; h++) {
    size_t ho = h * d_head;
    for (size_t i = 0; i < t_q; i++)
      for (size_t j = 0; j < t_kv; j++) {
        float dot = 0.0f;
        for (size_t d = 0; d < d_head; d++)
          dot += q[i * d_model + ho + d] * k[j * d_model + ho + d];
        scores[i * t_kv + j] = dot * scale;
      }
    for (size_t i = 0; i < t_q; i++) {
      float *row = scores + i * t_kv;
      if (causal) {
        size_t valid = i + 1 < t_kv ? i + 1 : t_kv;
        ora_softmax_inplace(row, valid);
        for (size_t j = valid; j < t_kv; j++) row[j] = 0.0f;
      } else {
        ora_softmax_inplace(row, t_kv);
      }
    }
    for (size_t i = 0; i < t_q; i++)
      for (size_t d = 0; d < d_head; d++) {
        float sum = 0.0f;
        for (size_t j = 0; j < t_kv; j++)
          sum += scores[i * t_kv + j] * v[j * d_model + ho + d];
        out[i * d_model + ho + d] = sum;
      }
  }
  free(scores);
  return 0;
}

/* --------------------------------------------------- grouped decode driver */

typedef struct {
  const float *q, *k, *v;
  float *out;
  size_t group_size, t_kv, n_heads, d_model, n_rows;
  volatile size_t next;
} dec_job;

static void *dec_worker(void *arg) {
  dec_job *job = (dec_job *)arg;
  for (;;) {
    size_t row = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (row >= job->n_rows) break;
    size_t g = row / job->group_size;
    size_t kv_off = g * job->t_kv * job->d_model;
    ora_single_token_mha_d64(job->q + row * job->d_model, job->k + kv_off,
                             job->v + kv_off, job->t_kv, job->n_heads,
                             job->d_model, job->out + row * job->d_model);
  }
  return NULL;
}

int ora_decode_grouped(const float *q, const float *k, const float *v,
                       size_t n_groups, size_t group_size, size_t t_kv,
                       size_t n_heads, size_t d_model, float *out,
                       int n_threads) {
  if (n_heads * 64 != d_model) return -1;
  dec_job job;
  job.q = q;
  job.k = k;
  job.v = v;
  job.out = out;
  job.group_size = group_size;
  job.t_kv = t_kv;
  job.n_heads = n_heads;
  job.d_model = d_model;
  job.n_rows = n_groups * group_size;
  job.next = 0;
  if (job.n_rows == 0) return 0;
  run_pool(dec_worker, &job, n_threads, job.n_rows);
  return 0;
}

/* ------------------------------------------------------------------- RNG */

/* crates/tensor/tests/test_flash_attention_tiled.rs:15-35: xorshift32, then
 * (x as f32 / u32::MAX as f32) * 2.0 - 1.0 with round-to-nearest casts. */
void ora_xorshift_fill(uint32_t *state, float *out, size_t n) {
  uint32_t x = *state;
  const float denom = (float)UINT32_MAX;
  for (size_t i = 0; i < n; i++) {
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    out[i] = ((float)x / denom) * 2.0f - 1.0f;
  }
  *state = x;
}
