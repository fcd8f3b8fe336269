/*
 * wattn_oracle.h -- CPU restatement of whisper.rs's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * path and the timed CPU baseline of bench.py; nothing in the product links
 * or calls it. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm may load it.
 *
 * Every function restates one function of the reference (paths relative to
 * the whisper.rs project root):
 *   ora_softmax_inplace          crates/tensor/src/ops/softmax.rs:1-24
 *   ora_dot_f32_scalar           crates/tensor/src/simd.rs:24-45
 *   ora_flash_attention_2        crates/tensor/src/ops/attention.rs:68-242
 *   ora_single_token_mha_d64     crates/tensor/src/ops/attention.rs:246-390
 *                                (AVX2 lane order, q pre-scaled, p<1e-7 skip)
 *   ora_single_token_mha_d64_scalar  attention.rs:393-434
 *   ora_mha_with_cache           crates/whisper/src/decoder.rs:835-892
 *   ora_capture_heads            crates/whisper/src/decoder.rs:796-828
 *   ora_linear                   crates/tensor/src/ops/matmul.rs:4-110
 *   ora_layer_norm               crates/tensor/src/ops/norm.rs:67-142
 *   ora_materialized             crates/tensor/tests/test_flash_attention_tiled.rs:41-89
 *   ora_xorshift_fill            crates/tensor/tests/test_flash_attention_tiled.rs:15-35
 *
 * Parity is pinned by tolerance, not bitwise: the reference's two GEMMs are
 * matrixmultiply 0.3.11 sgemm calls (third-party, not vendored; call sites
 * attention.rs:141,207) whose summation order is restated here as plain f32
 * FMA dot products.
 */
#ifndef WATTN_ORACLE_H
#define WATTN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void ora_softmax_inplace(float *x, size_t n);
float ora_dot_f32_scalar(const float *a, const float *b, size_t n);

/* Returns 0, or -1 on the argument errors the reference asserts on. */
int ora_flash_attention_2(const float *q, const float *k, const float *v,
                          size_t t_q, size_t t_kv, size_t n_heads,
                          size_t d_model, int causal, float *out,
                          int n_threads);

int ora_single_token_mha_d64(const float *q, const float *k, const float *v,
                             size_t t_kv, size_t n_heads, size_t d_model,
                             float *out);

int ora_single_token_mha_d64_scalar(const float *q, const float *k,
                                    const float *v, size_t t_kv,
                                    size_t n_heads, size_t d_model,
                                    float *out);

int ora_mha_with_cache(const float *q, const float *k, const float *v,
                       size_t n_tokens, size_t total_tokens, size_t t_past,
                       size_t n_heads, size_t d_model, float *out);

int ora_layer_norm(const float *x, const float *gamma, const float *beta, float eps, size_t rows,
                   size_t d, float *y);

int ora_linear(const float *x, const float *w, const float *bias, size_t m, size_t n, size_t k,
               float *y, int n_threads);

int ora_capture_heads(const float *q, const float *k, size_t n_tokens, size_t n_audio,
                      size_t n_heads, size_t d_model, const int *sel_slot,
                      const int *sel_head, size_t n_sel, size_t n_selected,
                      size_t row_offset, float *out);

int ora_materialized(const float *q, const float *k, const float *v,
                     size_t t_q, size_t t_kv, size_t n_heads, size_t d_model,
                     int causal, float *out);

/* Batched driver used by tests and the CPU baseline: `batch` independent
 * flash_attention_2 calls on [batch][t][d_model] buffers (the reference has no
 * batch dimension; one call per utterance, crates/whisper/src/encoder.rs:289). */
int ora_flash_attention_2_batched(const float *q, const float *k,
                                  const float *v, size_t batch, size_t t_q,
                                  size_t t_kv, size_t n_heads, size_t d_model,
                                  int causal, float *out, int n_threads);

/* Grouped decode driver: `n_groups` groups of `group_size` query rows, each
 * group attending its own K/V [t_kv][d_model] (cross-attention of beams that
 * share one utterance's encoder states, decoder.rs:688-724). One
 * single_token_mha_d64 call per query row, spread over n_threads. */
int ora_decode_grouped(const float *q, const float *k, const float *v,
                       size_t n_groups, size_t group_size, size_t t_kv,
                       size_t n_heads, size_t d_model, float *out,
                       int n_threads);

/* xorshift32 -> U[-1,1) exactly as the reference tests generate inputs. */
void ora_xorshift_fill(uint32_t *state, float *out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
