/*
 * wattn.h -- C ABI of the B200 (sm_100a) attention path for whisper.rs.
 *
 * This library replaces whisper.rs's attention hot path:
 *   crates/tensor/src/ops/attention.rs      flash_attention_2 (:68),
 *                                           multi_head_attention (:29),
 *                                           single_token_mha_d64 (:246)
 *   crates/whisper/src/decoder.rs           multi_head_attention_with_cache
 *                                           (:835), DecoderKvCache (:131-264)
 * Each entry point names the reference interface it stands in for.
 *
 * Conventions
 *   - Layout is the reference's: per utterance a row-major [t][n_heads*64]
 *     matrix, head h at columns h*64 .. h*64+63 (attention.rs:117,124). Every
 *     device entry point also takes explicit row strides (in elements), so a
 *     fused [T][3*d_model] QKV buffer can be passed without splitting it
 *     (crates/whisper/src/encoder.rs:279-286).
 *   - Head dimension must be 64 (every Whisper model); other values return
 *     WATTN_ERR_UNSUPPORTED. There is no CPU fallback.
 *   - Device entry points are asynchronous on the caller's stream
 *     (a cudaStream_t passed as void*; NULL = legacy default stream) and take
 *     device pointers only. Host entry points (wattn_*_host and the four
 *     reference-signature mirrors) take host pointers and return when the
 *     output is in host memory.
 *   - Every function returns a status: 0 = OK, negative = error. Nothing
 *     aborts or prints. wattn_last_error() gives the calling thread's last
 *     error message. All entry points are thread-safe and re-entrant.
 *   - Kernel-side waits are bounded; a wait that runs out sets a per-device
 *     status word, read (and cleared) by wattn_device_status().
 */
#ifndef WATTN_H
#define WATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define WATTN_OK 0
#define WATTN_ERR_INVALID (-1)     /* bad argument (the reference asserts) */
#define WATTN_ERR_UNSUPPORTED (-2) /* e.g. head dimension != 64 */
#define WATTN_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define WATTN_ERR_TIMEOUT (-4)     /* a bounded device wait ran out */
#define WATTN_ERR_NOMEM (-5)       /* device or page-pool memory exhausted */
#define WATTN_ERR_RANGE (-6)       /* slot / layer / position out of range */

/* ------------------------------------------------------------ element types */
#define WATTN_F32 0
#define WATTN_F16 1
#define WATTN_BF16 2

/* ABI version (major*10000 + minor*100 + patch). */
int wattn_version(void);

/* Static description of a status code. Never NULL. */
const char *wattn_status_string(int status);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len). Returns the status code of that error (0 if none). */
int wattn_last_error(char *buf, size_t len);

/* Reads and clears the device status word of `device` (the current device
 * if device < 0): WATTN_OK, or WATTN_ERR_TIMEOUT if a kernel's bounded wait
 * ran out since the last call. Synchronises that device. */
int wattn_device_status(int device, int *status);

/* ======================================================================
 * Encoder / general attention (device pointers)
 *
 * Replaces flash_attention_2 / multi_head_attention
 * (crates/tensor/src/ops/attention.rs:29-41, :68-242) for `batch`
 * independent calls. O[b] = softmax(scale * Q[b] K[b]^T [+mask]) V[b] per
 * head. causal != 0 masks key j for query i when j > i + q_pos_offset
 * (q_pos_offset = 0 is attention.rs's causal rule :161-165; t_past is
 * decoder.rs:864's). Rows whose every key is masked, and t_kv == 0, give 0.
 *
 * in_dtype  WATTN_F16 / WATTN_BF16: tcgen05 tensor-core kernel, f32
 *           accumulation. WATTN_F32: tcgen05 kernel on split-f16 operands
 *           (each f32 value as a hi and a lo f16 part, three products per
 *           product), f32 softmax and accumulation: the reference's
 *           precision (1e-5).
 * out_dtype WATTN_F32, or the input type.
 * Strides are in elements: *_row_stride between rows t and t+1 of one
 * utterance, *_batch_stride between utterances. K and V share strides.
 * 16-bit inputs need 16-byte aligned q/k/v and row/batch strides that are
 * multiples of 8 elements; outputs need 16-byte aligned rows.
 * Scratch memory is the calling host thread's library-owned workspace: one
 * thread's calls on different streams must not overlap (each host thread
 * has its own).
 * ====================================================================== */
int wattn_attention_fwd(const void *q, const void *k, const void *v, void *o,
                        int in_dtype, int out_dtype, int batch, int t_q,
                        int t_kv, int n_heads, int d_head,
                        int64_t q_row_stride, int64_t kv_row_stride,
                        int64_t o_row_stride, int64_t q_batch_stride,
                        int64_t kv_batch_stride, int64_t o_batch_stride,
                        float scale, int causal, int q_pos_offset,
                        void *stream);

/* ======================================================================
 * Decoder decode attention over dense K/V (device pointers)
 *
 * Replaces single_token_mha_d64 (attention.rs:246-434), reached from
 * flash_attention_2 for t_q == 1 (:102-104) and from the decoder's
 * cross-attention (decoder.rs:698). n_groups groups of group_size query
 * rows; every row of group g attends the same K/V block of t_kv rows
 * (the beams of one utterance share its cross-attention K/V,
 * decoder.rs:137-139). Query row r = g*group_size + i lives at
 * q + r*q_row_stride, its output at o + r*o_row_stride; group g's keys at
 * k + g*kv_group_stride + j*kv_row_stride (same for v).
 *
 * Split-KV: the keys are cut into chunks processed by separate CTAs and
 * merged by a log-sum-exp reduction. `workspace` (device memory of at least
 * wattn_decode_workspace_bytes() bytes, zero-filled before its first use and
 * left zeroed by every call) holds the partials; pass NULL to use a
 * library-owned workspace of the calling host thread (one per device).
 * Calls that pass NULL share that workspace, so one thread's NULL-workspace
 * calls on different streams must not run at the same time; give each
 * stream its own workspace instead. wattn_attention_fwd has no workspace
 * argument and always uses that per-thread buffer (split partials, V's f16
 * copy, the split f32 operands), so the same rule applies to it.
 * q_dtype / out_dtype: F32, F16 or BF16. kv_dtype: F32, F16 or BF16.
 * k and v: 16-byte aligned, row and group strides multiples of 16 bytes;
 * q and o: aligned to their element size (a 16-bit q: 4 bytes, with an even
 * row stride). Misaligned pointers return WATTN_ERR_INVALID.
 * ====================================================================== */
size_t wattn_decode_workspace_bytes(int n_groups, int group_size, int t_kv,
                                    int n_heads);

int wattn_decode_fwd(const void *q, const void *k, const void *v, void *o,
                     int q_dtype, int kv_dtype, int out_dtype, int n_groups,
                     int group_size, int t_kv, int n_heads, int d_head,
                     int64_t q_row_stride, int64_t kv_row_stride,
                     int64_t kv_group_stride, int64_t o_row_stride,
                     float scale, void *workspace, size_t workspace_bytes,
                     void *stream);

/* Cross-attention decode with alignment-head capture: the DTW path of
 * decode_with_alignment_heads, where multi_head_attention over the encoder
 * states is followed by capture_cross_attention_heads
 * (crates/whisper/src/decoder.rs:698-722, 796-828). Same arguments and
 * output as wattn_decode_fwd, plus the capture, computed from the same dot
 * products as the attention (one pass over K):
 *   sel_slot[i], sel_head[i], i < n_sel: the reference's `selected` pairs
 *     (capture slot, model head); each head at most once per call
 *     (WATTN_ERR_UNSUPPORTED otherwise), heads < 64;
 *   capture: device f32, [rows][n_selected][t_kv]; query row r (over all
 *     groups, r = group * group_size + i) gets, for each selected pair,
 *     softmax_j(scale * q_r . k_j) at capture[((row_offset + r) * n_selected
 *     + slot) * t_kv + j]; other slots are left as they are.
 * The softmax is exact in f32 over the kernel's dot products (the p < 1e-7
 * skip of the attention output does not apply to the capture, as in the
 * reference). */
int wattn_decode_fwd_capture(const void *q, const void *k, const void *v, void *o,
                             int q_dtype, int kv_dtype, int out_dtype, int n_groups,
                             int group_size, int t_kv, int n_heads, int d_head,
                             int64_t q_row_stride, int64_t kv_row_stride,
                             int64_t kv_group_stride, int64_t o_row_stride,
                             float scale, void *workspace, size_t workspace_bytes,
                             const int *sel_slot, const int *sel_head, int n_sel,
                             int n_selected, int row_offset, float *capture,
                             void *stream);

/* Linear projection y = x W^T (+ bias) on the tensor cores: Weight::linear
 * (crates/tensor/src/weight.rs:121, ops/matmul.rs:4-110: output[t][r] =
 * sum_c x[t][c] W[r][c] + bias[r]) with 16-bit x and W (both in_dtype:
 * f16 or bf16; f32 accumulation). x [m][k] (row stride x_row_stride), W
 * [n][k] (w_row_stride), y [m][n] (y_row_stride) in out_dtype; bias: device
 * f32 [n] or NULL. x and W must be 16-byte aligned with row strides whose
 * byte size is a multiple of 16; y and bias aligned to their element size. */
int wattn_linear_fwd(const void *x, const void *w, const float *bias, void *y,
                     int in_dtype, int out_dtype, int m, int n, int k,
                     int64_t x_row_stride, int64_t w_row_stride,
                     int64_t y_row_stride, void *stream);

/* precompute_cross_attn for one layer (crates/whisper/src/decoder.rs:423-447)
 * on the device: k_out = enc Wk^T and v_out = enc Wv^T + bv, [n_tokens]
 * [d_model] each (row stride kv_row_stride), with Wk, Wv [d_model][d_model]
 * in in_dtype and bv device f32 [d_model]. The outputs are the K and V that
 * wattn_decode_fwd reads for one utterance (n_tokens = its encoder states). */
int wattn_cross_kv_project(const void *enc, const void *wk, const void *wv,
                           const float *bv, void *k_out, void *v_out,
                           int in_dtype, int out_dtype, int n_tokens, int d_model,
                           int64_t enc_row_stride, int64_t kv_row_stride,
                           void *stream);

/* The attention sub-block of an encoder layer (crates/whisper/src/encoder.rs:
 * 276-303) after its pre-LN: qkv = x W_qkv^T + b_qkv (W_qkv [3d][d]), the
 * non-causal attention of each utterance's T rows over q, k, v read in place
 * from the fused [T][3d] rows (the reference splits them into three copies,
 * :281-286), then y = attn W_out^T + b_out. x [batch*t][d] and the weights
 * in in_dtype (f16/bf16), biases device f32, y in out_dtype; d = n_heads*64.
 * The residual add (:304) stays with the caller. workspace: device, 256-byte
 * aligned, at least wattn_encoder_attention_workspace_bytes() bytes. */
size_t wattn_encoder_attention_workspace_bytes(int batch, int t, int n_heads);
int wattn_encoder_attention(const void *x, const void *w_qkv, const float *b_qkv,
                            const void *w_out, const float *b_out, void *y,
                            int in_dtype, int out_dtype, int batch, int t,
                            int n_heads, void *workspace, size_t workspace_bytes,
                            void *stream);

/* The whole attention sub-block of an encoder layer, steps (a)-(d) of
 * crates/whisper/src/encoder.rs:266-304, in place on the f32 residual stream
 * x [batch*t][d]: x += out_proj(attention(qkv_proj(layer_norm(x)))), with
 * layer_norm(eps 1e-5, ln_w / ln_b f32, crates/tensor/src/ops/norm.rs:116)
 * rounded to `dtype` (f16/bf16) for the projections, the weights in dtype,
 * the biases f32. Same workspace as wattn_encoder_attention. */
int wattn_encoder_attention_residual(float *x, const float *ln_w, const float *ln_b,
                                     const void *w_qkv, const float *b_qkv,
                                     const void *w_out, const float *b_out, int dtype,
                                     int batch, int t, int n_heads, void *workspace,
                                     size_t workspace_bytes, void *stream);

/* Decode without any allocation. This entry point has no counterpart in the
 * reference: it exists for callers that may not allocate device memory at
 * all (a real-time audio callback, a host whose allocator is frozen after
 * start-up, a runtime that only hands out pre-registered buffers), so they
 * can neither pass a workspace nor let wattn_decode_fwd allocate one.
 * Same arguments and results as wattn_decode_fwd without the workspace: the
 * split partials and merge counters live in an 8 MiB array compiled into
 * the library, which every GPU that loads the library keeps until the
 * process exits. A call whose plan needs more scratch than that returns
 * WATTN_ERR_RANGE. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. The address is kept for the life of the
 * process: after cudaDeviceReset on a device, do not call this entry point
 * there again. All calls on a device share the array: calls whose kernels
 * overlap on the GPU race and give wrong results. Arguments are checked by
 * the same rules as wattn_decode_fwd before anything is launched. No
 * cudaMalloc, cudaFree or other allocating routine is called. */
int wattn_decode_fwd_noalloc(const void *q, const void *k, const void *v,
                             void *o, int q_dtype, int kv_dtype,
                             int out_dtype, int n_groups, int group_size,
                             int t_kv, int n_heads, int d_head,
                             int64_t q_row_stride, int64_t kv_row_stride,
                             int64_t kv_group_stride, int64_t o_row_stride,
                             float scale, void *stream);

/* ======================================================================
 * Device-resident paged KV cache (replaces DecoderKvCache,
 * crates/whisper/src/decoder.rs:131-264, and the per-slot truncate/append
 * of decode_batch_inner, decoder.rs:616-647)
 *
 * One cache holds the self-attention K/V of n_layers layers for a set of
 * slots (beam hypotheses). Storage is a pool of pages on the device; a page
 * holds page_rows consecutive positions of one slot for every layer, K and
 * V, every head: [page][layer][K|V][head][page_rows][64]. A slot's history is
 * its page table (host-side, mirrored to the device when it changes) plus
 * a start offset (rows dropped by slide_to_fit) and its length t_past.
 * Forking a slot (copy_slot) shares its full pages and copies only the
 * partially filled last page; a shared page is copied before it is
 * written (copy on write).
 *
 * Semantics follow the reference exactly: append() writes n rows at
 * positions t_past .. t_past+n-1 after dropping rows >= t_past (the rewind
 * of decoder.rs:631-633); attend() runs causal attention of those n rows
 * over positions 0 .. t_past+i (decoder.rs:835-892); advance() adds n to
 * t_past after the last layer (decoder.rs:765-767).
 * All functions taking a stream enqueue their device work on it; the others
 * only change host-side state.
 * ====================================================================== */
typedef struct wattn_kv_cache wattn_kv_cache;

/* DecoderKvCache::new (decoder.rs:147). n_pages = 0 sizes the pool for every
 * slot at max_ctx plus one copy-on-write page per slot. The cache lives on
 * the current device. */
int wattn_kv_create(wattn_kv_cache **out, int n_layers, int n_slots,
                    int n_heads, int d_head, int max_ctx, int page_rows,
                    int n_pages, int dtype);
int wattn_kv_destroy(wattn_kv_cache *cache);

int wattn_kv_clear(wattn_kv_cache *cache);                 /* :161-173 */
int wattn_kv_clear_slot(wattn_kv_cache *cache, int slot);  /* :176-186 */
int wattn_kv_ensure_slots(wattn_kv_cache *cache, int n_slots); /* :203-214 */
int wattn_kv_copy_slot(wattn_kv_cache *cache, int dst, int src,
                       void *stream);                      /* :220-234 */

/* The slot assignment of BeamSearch::step (crates/whisper/src/beam.rs:418-460)
 * as one call: parent_slot[i] is the slot of retained branch i (in ranking
 * order). Every parent slot is reserved; the first child of a parent keeps
 * its slot, each further child gets the lowest free slot at or after the
 * previous one and a fork of its parent (copy_slot: the pages are shared,
 * nothing is copied until a write). out_slot[i] receives branch i's slot.
 * WATTN_ERR_RANGE if the slots run out (the reference panics: "beam slot
 * arena exhausted"); the cache is then unchanged. */
int wattn_kv_assign_beams(wattn_kv_cache *cache, const int *parent_slot,
                          int n_branches, int *out_slot);
int wattn_kv_slot_len(const wattn_kv_cache *cache, int slot,
                      int *len);                           /* :237-239 */
int wattn_kv_slide_to_fit(wattn_kv_cache *cache, int slot, int n_new,
                          int max_ctx, int *pos);          /* :248-263 */
/* The C API rewind: whisper_decode_with_state sets t_past = n_past
 * (crates/ffi/src/lib.rs:2352). Rows >= n_past are dropped by the next
 * append. n_past may not exceed the slot's current length. */
int wattn_kv_set_t_past(wattn_kv_cache *cache, int slot, int n_past);
/* t_past[slots[i]] += n_tokens[i] (decoder.rs:765-767). */
int wattn_kv_advance(wattn_kv_cache *cache, const int *slots,
                     const int *n_tokens, int n_seqs);

/* Append n_tokens[i] new K/V rows for slots[i] into `layer`
 * (decoder.rs:631-635). Rows are packed sequence-major as in the reference
 * (k_rows + (sum_{i'<i} n_tokens[i'] + t) * row_stride), width
 * n_heads*64, type src_dtype, aligned to its element size. slots /
 * n_tokens are host arrays. */
int wattn_kv_append(wattn_kv_cache *cache, int layer, const int *slots,
                    const int *n_tokens, int n_seqs, const void *k_rows,
                    const void *v_rows, int src_dtype, int64_t row_stride,
                    void *stream);

/* Causal self-attention of the appended rows over each slot's history in
 * `layer` (multi_head_attention_with_cache, decoder.rs:835-892). q / o rows
 * packed like k_rows above, each aligned to its element size (a 16-bit q:
 * 4 bytes, with an even row stride). `workspace` as for wattn_decode_fwd
 * (wattn_kv_workspace_bytes), or NULL. */
size_t wattn_kv_workspace_bytes(const wattn_kv_cache *cache, int n_rows);
int wattn_kv_attend(wattn_kv_cache *cache, int layer, const int *slots,
                    const int *n_tokens, int n_seqs, const void *q,
                    int q_dtype, int64_t q_row_stride, void *o, int out_dtype,
                    int64_t o_row_stride, float scale, void *workspace,
                    size_t workspace_bytes, void *stream);

/* Device copy of one slot's rows of one layer, in the reference's flat
 * layout ([t_past][n_heads*64], dtype out_dtype), for inspection and tests
 * (the k_self / v_self fields of decoder.rs:133-135). `which` 0 = K, 1 = V. */
int wattn_kv_read_slot(wattn_kv_cache *cache, int layer, int slot, int which,
                       void *out, int out_dtype, void *stream);

/* Pool statistics: pages in use and pool size. */
int wattn_kv_stats(const wattn_kv_cache *cache, int *pages_used,
                   int *pages_total);

/* ======================================================================
 * Host-buffer entry points (the reference-facing calls)
 *
 * Same math as the device entry points, on host buffers: inputs are copied
 * to the current device, computed, and copied back before returning. Each
 * calling thread gets its own device buffers and streams, kept between
 * calls. Pinned (page-locked) host buffers give full copy bandwidth; large
 * batches are processed in chunks whose copies overlap the kernels.
 * ====================================================================== */

/* flash_attention_2 (attention.rs:68), f32 host slices, one utterance:
 * q [t_q][d_model], k/v [t_kv][d_model], output [t_q][d_model]. */
int wattn_flash_attention_2(const float *q, const float *k, const float *v,
                            size_t t_q, size_t t_kv, size_t n_heads,
                            size_t d_model, int causal, float *output);

/* multi_head_attention (attention.rs:29): same as flash_attention_2. */
int wattn_multi_head_attention(const float *q, const float *k, const float *v,
                               size_t t_q, size_t t_kv, size_t n_heads,
                               size_t d_model, int causal, float *output);

/* single_token_mha_d64 (attention.rs:246): one query row, t_kv keys. */
int wattn_single_token_mha_d64(const float *q, const float *k, const float *v,
                               size_t t_kv, size_t n_heads, size_t d_model,
                               float *output);

/* multi_head_attention_with_cache (decoder.rs:835): n_tokens queries at
 * positions t_past .. t_past+n_tokens-1 over total_tokens cached rows. */
int wattn_multi_head_attention_with_cache(const float *q, const float *k,
                                          const float *v, size_t n_tokens,
                                          size_t total_tokens, size_t t_past,
                                          size_t n_heads, size_t d_model,
                                          float *output);

/* capture_cross_attention_heads (crates/whisper/src/decoder.rs:796-828) on
 * host f32 slices: q [n_tokens][d_model], k [n_audio][d_model]; for every
 * (sel_slot[i], sel_head[i]) and token row t, out[((row_offset + t) *
 * n_selected + slot) * n_audio + j] = softmax_j(q_t . k_j / sqrt(d_head))
 * over the head's 64 dims; the other slots of `out` are left unchanged.
 * Runs the fused capture of wattn_decode_fwd_capture. d_model must be
 * n_heads * 64; heads < 64, each selected at most once. */
int wattn_capture_cross_attention_heads(const float *q, const float *k, size_t n_tokens,
                                        size_t n_audio, size_t n_heads, size_t d_model,
                                        const int *sel_slot, const int *sel_head,
                                        size_t n_sel, size_t n_selected,
                                        size_t row_offset, float *out);

/* Batched host-buffer encoder attention: contiguous [batch][t][n_heads*64]
 * host buffers of in_dtype; output [batch][t_q][n_heads*64] of out_dtype. */
int wattn_attention_host(const void *q, const void *k, const void *v, void *o,
                         int in_dtype, int out_dtype, int batch, int t_q,
                         int t_kv, int n_heads, float scale, int causal);

/* Batched host-buffer decode: q [n_groups*group_size][n_heads*64] (q_dtype),
 * k/v [n_groups][t_kv][n_heads*64] (kv_dtype), o like q (out_dtype). */
int wattn_decode_host(const void *q, const void *k, const void *v, void *o,
                      int q_dtype, int kv_dtype, int out_dtype, int n_groups,
                      int group_size, int t_kv, int n_heads, float scale);

/* ======================================================================
 * Self-test of the bounded-wait machinery: launches one kernel that waits,
 * with a limit of `limit_us` microseconds, on a device flag that nothing
 * sets, then reports through the device status word. Returns
 * WATTN_ERR_TIMEOUT when the wait ran out as designed (and the device stays
 * usable), WATTN_OK if the flag was somehow set.
 * ====================================================================== */
int wattn_selftest_bounded_wait(int limit_us, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* WATTN_H */
