// api.cu -- the extern "C" boundary: argument checks, dispatch to the
// kernels, error reporting, host-buffer entry points and the bounded-wait
// self-test. Declarations and contracts are in include/wattn.h.

#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "wattn_common.cuh"
#include "wattn_internal.h"

namespace wattn {

// [0] status word, [1] site of the first bounded wait that ran out.
__device__ int g_status[2] = {WATTN_OK, 0};

namespace {

thread_local int t_err_status = WATTN_OK;
thread_local char t_err_msg[512] = {0};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int *g_status_ptr[kMaxDevices] = {nullptr};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int set_error(int status, const char *fmt, ...) {
  t_err_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err_msg, sizeof(t_err_msg), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() {
  t_err_status = WATTN_OK;
  t_err_msg[0] = 0;
}

int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return WATTN_OK;
  return set_error(WATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int *device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error(WATTN_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) {
      check_launch("cudaGetSymbolAddress(status word)");
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<int *>(p);
  }
  return g_status_ptr[dev];
}

int encode_tmap(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, const void *base,
                const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      void *fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        cudaGetLastError();
        return set_error(WATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, dtype, rank, const_cast<void *>(base), d, s, b, e,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(WATTN_ERR_INVALID,
                     "TMA descriptor rejected (error %d): base %p must be 16-byte aligned and "
                     "row strides multiples of 16 bytes",
                     (int)r, base);
  return WATTN_OK;
}

namespace {

struct Workspace {
  void *ptr = nullptr;
  size_t bytes = 0;
};
thread_local Workspace t_ws[kMaxDevices];

}  // namespace

void *thread_workspace(size_t bytes, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  Workspace &w = t_ws[dev];
  if (w.bytes < bytes) {
    if (w.ptr) {
      cudaDeviceSynchronize();
      cudaFree(w.ptr);
    }
    w.ptr = nullptr;
    w.bytes = 0;
    const size_t sz = std::max(bytes, (size_t)1 << 20);
    if (cudaMalloc(&w.ptr, sz) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    if (cudaMemsetAsync(w.ptr, 0, sz, stream) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(w.ptr);
      w.ptr = nullptr;
      return nullptr;
    }
    w.bytes = sz;
  }
  return w.ptr;
}

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__global__ void bounded_wait_kernel(volatile int *flag, int *status,
                                    unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer_ns();
  while (*flag == 0) {
    if (globaltimer_ns() - t0 > limit_ns) {
      report_timeout(status, (9 << 24));
      return;
    }
    __nanosleep(1000);
  }
}

// ----------------------------------------------------------- host contexts
// Per calling thread and device: two streams and their device buffers, so a
// host-buffer call can overlap the copies of one chunk with the kernel of
// the previous one.
struct HostCtx {
  cudaStream_t st[2] = {nullptr, nullptr};
  void *buf[2] = {nullptr, nullptr};
  size_t buf_bytes[2] = {0, 0};
  void *ws[2] = {nullptr, nullptr};
  size_t ws_bytes[2] = {0, 0};
  bool ok = false;
};
thread_local HostCtx t_host[kMaxDevices];

HostCtx *host_ctx() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error(WATTN_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  HostCtx &h = t_host[dev];
  if (!h.ok) {
    for (int i = 0; i < 2; ++i)
      if (cudaStreamCreateWithFlags(&h.st[i], cudaStreamNonBlocking) != cudaSuccess) {
        check_launch("cudaStreamCreate");
        return nullptr;
      }
    h.ok = true;
  }
  return &h;
}

int grow(void **p, size_t *have, size_t need, bool zero, cudaStream_t st) {
  if (*have >= need) return WATTN_OK;
  if (*p) {
    cudaStreamSynchronize(st);
    cudaFree(*p);
  }
  *p = nullptr;
  *have = 0;
  if (cudaMalloc(p, need) != cudaSuccess) {
    cudaGetLastError();
    return set_error(WATTN_ERR_NOMEM, "cudaMalloc(%zu) failed", need);
  }
  if (zero && cudaMemsetAsync(*p, 0, need, st) != cudaSuccess) return check_launch("cudaMemsetAsync");
  *have = need;
  return WATTN_OK;
}

int h2d(void *dst, const void *src, size_t n, cudaStream_t st) {
  if (n == 0) return WATTN_OK;
  if (cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return check_launch("cudaMemcpyAsync H2D");
  return WATTN_OK;
}
int d2h(void *dst, const void *src, size_t n, cudaStream_t st) {
  if (n == 0) return WATTN_OK;
  if (cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return check_launch("cudaMemcpyAsync D2H");
  return WATTN_OK;
}

// Ends a host-buffer call: waits for both streams, then reports CUDA errors
// and the device status word.
int consume_status();

// After a bounded wait ran out, a kernel may have left split counters
// counted up: zero the counter regions of the calling thread's workspaces on
// the current device, so that the next launch's last-part detection starts
// clean. (Caller-owned workspaces are zeroed by the launches that use them.)
void reset_split_counters() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  cudaDeviceSynchronize();
  if (t_ws[dev].ptr) cudaMemset(t_ws[dev].ptr, 0, std::min(t_ws[dev].bytes, kCounterBytes));
  HostCtx &h = t_host[dev];
  for (int i = 0; i < 2; ++i)
    if (h.ws[i]) cudaMemset(h.ws[i], 0, std::min(h.ws_bytes[i], kCounterBytes));
  cudaDeviceSynchronize();
}

int finish_host(HostCtx *h, int rc) {
  for (int i = 0; i < 2; ++i)
    if (cudaStreamSynchronize(h->st[i]) != cudaSuccess && rc == WATTN_OK)
      rc = check_launch("cudaStreamSynchronize");
  if (rc != WATTN_OK) return rc;
  return consume_status();
}

// After the device's work is complete: reports (and clears) a bounded wait
// that ran out, from the current device's status word.
int consume_status() {
  int *sp = device_status_ptr();
  int s[2] = {WATTN_OK, 0};
  if (sp && cudaMemcpy(s, sp, sizeof(s), cudaMemcpyDeviceToHost) == cudaSuccess &&
      s[0] != WATTN_OK) {
    const int zero[2] = {WATTN_OK, 0};
    cudaMemcpy(sp, zero, sizeof(zero), cudaMemcpyHostToDevice);
    reset_split_counters();
    return set_error(s[0], "a kernel's bounded wait ran out (site 0x%08x)", s[1]);
  }
  return WATTN_OK;
}

// Bytes that one utterance moves through a host-buffer attention call.
struct AttnSizes {
  size_t q, kv, o;
};

// Shape, type and scalar checks shared by the device and host entry points.
int validate_attention_shape(int in_dt, int out_dt, int batch, int t_q, int t_kv, int n_heads,
                             int d_head, float scale, int causal, int q_pos_offset) {
  if (d_head != kHeadDim)
    return set_error(WATTN_ERR_UNSUPPORTED, "head dimension %d is not supported (64 only)", d_head);
  if (!valid_dtype(in_dt) || !valid_dtype(out_dt))
    return set_error(WATTN_ERR_INVALID, "unknown dtype (%d, %d)", in_dt, out_dt);
  if (out_dt != WATTN_F32 && out_dt != in_dt)
    return set_error(WATTN_ERR_INVALID, "out_dtype must be F32 or the input type");
  if (batch < 0 || t_q < 0 || t_kv < 0 || n_heads <= 0)
    return set_error(WATTN_ERR_INVALID, "negative size or n_heads <= 0");
  if (batch > 65535 || n_heads > 65535)
    return set_error(WATTN_ERR_INVALID, "batch and n_heads must be <= 65535");
  if (!(scale > 0.f) || scale > 3.0e38f)
    return set_error(WATTN_ERR_INVALID, "scale must be finite and positive");
  if (causal && q_pos_offset < 0) return set_error(WATTN_ERR_INVALID, "q_pos_offset must be >= 0");
  return WATTN_OK;
}

int validate_attention(const void *q, const void *k, const void *v, const void *o, int in_dt,
                       int out_dt, int batch, int t_q, int t_kv, int n_heads, int d_head,
                       int64_t q_rs, int64_t kv_rs, int64_t o_rs, int64_t q_bs, int64_t kv_bs,
                       int64_t o_bs, float scale, int causal, int q_pos_offset) {
  int rc = validate_attention_shape(in_dt, out_dt, batch, t_q, t_kv, n_heads, d_head, scale,
                                    causal, q_pos_offset);
  if (rc != WATTN_OK) return rc;
  const int64_t w = (int64_t)n_heads * kHeadDim;
  if (q_rs < w || kv_rs < w || o_rs < w)
    return set_error(WATTN_ERR_INVALID, "row strides must be >= n_heads * 64");
  if (q_bs < 0 || kv_bs < 0 || o_bs < 0) return set_error(WATTN_ERR_INVALID, "negative batch stride");
  if (batch == 0 || t_q == 0) return WATTN_OK;
  if (!q || !o || (t_kv > 0 && (!k || !v))) return set_error(WATTN_ERR_INVALID, "NULL tensor");
  const int es_in = elem_size(in_dt), es_out = elem_size(out_dt);
  const int64_t unit = 16 / es_in;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || q_rs % unit || kv_rs % unit ||
      q_bs % unit || kv_bs % unit)
    return set_error(WATTN_ERR_INVALID,
                     "q/k/v must be 16-byte aligned with row and batch strides that are "
                     "multiples of 16 bytes");
  if (!aligned16(o) || (o_rs * es_out) % 16 || (o_bs * es_out) % 16)
    return set_error(WATTN_ERR_INVALID, "o must be 16-byte aligned with 16-byte multiple strides");
  return WATTN_OK;
}

int attention_device(const void *q, const void *k, const void *v, void *o, int in_dt, int out_dt,
                     int batch, int t_q, int t_kv, int n_heads, int64_t q_rs, int64_t kv_rs,
                     int64_t o_rs, int64_t q_bs, int64_t kv_bs, int64_t o_bs, float scale,
                     int causal, int q_pos_offset, cudaStream_t st, void *split_ws = nullptr,
                     size_t split_ws_bytes = 0) {
  if (batch == 0 || t_q == 0) return WATTN_OK;
  if (t_kv == 0) return launch_zero_rows(o, out_dt, batch, t_q, n_heads * kHeadDim, o_rs, o_bs, st);
  if (in_dt == WATTN_F32)
    return launch_attn_f32((const float *)q, (const float *)k, (const float *)v, (float *)o, batch,
                           t_q, t_kv, n_heads, q_rs, kv_rs, o_rs, q_bs, kv_bs, o_bs, scale,
                           causal, q_pos_offset, st, split_ws, split_ws_bytes);
  return launch_attn_tc(q, k, v, o, in_dt, out_dt, batch, t_q, t_kv, n_heads, q_rs, kv_rs, o_rs,
                        q_bs, kv_bs, o_bs, scale, causal, q_pos_offset, st, split_ws,
                        split_ws_bytes);
}

int validate_decode(const void *q, const void *k, const void *v, const void *o, int q_dt,
                    int kv_dt, int out_dt, int n_groups, int group_size, int t_kv, int n_heads,
                    int d_head, int64_t q_rs, int64_t kv_rs, int64_t kv_gs, int64_t o_rs,
                    float scale) {
  if (d_head != kHeadDim)
    return set_error(WATTN_ERR_UNSUPPORTED, "head dimension %d is not supported (64 only)", d_head);
  if (!valid_dtype(q_dt) || !valid_dtype(kv_dt) || !valid_dtype(out_dt))
    return set_error(WATTN_ERR_INVALID, "unknown dtype");
  if (n_groups < 0 || group_size <= 0 || t_kv < 0 || n_heads <= 0)
    return set_error(WATTN_ERR_INVALID, "invalid sizes");
  if (n_heads > 65535) return set_error(WATTN_ERR_INVALID, "n_heads must be <= 65535");
  if ((int64_t)n_groups * ((group_size + 7) / 8) > 65535)
    return set_error(WATTN_ERR_INVALID, "too many query row groups in one call (max 65535 x 8 rows)");
  if (!(scale > 0.f) || scale > 3.0e38f)
    return set_error(WATTN_ERR_INVALID, "scale must be finite and positive");
  const int64_t w = (int64_t)n_heads * kHeadDim;
  if (q_rs < w || kv_rs < w || o_rs < w) return set_error(WATTN_ERR_INVALID, "row strides must be >= n_heads * 64");
  if (kv_gs < 0) return set_error(WATTN_ERR_INVALID, "negative group stride");
  if (n_groups == 0) return WATTN_OK;
  if (!q || !o || (t_kv > 0 && (!k || !v))) return set_error(WATTN_ERR_INVALID, "NULL tensor");
  if (!elem_aligned(q, q_dt) || !elem_aligned(o, out_dt))
    return set_error(WATTN_ERR_INVALID, "q and o must be aligned to their element size");
  const int es = elem_size(kv_dt);
  if (!aligned16(k) || !aligned16(v) || (kv_rs * es) % 16 || (kv_gs * es) % 16)
    return set_error(WATTN_ERR_INVALID,
                     "k/v must be 16-byte aligned with row and group strides that are multiples "
                     "of 16 bytes");
  if (q_dt != WATTN_F32 && ((reinterpret_cast<uintptr_t>(q) & 3) || (q_rs & 1)))
    return set_error(WATTN_ERR_INVALID, "16-bit q must be 4-byte aligned with an even row stride");
  return WATTN_OK;
}

int decode_device(const void *q, const void *k, const void *v, void *o, int q_dt, int kv_dt,
                  int out_dt, int n_groups, int group_size, int t_kv, int n_heads, int64_t q_rs,
                  int64_t kv_rs, int64_t kv_gs, int64_t o_rs, float scale, void *ws,
                  size_t ws_bytes, cudaStream_t st, const CaptureSpec *cap = nullptr) {
  if (n_groups == 0) return WATTN_OK;
  if (t_kv == 0)
    return launch_zero_rows(o, out_dt, 1, n_groups * group_size, n_heads * kHeadDim, o_rs, 0, st);
  if (ws == nullptr) {
    const DecodePlan pl = plan_decode(n_groups, group_size, t_kv, n_heads, q_dt, kv_dt);
    ws = thread_workspace(pl.workspace_bytes, st);
    if (ws == nullptr) return set_error(WATTN_ERR_NOMEM, "decode workspace allocation failed");
    ws_bytes = std::max(pl.workspace_bytes, (size_t)1 << 20);
  }
  return launch_decode(q, k, v, o, q_dt, kv_dt, out_dt, n_groups, group_size, t_kv, n_heads, q_rs,
                       kv_rs, kv_gs, o_rs, scale, ws, ws_bytes, st, cap);
}

// (slot, head) pairs of an alignment-head capture (decoder.rs:796-828's
// `selected`) -> CaptureSpec. Each head may be captured once per call.
int parse_selection(CaptureSpec *cap, const int *sel_slot, const int *sel_head, int n_sel,
                    int n_selected, int n_heads) {
  if (n_sel < 0 || n_selected < 0)
    return set_error(WATTN_ERR_INVALID, "capture: negative count");
  if (n_sel > 0 && (!sel_slot || !sel_head))
    return set_error(WATTN_ERR_INVALID, "capture: NULL selection");
  if (n_sel > 0 && n_heads > 64)
    return set_error(WATTN_ERR_UNSUPPORTED, "capture: %d heads (at most 64)", n_heads);
  cap->n_selected = n_selected;
  for (int h = 0; h < 64; ++h) cap->slot_of_head[h] = -1;
  for (int i = 0; i < n_sel; ++i) {
    if (sel_head[i] < 0 || sel_head[i] >= n_heads)
      return set_error(WATTN_ERR_RANGE, "capture: head %d outside [0, %d)", sel_head[i], n_heads);
    if (sel_slot[i] < 0 || sel_slot[i] >= n_selected)
      return set_error(WATTN_ERR_RANGE, "capture: slot %d outside [0, %d)", sel_slot[i],
                       n_selected);
    if (cap->slot_of_head[sel_head[i]] >= 0)
      return set_error(WATTN_ERR_UNSUPPORTED, "capture: head %d selected twice", sel_head[i]);
    cap->slot_of_head[sel_head[i]] = sel_slot[i];
  }
  return WATTN_OK;
}

int build_capture(CaptureSpec *cap, const int *sel_slot, const int *sel_head, int n_sel,
                  int n_selected, int row_offset, float *out, int n_heads) {
  if (row_offset < 0) return set_error(WATTN_ERR_INVALID, "capture: negative row offset");
  if (n_sel > 0 && !out) return set_error(WATTN_ERR_INVALID, "capture: NULL buffer");
  if (reinterpret_cast<uintptr_t>(out) & 3)
    return set_error(WATTN_ERR_INVALID, "capture: buffer must be 4-byte aligned");
  cap->out = out;
  cap->row0 = row_offset;
  return parse_selection(cap, sel_slot, sel_head, n_sel, n_selected, n_heads);
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Host-buffer attention over contiguous [batch][t][w] buffers, in chunks of
// utterances alternating between two streams.
int attention_host(const void *q, const void *k, const void *v, void *o, int in_dt, int out_dt,
                   int batch, int t_q, int t_kv, int n_heads, float scale, int causal,
                   int q_pos_offset) {
  const int w = n_heads * kHeadDim;
  // Host pointers need no alignment: the device copies made below are aligned.
  int rc = validate_attention_shape(in_dt, out_dt, batch, t_q, t_kv, n_heads, kHeadDim, scale,
                                    causal, q_pos_offset);
  if (rc != WATTN_OK) return rc;
  if (batch == 0 || t_q == 0) return WATTN_OK;
  if (!q || !o || (t_kv > 0 && (!k || !v))) return set_error(WATTN_ERR_INVALID, "NULL buffer");
  HostCtx *h = host_ctx();
  if (!h) return WATTN_ERR_CUDA;
  const size_t es_in = elem_size(in_dt), es_out = elem_size(out_dt);
  const size_t qb = (size_t)t_q * w * es_in, kvb = (size_t)t_kv * w * es_in,
               ob = (size_t)t_q * w * es_out;
  const size_t per = round_up(qb, 256) + 2 * round_up(kvb, 256) + round_up(ob, 256);
  // ~32 MB of device staging per stream, at least one utterance: the call
  // returns with its output written, so the first chunk's upload and the
  // last chunk's kernel and download overlap nothing; smaller chunks shorten
  // that, and their kernels still hide behind the uploads (measured on B200
  // with config 3: 32 MB, two utterances, 248 ms per 32-layer step; 48 MB
  // 253; 64 MB 264; 16 MB 281).
  const int chunk = (int)std::max<size_t>(1, std::min<size_t>(batch, ((size_t)32 << 20) / per));
  for (int i = 0; i < 2; ++i)
    if ((rc = grow(&h->buf[i], &h->buf_bytes[i], per * chunk, false, h->st[i])) != WATTN_OK)
      return finish_host(h, rc);
  // Each stream's kernels keep their workspaces (key-tile split partials,
  // V's f16 copy for bf16 inputs, the split operands of f32 inputs) apart.
  {
    int dev = 0, n_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return finish_host(h, check_launch("attention_host: device query"));
    const size_t ws_need = in_dt == WATTN_F32
                               ? attn_f32_workspace_bytes(chunk, t_q, t_kv, n_heads, n_sm)
                               : attn_workspace_bytes(in_dt, chunk, t_kv, n_heads, n_sm);
    for (int i = 0; i < 2; ++i)
      if ((rc = grow(&h->ws[i], &h->ws_bytes[i], ws_need, true, h->st[i])) != WATTN_OK)
        return finish_host(h, rc);
  }
  for (int c0 = 0, ci = 0; c0 < batch; c0 += chunk, ++ci) {
    const int nb = std::min(chunk, batch - c0);
    cudaStream_t st = h->st[ci & 1];
    uint8_t *base = (uint8_t *)h->buf[ci & 1];
    uint8_t *dq = base, *dk = dq + round_up(qb, 256) * nb, *dv = dk + round_up(kvb, 256) * nb,
            *dout = dv + round_up(kvb, 256) * nb;
    // Packed per chunk: [nb][t][w] with utterance stride = its byte size rounded to 256.
    const int64_t qbs = round_up(qb, 256) / es_in, kvbs = round_up(kvb, 256) / es_in,
                  obs = round_up(ob, 256) / es_out;
    for (int b = 0; b < nb && rc == WATTN_OK; ++b) {
      rc = h2d(dq + round_up(qb, 256) * b, (const uint8_t *)q + (c0 + b) * qb, qb, st);
      if (rc == WATTN_OK) rc = h2d(dk + round_up(kvb, 256) * b, (const uint8_t *)k + (c0 + b) * kvb, kvb, st);
      if (rc == WATTN_OK) rc = h2d(dv + round_up(kvb, 256) * b, (const uint8_t *)v + (c0 + b) * kvb, kvb, st);
    }
    if (rc == WATTN_OK)
      rc = attention_device(dq, dk, dv, dout, in_dt, out_dt, nb, t_q, t_kv, n_heads, w, w, w, qbs,
                            kvbs, obs, scale, causal, q_pos_offset, st, h->ws[ci & 1],
                            h->ws_bytes[ci & 1]);
    for (int b = 0; b < nb && rc == WATTN_OK; ++b)
      rc = d2h((uint8_t *)o + (c0 + b) * ob, dout + round_up(ob, 256) * b, ob, st);
    if (rc != WATTN_OK) break;
  }
  return finish_host(h, rc);
}

// Host-buffer decode: q [n_groups*G][w], k/v [n_groups][t_kv][w], o like q.
int decode_host(const void *q, const void *k, const void *v, void *o, int q_dt, int kv_dt,
                int out_dt, int n_groups, int group_size, int t_kv, int n_heads, int64_t kv_rs,
                float scale) {
  const int w = n_heads * kHeadDim;
  if (!valid_dtype(q_dt) || !valid_dtype(kv_dt) || !valid_dtype(out_dt) || n_groups < 0 ||
      group_size <= 0 || t_kv < 0 || n_heads <= 0 || kv_rs < w || !(scale > 0.f))
    return set_error(WATTN_ERR_INVALID, "decode_host: invalid arguments");
  if (n_groups == 0) return WATTN_OK;
  if (!q || !o || (t_kv > 0 && (!k || !v))) return set_error(WATTN_ERR_INVALID, "decode_host: NULL tensor");
  HostCtx *h = host_ctx();
  if (!h) return WATTN_ERR_CUDA;
  const size_t es_q = elem_size(q_dt), es_kv = elem_size(kv_dt), es_o = elem_size(out_dt);
  const int64_t dkv_rs = round_up((size_t)w, 16 / es_kv);  // device row stride (16-byte multiple)
  const size_t qb = (size_t)group_size * w * es_q, ob = (size_t)group_size * w * es_o;
  const size_t kvb_host = (size_t)t_kv * kv_rs * es_kv;
  const size_t kvb_dev = round_up((size_t)t_kv * dkv_rs * es_kv, 256);
  const size_t per = round_up(qb, 256) + 2 * kvb_dev + round_up(ob, 256);
  const int chunk = (int)std::max<size_t>(1, std::min<size_t>(n_groups, ((size_t)64 << 20) / per));
  int rc = WATTN_OK;
  const DecodePlan pl = plan_decode(chunk, group_size, t_kv, n_heads, q_dt, kv_dt);
  for (int i = 0; i < 2 && rc == WATTN_OK; ++i) {
    rc = grow(&h->buf[i], &h->buf_bytes[i], per * chunk, false, h->st[i]);
    if (rc == WATTN_OK) rc = grow(&h->ws[i], &h->ws_bytes[i], pl.workspace_bytes, true, h->st[i]);
  }
  if (rc != WATTN_OK) return finish_host(h, rc);
  for (int c0 = 0, ci = 0; c0 < n_groups; c0 += chunk, ++ci) {
    const int ng = std::min(chunk, n_groups - c0);
    cudaStream_t st = h->st[ci & 1];
    uint8_t *base = (uint8_t *)h->buf[ci & 1];
    uint8_t *dq = base, *dk = dq + round_up(qb, 256) * chunk, *dv = dk + kvb_dev * chunk,
            *dout = dv + kvb_dev * chunk;
    rc = h2d(dq, (const uint8_t *)q + (size_t)c0 * qb, qb * ng, st);  // rows contiguous
    for (int g = 0; g < ng && rc == WATTN_OK; ++g) {
      const uint8_t *ks = (const uint8_t *)k + (size_t)(c0 + g) * kvb_host;
      const uint8_t *vs = (const uint8_t *)v + (size_t)(c0 + g) * kvb_host;
      if (dkv_rs == kv_rs) {
        rc = h2d(dk + kvb_dev * g, ks, kvb_host, st);
        if (rc == WATTN_OK) rc = h2d(dv + kvb_dev * g, vs, kvb_host, st);
      } else {
        if (cudaMemcpy2DAsync(dk + kvb_dev * g, dkv_rs * es_kv, ks, kv_rs * es_kv, w * es_kv, t_kv,
                              cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpy2DAsync(dv + kvb_dev * g, dkv_rs * es_kv, vs, kv_rs * es_kv, w * es_kv, t_kv,
                              cudaMemcpyHostToDevice, st) != cudaSuccess)
          rc = check_launch("cudaMemcpy2DAsync");
      }
    }
    if (rc == WATTN_OK)
      rc = decode_device(dq, dk, dv, dout, q_dt, kv_dt, out_dt, ng, group_size, t_kv, n_heads, w,
                         dkv_rs, (int64_t)(kvb_dev / es_kv), w, scale, h->ws[ci & 1],
                         h->ws_bytes[ci & 1], st);
    if (rc == WATTN_OK) rc = d2h((uint8_t *)o + (size_t)c0 * ob, dout, ob * ng, st);
    if (rc != WATTN_OK) break;
  }
  return finish_host(h, rc);
}

}  // namespace

int validate_decode_args(const void *q, const void *k, const void *v, const void *o, int q_dt,
                         int kv_dt, int out_dt, int n_groups, int group_size, int t_kv,
                         int n_heads, int d_head, int64_t q_rs, int64_t kv_rs, int64_t kv_gs,
                         int64_t o_rs, float scale) {
  return validate_decode(q, k, v, o, q_dt, kv_dt, out_dt, n_groups, group_size, t_kv, n_heads,
                         d_head, q_rs, kv_rs, kv_gs, o_rs, scale);
}

}  // namespace wattn

using namespace wattn;

extern "C" {

int wattn_version(void) { return 100; }

const char *wattn_status_string(int status) {
  switch (status) {
    case WATTN_OK: return "ok";
    case WATTN_ERR_INVALID: return "invalid argument";
    case WATTN_ERR_UNSUPPORTED: return "unsupported configuration";
    case WATTN_ERR_CUDA: return "CUDA error";
    case WATTN_ERR_TIMEOUT: return "bounded device wait ran out";
    case WATTN_ERR_NOMEM: return "out of memory";
    case WATTN_ERR_RANGE: return "out of range";
    default: return "unknown status";
  }
}

int wattn_last_error(char *buf, size_t len) {
  if (buf && len > 0) {
    strncpy(buf, t_err_msg, len - 1);
    buf[len - 1] = 0;
  }
  return t_err_status;
}

int wattn_device_status(int device, int *status) {
  clear_error();
  if (!status) return set_error(WATTN_ERR_INVALID, "status is NULL");
  int prev = 0;
  cudaGetDevice(&prev);
  if (device >= 0 && device != prev && cudaSetDevice(device) != cudaSuccess)
    return check_launch("cudaSetDevice");
  int rc = WATTN_OK;
  int *sp = device_status_ptr();
  if (!sp) rc = WATTN_ERR_CUDA;
  if (rc == WATTN_OK && cudaDeviceSynchronize() != cudaSuccess) rc = check_launch("cudaDeviceSynchronize");
  int s[2] = {WATTN_OK, 0};
  if (rc == WATTN_OK && cudaMemcpy(s, sp, sizeof(s), cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = check_launch("read status word");
  const int zero[2] = {WATTN_OK, 0};
  if (rc == WATTN_OK && cudaMemcpy(sp, zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess)
    rc = check_launch("clear status word");
  if (rc == WATTN_OK && s[0] != WATTN_OK) reset_split_counters();
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  *status = s[0];
  if (rc == WATTN_OK && s[0] != WATTN_OK)
    set_error(s[0], "bounded wait ran out at site 0x%08x", s[1]);
  return rc;
}

int wattn_attention_fwd(const void *q, const void *k, const void *v, void *o, int in_dtype,
                        int out_dtype, int batch, int t_q, int t_kv, int n_heads, int d_head,
                        int64_t q_row_stride, int64_t kv_row_stride, int64_t o_row_stride,
                        int64_t q_batch_stride, int64_t kv_batch_stride, int64_t o_batch_stride,
                        float scale, int causal, int q_pos_offset, void *stream) {
  clear_error();
  int rc = validate_attention(q, k, v, o, in_dtype, out_dtype, batch, t_q, t_kv, n_heads, d_head,
                              q_row_stride, kv_row_stride, o_row_stride, q_batch_stride,
                              kv_batch_stride, o_batch_stride, scale, causal, q_pos_offset);
  if (rc != WATTN_OK) return rc;
  return attention_device(q, k, v, o, in_dtype, out_dtype, batch, t_q, t_kv, n_heads, q_row_stride,
                          kv_row_stride, o_row_stride, q_batch_stride, kv_batch_stride,
                          o_batch_stride, scale, causal ? 1 : 0, causal ? q_pos_offset : 0,
                          (cudaStream_t)stream);
}

size_t wattn_decode_workspace_bytes(int n_groups, int group_size, int t_kv, int n_heads) {
  if (n_groups <= 0 || group_size <= 0 || t_kv <= 0 || n_heads <= 0) return 0;
  // The largest of the plans of the three kernel families (tensor-core,
  // CUDA-core over 16-bit K/V, CUDA-core over f32 K/V), so the size serves
  // every dtype combination.
  const DecodePlan a = plan_decode(n_groups, group_size, t_kv, n_heads, WATTN_F16, WATTN_F16);
  const DecodePlan b = plan_decode(n_groups, group_size, t_kv, n_heads, WATTN_F32, WATTN_F16);
  const DecodePlan c = plan_decode(n_groups, group_size, t_kv, n_heads, WATTN_F32, WATTN_F32);
  return std::max(a.workspace_bytes, std::max(b.workspace_bytes, c.workspace_bytes));
}

int wattn_decode_fwd(const void *q, const void *k, const void *v, void *o, int q_dtype,
                     int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                     int n_heads, int d_head, int64_t q_row_stride, int64_t kv_row_stride,
                     int64_t kv_group_stride, int64_t o_row_stride, float scale, void *workspace,
                     size_t workspace_bytes, void *stream) {
  clear_error();
  int rc = validate_decode(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                           n_heads, d_head, q_row_stride, kv_row_stride, kv_group_stride,
                           o_row_stride, scale);
  if (rc != WATTN_OK) return rc;
  return decode_device(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                       n_heads, q_row_stride, kv_row_stride, kv_group_stride, o_row_stride, scale,
                       workspace, workspace_bytes, (cudaStream_t)stream);
}

int wattn_attention_host(const void *q, const void *k, const void *v, void *o, int in_dtype,
                         int out_dtype, int batch, int t_q, int t_kv, int n_heads, float scale,
                         int causal) {
  clear_error();
  return attention_host(q, k, v, o, in_dtype, out_dtype, batch, t_q, t_kv, n_heads, scale,
                        causal ? 1 : 0, 0);
}

int wattn_decode_host(const void *q, const void *k, const void *v, void *o, int q_dtype,
                      int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                      int n_heads, float scale) {
  clear_error();
  return decode_host(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                     n_heads, (int64_t)n_heads * kHeadDim, scale);
}

// ---- reference-signature mirrors (f32 host slices) -------------------------

static int ref_shape(size_t n_heads, size_t d_model, int *d_head) {
  // attention.rs:79-84 asserts n_heads > 0 and d_model % n_heads == 0.
  if (n_heads == 0) return set_error(WATTN_ERR_INVALID, "n_heads must be non-zero");
  if (d_model % n_heads != 0)
    return set_error(WATTN_ERR_INVALID, "d_model (%zu) is not divisible by n_heads (%zu)", d_model,
                     n_heads);
  if (n_heads > 65535 || d_model > (1u << 24)) return set_error(WATTN_ERR_INVALID, "size too large");
  *d_head = (int)(d_model / n_heads);
  if (*d_head != kHeadDim)
    return set_error(WATTN_ERR_UNSUPPORTED, "head dimension %d is not supported (64 only)", *d_head);
  return WATTN_OK;
}

int wattn_flash_attention_2(const float *q, const float *k, const float *v, size_t t_q,
                            size_t t_kv, size_t n_heads, size_t d_model, int causal,
                            float *output) {
  clear_error();
  int d_head = 0;
  int rc = ref_shape(n_heads, d_model, &d_head);
  if (rc != WATTN_OK) return rc;
  if (t_q > (size_t)INT32_MAX || t_kv > (size_t)INT32_MAX) return set_error(WATTN_ERR_INVALID, "size too large");
  if (t_q == 0) return WATTN_OK;  // attention.rs:90-92
  if (!q || !output || (t_kv > 0 && (!k || !v))) return set_error(WATTN_ERR_INVALID, "NULL slice");
  if (t_kv == 0) {  // attention.rs:93-96
    memset(output, 0, sizeof(float) * t_q * d_model);
    return WATTN_OK;
  }
  if (t_q == 1 && !causal)  // attention.rs:102-104
    return decode_host(q, k, v, output, WATTN_F32, WATTN_F32, WATTN_F32, 1, 1, (int)t_kv,
                       (int)n_heads, (int64_t)d_model, 0.125f);
  const float scale = 1.0f / sqrtf((float)d_head);  // attention.rs:107
  return attention_host(q, k, v, output, WATTN_F32, WATTN_F32, 1, (int)t_q, (int)t_kv,
                        (int)n_heads, scale, causal ? 1 : 0, 0);
}

int wattn_multi_head_attention(const float *q, const float *k, const float *v, size_t t_q,
                               size_t t_kv, size_t n_heads, size_t d_model, int causal,
                               float *output) {
  return wattn_flash_attention_2(q, k, v, t_q, t_kv, n_heads, d_model, causal, output);
}

int wattn_single_token_mha_d64(const float *q, const float *k, const float *v, size_t t_kv,
                               size_t n_heads, size_t d_model, float *output) {
  clear_error();
  if (n_heads == 0 || n_heads * kHeadDim != d_model)
    return set_error(n_heads == 0 ? WATTN_ERR_INVALID : WATTN_ERR_UNSUPPORTED,
                     "single_token_mha_d64 needs d_model == n_heads * 64");
  if (t_kv > (size_t)INT32_MAX || n_heads > 65535) return set_error(WATTN_ERR_INVALID, "size too large");
  if (!q || !output) return set_error(WATTN_ERR_INVALID, "NULL slice");
  if (t_kv == 0) {
    // softmax of an empty row leaves the accumulators at zero (attention.rs:355-388)
    memset(output, 0, sizeof(float) * d_model);
    return WATTN_OK;
  }
  if (!k || !v) return set_error(WATTN_ERR_INVALID, "NULL slice");
  return decode_host(q, k, v, output, WATTN_F32, WATTN_F32, WATTN_F32, 1, 1, (int)t_kv,
                     (int)n_heads, (int64_t)d_model, 0.125f);
}

int wattn_multi_head_attention_with_cache(const float *q, const float *k, const float *v,
                                          size_t n_tokens, size_t total_tokens, size_t t_past,
                                          size_t n_heads, size_t d_model, float *output) {
  clear_error();
  int d_head = 0;
  int rc = ref_shape(n_heads, d_model, &d_head);
  if (rc != WATTN_OK) return rc;
  if (t_past + n_tokens > total_tokens)  // decoder.rs:848-849 (k.len() == total_tokens * d_model)
    return set_error(WATTN_ERR_INVALID, "t_past + n_tokens exceeds total_tokens");
  if (total_tokens > (size_t)INT32_MAX) return set_error(WATTN_ERR_INVALID, "size too large");
  if (n_tokens == 0) return WATTN_OK;
  if (!q || !k || !v || !output) return set_error(WATTN_ERR_INVALID, "NULL slice");
  if (n_tokens == 1)  // decoder.rs:852-854: single_token_mha_d64 over t_past + 1 keys
    return decode_host(q, k, v, output, WATTN_F32, WATTN_F32, WATTN_F32, 1, 1, (int)(t_past + 1),
                       (int)n_heads, (int64_t)d_model, 0.125f);
  const float scale = 1.0f / sqrtf((float)d_head);
  return attention_host(q, k, v, output, WATTN_F32, WATTN_F32, 1, (int)n_tokens,
                        (int)(t_past + n_tokens), (int)n_heads, scale, 1, (int)t_past);
}

int wattn_decode_fwd_capture(const void *q, const void *k, const void *v, void *o, int q_dtype,
                             int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                             int n_heads, int d_head, int64_t q_row_stride, int64_t kv_row_stride,
                             int64_t kv_group_stride, int64_t o_row_stride, float scale,
                             void *workspace, size_t workspace_bytes, const int *sel_slot,
                             const int *sel_head, int n_sel, int n_selected, int row_offset,
                             float *capture, void *stream) {
  clear_error();
  int rc = validate_decode(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                           n_heads, d_head, q_row_stride, kv_row_stride, kv_group_stride,
                           o_row_stride, scale);
  if (rc != WATTN_OK) return rc;
  CaptureSpec cap;
  if ((rc = build_capture(&cap, sel_slot, sel_head, n_sel, n_selected, row_offset, capture,
                          n_heads)) != WATTN_OK)
    return rc;
  return decode_device(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                       n_heads, q_row_stride, kv_row_stride, kv_group_stride, o_row_stride, scale,
                       workspace, workspace_bytes, (cudaStream_t)stream,
                       n_sel > 0 && t_kv > 0 ? &cap : nullptr);
}

int wattn_capture_cross_attention_heads(const float *q, const float *k, size_t n_tokens,
                                        size_t n_audio, size_t n_heads, size_t d_model,
                                        const int *sel_slot, const int *sel_head, size_t n_sel,
                                        size_t n_selected, size_t row_offset, float *out) {
  clear_error();
  int d_head = 0;
  int rc = ref_shape(n_heads, d_model, &d_head);
  if (rc != WATTN_OK) return rc;
  if (n_tokens > (size_t)INT32_MAX || n_audio > (size_t)INT32_MAX || n_sel > 64 ||
      n_selected > (size_t)INT32_MAX || row_offset > (size_t)INT32_MAX)
    return set_error(WATTN_ERR_INVALID, "size too large");
  CaptureSpec cap;
  if ((rc = parse_selection(&cap, sel_slot, sel_head, (int)n_sel, (int)n_selected,
                            (int)n_heads)) != WATTN_OK)
    return rc;
  if (n_tokens == 0 || n_sel == 0 || n_audio == 0) return WATTN_OK;
  if (!q || !k || !out) return set_error(WATTN_ERR_INVALID, "NULL slice");
  const size_t qb = n_tokens * d_model * 4, kb = n_audio * d_model * 4,
               cb = n_tokens * n_selected * n_audio * 4;
  float *host_rows = out + row_offset * n_selected * n_audio;
  uint8_t *buf = nullptr;
  if (cudaMalloc(&buf, 2 * qb + kb + cb) != cudaSuccess) {
    cudaGetLastError();
    return set_error(WATTN_ERR_NOMEM, "capture: device buffers of %zu bytes", 2 * qb + kb + cb);
  }
  float *dq = reinterpret_cast<float *>(buf), *dout = reinterpret_cast<float *>(buf + qb),
        *dk = reinterpret_cast<float *>(buf + 2 * qb),
        *dcap = reinterpret_cast<float *>(buf + 2 * qb + kb);
  // The device buffer holds rows row_offset .. row_offset + n_tokens of `out`.
  cap.out = dcap;
  cap.row0 = 0;
  // Slots not selected keep their contents: the rows go to the device and back.
  if (cudaMemcpy(dq, q, qb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dk, k, kb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dcap, host_rows, cb, cudaMemcpyHostToDevice) != cudaSuccess) {
    rc = check_launch("capture: host to device copy");
  } else {
    // The reference's multi_head_attention computes the attention output
    // beside the capture (decoder.rs:698-722); here V = K only keeps the
    // launch valid, the output is not returned.
    rc = decode_device(dq, dk, dk, dout, WATTN_F32, WATTN_F32, WATTN_F32, 1, (int)n_tokens,
                       (int)n_audio, (int)n_heads, (int64_t)d_model, (int64_t)d_model,
                       (int64_t)n_audio * d_model, (int64_t)d_model,
                       1.0f / sqrtf((float)d_head), nullptr, 0, 0, &cap);
    if (rc == WATTN_OK && cudaMemcpy(host_rows, dcap, cb, cudaMemcpyDeviceToHost) != cudaSuccess)
      rc = check_launch("capture: device to host copy");
    if (rc == WATTN_OK) rc = consume_status();
  }
  cudaFree(buf);
  return rc;
}

int validate_linear(const void *x, const void *w, const void *y, int in_dtype, int out_dtype,
                    int m, int n, int k, int64_t x_rs, int64_t w_rs, int64_t y_rs,
                    const float *bias) {
  if (in_dtype != WATTN_F16 && in_dtype != WATTN_BF16)
    return set_error(WATTN_ERR_UNSUPPORTED, "linear: inputs must be f16 or bf16");
  if (!valid_dtype(out_dtype)) return set_error(WATTN_ERR_INVALID, "linear: bad output dtype");
  if (m < 0 || n < 0 || k < 1) return set_error(WATTN_ERR_INVALID, "linear: bad sizes");
  if (x_rs < k || w_rs < k || y_rs < n)
    return set_error(WATTN_ERR_INVALID, "linear: row stride below the row length");
  if (m == 0 || n == 0) return WATTN_OK;
  if (!x || !w || !y) return set_error(WATTN_ERR_INVALID, "linear: NULL tensor");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) ||
      ((x_rs * 2) & 15) || ((w_rs * 2) & 15))
    return set_error(WATTN_ERR_INVALID,
                     "linear: x and W need 16-byte aligned rows (base and row stride)");
  if (!elem_aligned(y, out_dtype) || !elem_aligned(bias, WATTN_F32))
    return set_error(WATTN_ERR_INVALID, "linear: y and the bias must be aligned to their element size");
  return WATTN_OK;
}

int wattn_linear_fwd(const void *x, const void *w, const float *bias, void *y, int in_dtype,
                     int out_dtype, int m, int n, int k, int64_t x_row_stride,
                     int64_t w_row_stride, int64_t y_row_stride, void *stream) {
  clear_error();
  int rc = validate_linear(x, w, y, in_dtype, out_dtype, m, n, k, x_row_stride, w_row_stride,
                           y_row_stride, bias);
  if (rc != WATTN_OK || m == 0 || n == 0) return rc;
  return launch_linear(x, w, bias, y, in_dtype, out_dtype, m, n, k, x_row_stride, w_row_stride,
                       y_row_stride, (cudaStream_t)stream);
}

int wattn_cross_kv_project(const void *enc, const void *wk, const void *wv, const float *bv,
                           void *k_out, void *v_out, int in_dtype, int out_dtype, int n_tokens,
                           int d_model, int64_t enc_row_stride, int64_t kv_row_stride,
                           void *stream) {
  clear_error();
  int rc = validate_linear(enc, wk, k_out, in_dtype, out_dtype, n_tokens, d_model, d_model,
                           enc_row_stride, d_model, kv_row_stride, nullptr);
  if (rc == WATTN_OK)
    rc = validate_linear(enc, wv, v_out, in_dtype, out_dtype, n_tokens, d_model, d_model,
                         enc_row_stride, d_model, kv_row_stride, bv);
  if (rc != WATTN_OK || n_tokens == 0) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // decoder.rs:433-442: K without bias, V with the value bias.
  rc = launch_linear(enc, wk, nullptr, k_out, in_dtype, out_dtype, n_tokens, d_model, d_model,
                     enc_row_stride, d_model, kv_row_stride, st);
  if (rc != WATTN_OK) return rc;
  return launch_linear(enc, wv, bv, v_out, in_dtype, out_dtype, n_tokens, d_model, d_model,
                       enc_row_stride, d_model, kv_row_stride, st);
}

size_t wattn_encoder_attention_workspace_bytes(int batch, int t, int n_heads) {
  if (batch <= 0 || t <= 0 || n_heads <= 0) return 0;
  const size_t rows = (size_t)batch * t, d = (size_t)n_heads * kHeadDim;
  // fused QKV [rows][3d], the attention output [rows][d] and (for the
  // residual form) the normalised rows [rows][d], 16-bit each; then the
  // attention's own workspace (key-tile split partials sized for the
  // current device, V's f16 copy for bf16 weights)
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    n_sm = 148;
  }
  return round_up(rows * 3 * d * 2, 256) + 2 * round_up(rows * d * 2, 256) +
         round_up(attn_workspace_bytes(WATTN_BF16, batch, t, n_heads, n_sm), 256);
}

static int encoder_attention_impl(const void *x, const void *w_qkv, const float *b_qkv,
                                  const void *w_out, const float *b_out, void *y, int in_dtype,
                                  int out_dtype, int batch, int t, int n_heads, void *workspace,
                                  size_t workspace_bytes, void *stream, bool add_residual);

int wattn_encoder_attention(const void *x, const void *w_qkv, const float *b_qkv,
                            const void *w_out, const float *b_out, void *y, int in_dtype,
                            int out_dtype, int batch, int t, int n_heads, void *workspace,
                            size_t workspace_bytes, void *stream) {
  clear_error();
  return encoder_attention_impl(x, w_qkv, b_qkv, w_out, b_out, y, in_dtype, out_dtype, batch, t,
                                n_heads, workspace, workspace_bytes, stream, false);
}

static int encoder_attention_impl(const void *x, const void *w_qkv, const float *b_qkv,
                                  const void *w_out, const float *b_out, void *y, int in_dtype,
                                  int out_dtype, int batch, int t, int n_heads, void *workspace,
                                  size_t workspace_bytes, void *stream, bool add_residual) {
  if (batch < 0 || t < 0 || n_heads <= 0)
    return set_error(WATTN_ERR_INVALID, "encoder_attention: bad sizes");
  if (batch == 0 || t == 0) return WATTN_OK;
  const int d = n_heads * kHeadDim;
  const long long rows_ll = (long long)batch * t;
  if (rows_ll > INT32_MAX) return set_error(WATTN_ERR_INVALID, "encoder_attention: too many rows");
  const int rows = (int)rows_ll;
  // (the QKV projection writes the workspace, [rows][3d]; the attention
  // output, also in the workspace, feeds the output projection)
  int rc = validate_linear(x, w_qkv, y, in_dtype, in_dtype, rows, 3 * d, d, d, d, 3 * d, b_qkv);
  if (rc == WATTN_OK)
    rc = validate_linear(x, w_out, y, in_dtype, out_dtype, rows, d, d, d, d, d, b_out);
  if (rc != WATTN_OK) return rc;
  const size_t need = wattn_encoder_attention_workspace_bytes(batch, t, n_heads);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(WATTN_ERR_INVALID,
                     "encoder_attention: a 256-byte aligned workspace of %zu bytes is needed", need);
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t *qkv = reinterpret_cast<uint8_t *>(workspace);
  uint8_t *attn = qkv + round_up((size_t)rows * 3 * d * 2, 256);
  // encoder.rs:276-279: the fused projection, [rows][q | k | v]
  rc = launch_linear(x, w_qkv, b_qkv, qkv, in_dtype, in_dtype, rows, 3 * d, d, d, d, 3 * d, st);
  if (rc != WATTN_OK) return rc;
  // encoder.rs:281-299: attention reads q, k, v in place (row stride 3d),
  // without the split copy; scale 1/sqrt(64) as flash_attention_2 uses
  const int64_t qkv_bs = (int64_t)t * 3 * d;
  uint8_t *split = attn + 2 * round_up((size_t)rows * d * 2, 256);
  const size_t split_bytes = workspace_bytes - (size_t)(split - qkv);
  rc = attention_device(qkv, qkv + (size_t)d * 2, qkv + (size_t)2 * d * 2, attn, in_dtype,
                        in_dtype, batch, t, t, n_heads, 3 * d, 3 * d, d, qkv_bs, qkv_bs,
                        (int64_t)t * d, 0.125f, 0, 0, st, split, split_bytes);
  if (rc != WATTN_OK) return rc;
  // encoder.rs:301-304: output projection (plus the residual add when the
  // output is the f32 residual stream being updated in place)
  return launch_linear(attn, w_out, b_out, y, in_dtype, out_dtype, rows, d, d, d, d, d, st,
                       add_residual ? static_cast<const float *>(y) : nullptr);
}

int wattn_encoder_attention_residual(float *x, const float *ln_w, const float *ln_b,
                                     const void *w_qkv, const float *b_qkv, const void *w_out,
                                     const float *b_out, int dtype, int batch, int t, int n_heads,
                                     void *workspace, size_t workspace_bytes, void *stream) {
  clear_error();
  if (batch < 0 || t < 0 || n_heads <= 0)
    return set_error(WATTN_ERR_INVALID, "encoder_attention_residual: bad sizes");
  if (batch == 0 || t == 0) return WATTN_OK;
  if (!x || !ln_w || !ln_b) return set_error(WATTN_ERR_INVALID, "encoder_attention_residual: NULL");
  if (!elem_aligned(x, WATTN_F32) || !elem_aligned(ln_w, WATTN_F32) || !elem_aligned(ln_b, WATTN_F32))
    return set_error(WATTN_ERR_INVALID,
                     "encoder_attention_residual: x and the LayerNorm weights must be 4-byte aligned");
  const int d = n_heads * kHeadDim;
  const long long rows_ll = (long long)batch * t;
  if (rows_ll > INT32_MAX) return set_error(WATTN_ERR_INVALID, "too many rows");
  const int rows = (int)rows_ll;
  const size_t need = wattn_encoder_attention_workspace_bytes(batch, t, n_heads);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(WATTN_ERR_INVALID,
                     "encoder_attention_residual: a 256-byte aligned workspace of %zu bytes is needed",
                     need);
  uint8_t *xn = reinterpret_cast<uint8_t *>(workspace) + round_up((size_t)rows * 3 * d * 2, 256) +
                round_up((size_t)rows * d * 2, 256);
  int rc = validate_linear(xn, w_qkv, x, dtype, dtype, rows, 3 * d, d, d, d, 3 * d, b_qkv);
  if (rc == WATTN_OK)
    rc = validate_linear(xn, w_out, x, dtype, WATTN_F32, rows, d, d, d, d, d, b_out);
  if (rc != WATTN_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // encoder.rs:266-274: pre-LN (eps 1e-5) into the 16-bit GEMM input
  rc = launch_layer_norm(x, ln_w, ln_b, xn, dtype, rows, d, 1e-5f, st);
  if (rc != WATTN_OK) return rc;
  return encoder_attention_impl(xn, w_qkv, b_qkv, w_out, b_out, x, dtype, WATTN_F32, batch, t,
                                n_heads, workspace, workspace_bytes, stream, true);
}

int wattn_selftest_bounded_wait(int limit_us, void *stream) {
  clear_error();
  if (limit_us <= 0 || limit_us > 2000000)
    return set_error(WATTN_ERR_INVALID, "limit_us must be in (0, 2e6]");
  int *sp = device_status_ptr();
  if (!sp) return WATTN_ERR_CUDA;
  int *flag = nullptr;
  if (cudaMalloc(&flag, sizeof(int)) != cudaSuccess) return check_launch("cudaMalloc(flag)");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = WATTN_OK;
  if (cudaMemsetAsync(flag, 0, sizeof(int), st) != cudaSuccess) rc = check_launch("memset flag");
  if (rc == WATTN_OK) {
    bounded_wait_kernel<<<1, 1, 0, st>>>(flag, sp, (unsigned long long)limit_us * 1000ull);
    rc = check_launch("bounded_wait_kernel");
  }
  if (rc == WATTN_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = check_launch("sync");
  cudaFree(flag);
  if (rc != WATTN_OK) return rc;
  int s = WATTN_OK;
  rc = wattn_device_status(-1, &s);
  if (rc != WATTN_OK) return rc;
  if (s != WATTN_OK) return set_error(s, "bounded wait ran out after %d us (as designed)", limit_us);
  return WATTN_OK;
}

}  // extern "C"
