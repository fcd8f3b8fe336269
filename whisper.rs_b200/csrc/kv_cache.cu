// kv_cache.cu -- device-resident paged KV cache for decoder self-attention.
//
// Replaces DecoderKvCache (crates/whisper/src/decoder.rs:131-264): the
// reference keeps one growable host Vec<f32> per (layer, slot) and forks a
// beam by copying t_past * d_model floats per layer (copy_slot, :220-234).
// Here the rows live in a pool of device pages. A page holds page_rows
// consecutive positions of one slot for every layer, K and V, every head:
//   pool[page][layer][K|V][head][page_rows][64]
// so one (page, layer, K|V, head) block is page_rows * 128 contiguous bytes
// (16-bit cache) and a 64-row block is one TMA box.
//
// A slot is a host-side page list plus `start` (rows dropped from the front
// by slide_to_fit, :248-263), `t_past` and `stored` (rows holding data; rows
// past t_past survive a rewind until the next append overwrites them,
// :631-633). Forks share pages by reference count; a page still shared when
// a slot writes into it is copied first (copy on write), so a fork costs
// O(pages) host work and at most one page copy per written page.
//
// The attention itself is decode.cu's paged split-KV kernel; this file owns
// the host state, the append (scatter) kernel and a gather kernel for tests.

#include <algorithm>
#include <mutex>
#include <vector>

#include "wattn_common.cuh"
#include "wattn_internal.h"

namespace wattn {

namespace {

constexpr int kAppendMaxRows = 1024;

struct AppendTable {
  int n_rows;
  int layer, n_layers, n_heads, page_rows;
  int64_t row_stride;
  int page[kAppendMaxRows];
  int row_in_page[kAppendMaxRows];
};

// Eight consecutive elements through f32 (exact for every type pair the
// cache stores: a 16-bit value round-trips through f32 unchanged).
template <typename T>
WATTN_DEVINL void load8(const T *src, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4 *>(src)[0];
    const float4 b = reinterpret_cast<const float4 *>(src)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4 *>(src);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = unpack2<T>(u[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
}

template <typename T>
WATTN_DEVINL void store8(T *dst, const float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4 *>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4 *>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    *reinterpret_cast<uint4 *>(dst) = make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]),
                                                 pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
  }
}

// Scatter new K/V rows ([n_rows][n_heads*64], src type) into their pages.
// VEC: source rows 16-byte aligned, so each thread moves 8 elements with
// vector loads and stores (page rows always are: 64 elements per head).
template <typename SrcT, typename DstT, bool VEC>
__global__ void kv_append_kernel(const SrcT *k_rows, const SrcT *v_rows, DstT *pool,
                                 const __grid_constant__ AppendTable t) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  const int r = blockIdx.x;
  const int width = t.n_heads * 64;
  const int64_t page_elems = (int64_t)t.n_layers * 2 * t.n_heads * t.page_rows * 64;
  DstT *layer_base = pool + (int64_t)t.page[r] * page_elems +
                     (int64_t)t.layer * 2 * t.n_heads * t.page_rows * 64;
  const int64_t kv_off = (int64_t)t.n_heads * t.page_rows * 64;
  if constexpr (VEC) {
    for (int i = threadIdx.x * 8; i < width; i += blockDim.x * 8) {
      const int h = i >> 6, d = i & 63;
      const int64_t dst = ((int64_t)h * t.page_rows + t.row_in_page[r]) * 64 + d;
      float f[8];
      load8<SrcT>(k_rows + (int64_t)r * t.row_stride + i, f);
      store8<DstT>(layer_base + dst, f);
      load8<SrcT>(v_rows + (int64_t)r * t.row_stride + i, f);
      store8<DstT>(layer_base + kv_off + dst, f);
    }
  } else {
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
      const int h = i >> 6, d = i & 63;
      const int64_t dst = ((int64_t)h * t.page_rows + t.row_in_page[r]) * 64 + d;
      layer_base[dst] = from_f32<DstT>(to_f32(k_rows[(int64_t)r * t.row_stride + i]));
      layer_base[kv_off + dst] = from_f32<DstT>(to_f32(v_rows[(int64_t)r * t.row_stride + i]));
    }
  }
}

constexpr int kGatherMaxPages = 64;
struct GatherTable {
  int n_rows, start, layer, n_layers, n_heads, page_rows, which;
  int pages[kGatherMaxPages];
};

// Gather one slot's rows of one layer back to the flat [t][n_heads*64] layout.
template <typename SrcT, typename DstT>
__global__ void kv_gather_kernel(const SrcT *pool, DstT *out, const __grid_constant__ GatherTable t) {
  const int r = blockIdx.x;
  const int prow = t.start + r;
  const int page = t.pages[prow / t.page_rows], rip = prow % t.page_rows;
  const int64_t page_elems = (int64_t)t.n_layers * 2 * t.n_heads * t.page_rows * 64;
  const SrcT *base = pool + (int64_t)page * page_elems +
                     ((int64_t)t.layer * 2 + t.which) * t.n_heads * t.page_rows * 64;
  const int width = t.n_heads * 64;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int h = i >> 6, d = i & 63;
    out[(int64_t)r * width + i] = from_f32<DstT>(to_f32(base[((int64_t)h * t.page_rows + rip) * 64 + d]));
  }
}

template <typename SrcT, bool VEC>
void launch_append_vec(int dst_dt, const SrcT *ks, const SrcT *vs, void *pool,
                       const AppendTable &t, cudaStream_t st) {
  const dim3 grid(t.n_rows);
  const int threads = VEC ? 160 : 256;  // VEC: 160 x 8 = the 1280 elements of a large-v3 row
  if (dst_dt == WATTN_F32)
    launch_pdl(kv_append_kernel<SrcT, float, VEC>, grid, dim3(threads), 0, st, ks, vs, (float *)pool, t);
  else if (dst_dt == WATTN_F16)
    launch_pdl(kv_append_kernel<SrcT, __half, VEC>, grid, dim3(threads), 0, st, ks, vs, (__half *)pool, t);
  else
    launch_pdl(kv_append_kernel<SrcT, __nv_bfloat16, VEC>, grid, dim3(threads), 0, st, ks, vs,
               (__nv_bfloat16 *)pool, t);
}

template <typename SrcT>
int launch_append_src(int dst_dt, const void *k, const void *v, void *pool, const AppendTable &t,
                      cudaStream_t st) {
  const SrcT *ks = (const SrcT *)k, *vs = (const SrcT *)v;
  const bool vec = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0 &&
                   (t.row_stride * (int64_t)sizeof(SrcT)) % 16 == 0;
  if (vec) launch_append_vec<SrcT, true>(dst_dt, ks, vs, pool, t, st);
  else launch_append_vec<SrcT, false>(dst_dt, ks, vs, pool, t, st);
  return check_launch("kv_append");
}

template <typename SrcT>
int launch_gather_src(int dst_dt, const void *pool, void *out, const GatherTable &t,
                      cudaStream_t st) {
  dim3 grid(t.n_rows);
  const SrcT *ps = (const SrcT *)pool;
  if (dst_dt == WATTN_F32)
    kv_gather_kernel<SrcT, float><<<grid, 256, 0, st>>>(ps, (float *)out, t);
  else if (dst_dt == WATTN_F16)
    kv_gather_kernel<SrcT, __half><<<grid, 256, 0, st>>>(ps, (__half *)out, t);
  else
    kv_gather_kernel<SrcT, __nv_bfloat16><<<grid, 256, 0, st>>>(ps, (__nv_bfloat16 *)out, t);
  return check_launch("kv_gather");
}

}  // namespace
}  // namespace wattn

using namespace wattn;

struct wattn_kv_cache {
  struct Slot {
    std::vector<int> pages;
    int start = 0;   // rows dropped from the front of pages[0]
    int t_past = 0;  // tokens already attended (decoder.rs:141)
    int stored = 0;  // rows holding data (>= t_past after a rewind)
  };
  int device = 0;
  int n_layers = 0, n_heads = 0, max_ctx = 0, page_rows = 0, n_pages = 0, dtype = 0;
  int max_pages_per_slot = 0;
  size_t page_bytes = 0;
  uint8_t *pool = nullptr;
  CUtensorMap map;       // the pool as [rows][64], boxes of kDecSubRows rows
  CUtensorMap map_tail;  // the same, boxes of kDecTailRows rows
  std::vector<int> refcnt;
  std::vector<int> free_pages;
  std::vector<Slot> slots;
  void *ws = nullptr;
  size_t ws_bytes = 0;
  std::mutex mu;

  int alloc_page() {
    if (free_pages.empty()) return -1;
    const int p = free_pages.back();
    free_pages.pop_back();
    refcnt[p] = 1;
    return p;
  }
  void release_page(int p) {
    if (--refcnt[p] == 0) free_pages.push_back(p);
  }
  void release_slot(Slot &s) {
    for (int p : s.pages) release_page(p);
    s.pages.clear();
    s.start = s.t_past = s.stored = 0;
  }
  int check_slot(int slot) const {
    if (slot < 0 || slot >= (int)slots.size())
      return set_error(WATTN_ERR_RANGE, "slot %d out of range (%zu slots)", slot, slots.size());
    return WATTN_OK;
  }
};

namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

int wattn_kv_create(wattn_kv_cache **out, int n_layers, int n_slots, int n_heads, int d_head,
                    int max_ctx, int page_rows, int n_pages, int dtype) {
  clear_error();
  if (out == nullptr) return set_error(WATTN_ERR_INVALID, "kv_create: out is NULL");
  *out = nullptr;
  if (d_head != 64) return set_error(WATTN_ERR_UNSUPPORTED, "kv_create: head dim %d (64 only)", d_head);
  if (n_layers <= 0 || n_slots < 0 || n_heads <= 0 || max_ctx <= 0 || n_pages < 0 ||
      !valid_dtype(dtype))
    return set_error(WATTN_ERR_INVALID, "kv_create: invalid sizes or dtype");
  if (page_rows <= 0 || page_rows % kDecSubRows != 0)
    return set_error(WATTN_ERR_INVALID, "kv_create: page_rows %d must be a positive multiple of %d",
                     page_rows, kDecSubRows);
  const int mpps = (max_ctx + 2 * page_rows - 2) / page_rows;  // start offset < page_rows
  if (mpps > kPagedMaxPages)
    return set_error(WATTN_ERR_UNSUPPORTED,
                     "kv_create: max_ctx %d needs %d pages of %d rows per slot (max %d); use larger pages",
                     max_ctx, mpps, page_rows, kPagedMaxPages);
  if (n_pages == 0) n_pages = std::max(1, n_slots) * (mpps + 1);
  const int es = elem_size(dtype);
  const size_t page_bytes = (size_t)n_layers * 2 * n_heads * page_rows * 64 * es;
  const uint64_t total_rows = (uint64_t)n_pages * n_layers * 2 * n_heads * page_rows;
  if (total_rows >= (1ull << 31))
    return set_error(WATTN_ERR_UNSUPPORTED, "kv_create: pool of %llu rows exceeds 2^31",
                     (unsigned long long)total_rows);
  wattn_kv_cache *c = new (std::nothrow) wattn_kv_cache();
  if (c == nullptr) return set_error(WATTN_ERR_NOMEM, "kv_create: host allocation failed");
  cudaGetDevice(&c->device);
  c->n_layers = n_layers;
  c->n_heads = n_heads;
  c->max_ctx = max_ctx;
  c->page_rows = page_rows;
  c->n_pages = n_pages;
  c->dtype = dtype;
  c->max_pages_per_slot = mpps;
  c->page_bytes = page_bytes;
  if (cudaMalloc(&c->pool, page_bytes * n_pages) != cudaSuccess) {
    cudaGetLastError();
    delete c;
    return set_error(WATTN_ERR_NOMEM, "kv_create: cudaMalloc of %zu bytes failed",
                     page_bytes * n_pages);
  }
  const uint64_t dims[2] = {64, total_rows};
  const uint64_t strides[1] = {64ull * es};
  const uint32_t box[2] = {(uint32_t)(128 / es), (uint32_t)kDecSubRows};
  const uint32_t box_tail[2] = {(uint32_t)(128 / es), (uint32_t)kDecTailRows};
  int rc = encode_tmap(&c->map, tmap_dtype(dtype), 2, c->pool, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == WATTN_OK)
    rc = encode_tmap(&c->map_tail, tmap_dtype(dtype), 2, c->pool, dims, strides, box_tail,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != WATTN_OK) {
    cudaFree(c->pool);
    delete c;
    return rc;
  }
  c->refcnt.assign(n_pages, 0);
  c->free_pages.reserve(n_pages);
  for (int p = n_pages - 1; p >= 0; --p) c->free_pages.push_back(p);
  c->slots.resize(n_slots);
  *out = c;
  return WATTN_OK;
}

int wattn_kv_destroy(wattn_kv_cache *c) {
  clear_error();
  if (c == nullptr) return WATTN_OK;
  {
    DeviceGuard g(c->device);
    cudaFree(c->pool);
    if (c->ws) cudaFree(c->ws);
  }
  delete c;
  return WATTN_OK;
}

int wattn_kv_clear(wattn_kv_cache *c) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_clear: NULL cache");
  std::lock_guard<std::mutex> lk(c->mu);
  for (auto &s : c->slots) c->release_slot(s);
  return WATTN_OK;
}

int wattn_kv_clear_slot(wattn_kv_cache *c, int slot) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_clear_slot: NULL cache");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = c->check_slot(slot);
  if (rc) return rc;
  c->release_slot(c->slots[slot]);
  return WATTN_OK;
}

int wattn_kv_ensure_slots(wattn_kv_cache *c, int n_slots) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_ensure_slots: NULL cache");
  std::lock_guard<std::mutex> lk(c->mu);
  if (n_slots > (int)c->slots.size()) c->slots.resize(n_slots);
  return WATTN_OK;
}

namespace {
// copy_slot with the cache locked and both slots checked: dst shares src's
// pages (reference counts); copies happen at the next write.
void fork_slot(wattn_kv_cache *c, int dst, int src) {
  if (dst == src) return;
  auto &d = c->slots[dst];
  const auto &s = c->slots[src];
  // Keep the source's pages alive before the destination drops its own
  // (they may be the same pages).
  std::vector<int> pages;
  int start = 0;
  if (s.t_past > 0) {
    const int need = (s.start + s.t_past + c->page_rows - 1) / c->page_rows;
    pages.assign(s.pages.begin(), s.pages.begin() + need);
    for (int p : pages) ++c->refcnt[p];
    start = s.start;
  }
  const int t = s.t_past;
  c->release_slot(d);
  d.pages = std::move(pages);
  d.start = start;
  d.t_past = d.stored = t;
}
}  // namespace

int wattn_kv_copy_slot(wattn_kv_cache *c, int dst, int src, void *stream) {
  clear_error();
  (void)stream;  // a fork only shares pages; copies happen at the next write
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_copy_slot: NULL cache");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = c->check_slot(dst);
  if (rc) return rc;
  if ((rc = c->check_slot(src))) return rc;
  fork_slot(c, dst, src);
  return WATTN_OK;
}

int wattn_kv_assign_beams(wattn_kv_cache *c, const int *parent_slot, int n_branches,
                          int *out_slot) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_assign_beams: NULL cache");
  if (n_branches < 0 || (n_branches > 0 && (!parent_slot || !out_slot)))
    return set_error(WATTN_ERR_INVALID, "kv_assign_beams: NULL or negative argument");
  std::lock_guard<std::mutex> lk(c->mu);
  const int n_slots = (int)c->slots.size();
  // Every retained branch's parent slot is reserved up front, so a sibling's
  // extra child cannot take the slot its owner is about to claim.
  std::vector<char> reserved(n_slots, 0), claimed(n_slots, 0);
  for (int i = 0; i < n_branches; ++i) {
    int rc = c->check_slot(parent_slot[i]);
    if (rc) return rc;
    reserved[parent_slot[i]] = 1;
  }
  // The first child of a parent keeps its slot; each further child forks
  // the parent into the next free slot. Planned first, so an exhausted
  // arena changes nothing.
  std::vector<int> plan(n_branches);
  int free_cursor = 0;
  for (int i = 0; i < n_branches; ++i) {
    const int parent = parent_slot[i];
    if (!claimed[parent]) {
      claimed[parent] = 1;
      plan[i] = parent;
      continue;
    }
    int ns = free_cursor;
    while (ns < n_slots && (reserved[ns] || claimed[ns])) ++ns;
    if (ns >= n_slots)
      return set_error(WATTN_ERR_RANGE, "kv_assign_beams: beam slot arena exhausted (%d slots)",
                       n_slots);
    claimed[ns] = 1;
    plan[i] = ns;
    free_cursor = ns;
  }
  for (int i = 0; i < n_branches; ++i) {
    if (plan[i] != parent_slot[i]) fork_slot(c, plan[i], parent_slot[i]);
    out_slot[i] = plan[i];
  }
  return WATTN_OK;
}

int wattn_kv_slot_len(const wattn_kv_cache *c, int slot, int *len) {
  clear_error();
  if (!c || !len) return set_error(WATTN_ERR_INVALID, "kv_slot_len: NULL argument");
  if (slot < 0 || slot >= (int)c->slots.size())
    return set_error(WATTN_ERR_RANGE, "slot %d out of range", slot);
  *len = c->slots[slot].t_past;
  return WATTN_OK;
}

int wattn_kv_slide_to_fit(wattn_kv_cache *c, int slot, int n_new, int max_ctx, int *pos) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_slide_to_fit: NULL cache");
  if (n_new < 0 || max_ctx < 0) return set_error(WATTN_ERR_INVALID, "kv_slide_to_fit: negative size");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = c->check_slot(slot);
  if (rc) return rc;
  auto &s = c->slots[slot];
  if (s.t_past + n_new > max_ctx) {
    const int drop = std::min(s.t_past + n_new - max_ctx, s.t_past);
    s.start += drop;
    s.t_past -= drop;
    s.stored = std::max(0, s.stored - drop);
    while (s.start >= c->page_rows && !s.pages.empty()) {
      c->release_page(s.pages.front());
      s.pages.erase(s.pages.begin());
      s.start -= c->page_rows;
    }
    if (s.pages.empty()) s.start = 0;
  }
  if (pos) *pos = s.t_past;
  return WATTN_OK;
}

int wattn_kv_set_t_past(wattn_kv_cache *c, int slot, int n_past) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_set_t_past: NULL cache");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = c->check_slot(slot);
  if (rc) return rc;
  auto &s = c->slots[slot];
  if (n_past < 0 || n_past > s.stored)
    return set_error(WATTN_ERR_RANGE, "kv_set_t_past: n_past %d outside [0, %d]", n_past, s.stored);
  s.t_past = n_past;
  return WATTN_OK;
}

int wattn_kv_advance(wattn_kv_cache *c, const int *slots, const int *n_tokens, int n_seqs) {
  clear_error();
  if (!c || (n_seqs > 0 && (!slots || !n_tokens)))
    return set_error(WATTN_ERR_INVALID, "kv_advance: NULL argument");
  std::lock_guard<std::mutex> lk(c->mu);
  for (int i = 0; i < n_seqs; ++i) {
    int rc = c->check_slot(slots[i]);
    if (rc) return rc;
    const auto &s = c->slots[slots[i]];
    if (n_tokens[i] < 0 || s.t_past + n_tokens[i] > s.stored)
      return set_error(WATTN_ERR_RANGE, "kv_advance: slot %d has %d rows, cannot advance %d past %d",
                       slots[i], s.stored, n_tokens[i], s.t_past);
  }
  for (int i = 0; i < n_seqs; ++i) c->slots[slots[i]].t_past += n_tokens[i];
  return WATTN_OK;
}

int wattn_kv_append(wattn_kv_cache *c, int layer, const int *slots, const int *n_tokens,
                    int n_seqs, const void *k_rows, const void *v_rows, int src_dtype,
                    int64_t row_stride, void *stream) {
  clear_error();
  if (!c || (n_seqs > 0 && (!slots || !n_tokens)))
    return set_error(WATTN_ERR_INVALID, "kv_append: NULL argument");
  if (layer < 0 || layer >= c->n_layers)
    return set_error(WATTN_ERR_RANGE, "kv_append: layer %d out of range", layer);
  if (!valid_dtype(src_dtype)) return set_error(WATTN_ERR_INVALID, "kv_append: bad dtype");
  if (row_stride < (int64_t)c->n_heads * 64)
    return set_error(WATTN_ERR_INVALID, "kv_append: row_stride %lld < width", (long long)row_stride);
  cudaStream_t st = (cudaStream_t)stream;
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  int total = 0;
  for (int i = 0; i < n_seqs; ++i) {
    int rc = c->check_slot(slots[i]);
    if (rc) return rc;
    if (n_tokens[i] < 0) return set_error(WATTN_ERR_INVALID, "kv_append: negative n_tokens");
    for (int j = 0; j < i; ++j)
      if (slots[j] == slots[i] && n_tokens[i] > 0 && n_tokens[j] > 0)
        return set_error(WATTN_ERR_INVALID, "kv_append: slot %d listed twice", slots[i]);
    const auto &s = c->slots[slots[i]];
    if ((int64_t)s.start + s.t_past + n_tokens[i] > (int64_t)c->max_pages_per_slot * c->page_rows)
      return set_error(WATTN_ERR_RANGE, "kv_append: slot %d would hold %d rows (capacity %d); "
                       "slide_to_fit first", slots[i], s.t_past + n_tokens[i], c->max_ctx);
    total += n_tokens[i];
  }
  if (total == 0) return WATTN_OK;
  if (k_rows == nullptr || v_rows == nullptr)
    return set_error(WATTN_ERR_INVALID, "kv_append: NULL rows");
  if (!elem_aligned(k_rows, src_dtype) || !elem_aligned(v_rows, src_dtype))
    return set_error(WATTN_ERR_INVALID, "kv_append: rows must be aligned to their element size");

  AppendTable t;
  t.layer = layer;
  t.n_layers = c->n_layers;
  t.n_heads = c->n_heads;
  t.page_rows = c->page_rows;
  t.row_stride = row_stride;
  t.n_rows = 0;
  const int es_src = elem_size(src_dtype);
  int row_base = 0;  // first source row of the current launch
  auto flush = [&]() -> int {
    if (t.n_rows == 0) return WATTN_OK;
    const uint8_t *k = (const uint8_t *)k_rows + (int64_t)row_base * row_stride * es_src;
    const uint8_t *v = (const uint8_t *)v_rows + (int64_t)row_base * row_stride * es_src;
    int rc;
    if (src_dtype == WATTN_F32) rc = launch_append_src<float>(c->dtype, k, v, c->pool, t, st);
    else if (src_dtype == WATTN_F16) rc = launch_append_src<__half>(c->dtype, k, v, c->pool, t, st);
    else rc = launch_append_src<__nv_bfloat16>(c->dtype, k, v, c->pool, t, st);
    row_base += t.n_rows;
    t.n_rows = 0;
    return rc;
  };
  for (int i = 0; i < n_seqs; ++i) {
    auto &s = c->slots[slots[i]];
    const int n = n_tokens[i];
    if (n == 0) continue;
    const int first = s.start + s.t_past, last = first + n - 1;  // physical rows written
    // Grow the page list, then give this slot private copies of shared pages
    // it is about to write.
    while ((int)s.pages.size() <= last / c->page_rows) {
      const int p = c->alloc_page();
      if (p < 0) return set_error(WATTN_ERR_NOMEM, "kv_append: page pool exhausted (%d pages)", c->n_pages);
      s.pages.push_back(p);
    }
    for (int pi = first / c->page_rows; pi <= last / c->page_rows; ++pi) {
      const int p = s.pages[pi];
      if (c->refcnt[p] > 1) {
        const int np = c->alloc_page();
        if (np < 0) return set_error(WATTN_ERR_NOMEM, "kv_append: page pool exhausted (%d pages)", c->n_pages);
        if (cudaMemcpyAsync(c->pool + (size_t)np * c->page_bytes, c->pool + (size_t)p * c->page_bytes,
                            c->page_bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
          return check_launch("kv_append copy-on-write");
        c->release_page(p);
        s.pages[pi] = np;
      }
    }
    for (int j = 0; j < n; ++j) {
      const int prow = first + j;
      t.page[t.n_rows] = s.pages[prow / c->page_rows];
      t.row_in_page[t.n_rows] = prow % c->page_rows;
      if (++t.n_rows == kAppendMaxRows) {
        int rc = flush();
        if (rc) return rc;
      }
    }
    s.stored = s.t_past + n;
  }
  return flush();
}

size_t wattn_kv_workspace_bytes(const wattn_kv_cache *c, int n_rows) {
  if (!c || n_rows <= 0) return 0;
  const int rows = std::min(n_rows, kPagedMaxRows);
  return paged_workspace_bytes(rows, c->n_heads, c->max_pages_per_slot * c->page_rows);
}

int wattn_kv_attend(wattn_kv_cache *c, int layer, const int *slots, const int *n_tokens,
                    int n_seqs, const void *q, int q_dtype, int64_t q_row_stride, void *o,
                    int out_dtype, int64_t o_row_stride, float scale, void *workspace,
                    size_t workspace_bytes, void *stream) {
  clear_error();
  if (!c || (n_seqs > 0 && (!slots || !n_tokens)))
    return set_error(WATTN_ERR_INVALID, "kv_attend: NULL argument");
  if (layer < 0 || layer >= c->n_layers)
    return set_error(WATTN_ERR_RANGE, "kv_attend: layer %d out of range", layer);
  if (!valid_dtype(q_dtype) || !valid_dtype(out_dtype))
    return set_error(WATTN_ERR_INVALID, "kv_attend: bad dtype");
  const int width = c->n_heads * 64;
  if (q_row_stride < width || o_row_stride < width)
    return set_error(WATTN_ERR_INVALID, "kv_attend: row stride below width");
  cudaStream_t st = (cudaStream_t)stream;
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  int total = 0;
  for (int i = 0; i < n_seqs; ++i) {
    int rc = c->check_slot(slots[i]);
    if (rc) return rc;
    const auto &s = c->slots[slots[i]];
    if (n_tokens[i] < 0) return set_error(WATTN_ERR_INVALID, "kv_attend: negative n_tokens");
    if (s.t_past + n_tokens[i] > s.stored)
      return set_error(WATTN_ERR_RANGE, "kv_attend: slot %d holds %d rows, needs %d (append first)",
                       slots[i], s.stored, s.t_past + n_tokens[i]);
    total += n_tokens[i];
  }
  if (total == 0) return WATTN_OK;
  if (!q || !o) return set_error(WATTN_ERR_INVALID, "kv_attend: NULL q/o");
  if (!elem_aligned(q, q_dtype) || !elem_aligned(o, out_dtype))
    return set_error(WATTN_ERR_INVALID, "kv_attend: q and o must be aligned to their element size");
  if (q_dtype != WATTN_F32 && ((reinterpret_cast<uintptr_t>(q) & 3) || (q_row_stride & 1)))
    return set_error(WATTN_ERR_INVALID, "kv_attend: 16-bit q must be 4-byte aligned with an even row stride");

  // Default workspace: owned by the cache, zeroed once, grown on demand.
  const size_t need = wattn_kv_workspace_bytes(c, total);
  if (workspace == nullptr) {
    if (c->ws_bytes < need) {
      if (c->ws) {
        cudaStreamSynchronize(st);
        cudaFree(c->ws);
      }
      c->ws = nullptr;
      c->ws_bytes = 0;
      if (cudaMalloc(&c->ws, need) != cudaSuccess) {
        cudaGetLastError();
        return set_error(WATTN_ERR_NOMEM, "kv_attend: workspace cudaMalloc(%zu) failed", need);
      }
      if (cudaMemsetAsync(c->ws, 0, need, st) != cudaSuccess) return check_launch("kv_attend memset");
      c->ws_bytes = need;
    }
    workspace = c->ws;
    workspace_bytes = c->ws_bytes;
  } else if (workspace_bytes < need) {
    return set_error(WATTN_ERR_INVALID, "kv_attend: workspace of %zu bytes, %zu needed",
                     workspace_bytes, need);
  }

  static thread_local PagedTable pt, sorted;  // ~29 KB each: keep them off the stack
  pt.layer = layer;
  pt.n_layers = c->n_layers;
  pt.page_rows = c->page_rows;
  pt.n_rows = 0;
  int row_base = 0, max_keys = 0;
  const int es_q = elem_size(q_dtype), es_o = elem_size(out_dtype);
  auto flush = [&]() -> int {
    if (pt.n_rows == 0) return WATTN_OK;
    const uint8_t *qp = (const uint8_t *)q + (int64_t)row_base * q_row_stride * es_q;
    uint8_t *op = (uint8_t *)o + (int64_t)row_base * o_row_stride * es_o;
    // Entries by descending key count (stable), each keeping its own row.
    int idx[kPagedMaxRows];
    for (int r = 0; r < pt.n_rows; ++r) idx[r] = r;
    std::stable_sort(idx, idx + pt.n_rows, [&](int a, int b) {
      return pt.kv_hi[a] - pt.kv_lo[a] > pt.kv_hi[b] - pt.kv_lo[b];
    });
    sorted.n_rows = pt.n_rows;
    sorted.layer = pt.layer;
    sorted.n_layers = pt.n_layers;
    sorted.page_rows = pt.page_rows;
    for (int e = 0; e < pt.n_rows; ++e) {
      const int r = idx[e];
      sorted.row_of[e] = r;
      sorted.kv_lo[e] = pt.kv_lo[r];
      sorted.kv_hi[e] = pt.kv_hi[r];
      for (int pi = 0; pi < kPagedMaxPages; ++pi) sorted.pages[e][pi] = pt.pages[r][pi];
    }
    int rc = launch_decode_paged(c->map, c->map_tail, qp, op, q_dtype, c->dtype, out_dtype, c->n_heads,
                                 q_row_stride, o_row_stride, scale, sorted, max_keys, workspace,
                                 workspace_bytes, st);
    row_base += pt.n_rows;
    pt.n_rows = 0;
    max_keys = 0;
    return rc;
  };
  for (int i = 0; i < n_seqs; ++i) {
    const auto &s = c->slots[slots[i]];
    for (int j = 0; j < n_tokens[i]; ++j) {
      const int r = pt.n_rows;
      pt.kv_lo[r] = s.start;
      pt.kv_hi[r] = s.start + s.t_past + j + 1;  // causal: positions 0 .. t_past + j
      for (int pi = 0; pi < kPagedMaxPages; ++pi)
        pt.pages[r][pi] = pi < (int)s.pages.size() ? s.pages[pi] : 0;
      max_keys = std::max(max_keys, pt.kv_hi[r] - (s.start & ~(kDecSubRows - 1)));
      if (++pt.n_rows == kPagedMaxRows) {
        int rc = flush();
        if (rc) return rc;
      }
    }
  }
  return flush();
}

int wattn_kv_read_slot(wattn_kv_cache *c, int layer, int slot, int which, void *out,
                       int out_dtype, void *stream) {
  clear_error();
  if (!c || !out) return set_error(WATTN_ERR_INVALID, "kv_read_slot: NULL argument");
  if (layer < 0 || layer >= c->n_layers) return set_error(WATTN_ERR_RANGE, "kv_read_slot: bad layer");
  if (which != 0 && which != 1) return set_error(WATTN_ERR_INVALID, "kv_read_slot: which must be 0 or 1");
  if (!valid_dtype(out_dtype)) return set_error(WATTN_ERR_INVALID, "kv_read_slot: bad dtype");
  if (!elem_aligned(out, out_dtype))
    return set_error(WATTN_ERR_INVALID, "kv_read_slot: out must be aligned to its element size");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = c->check_slot(slot);
  if (rc) return rc;
  const auto &s = c->slots[slot];
  if (s.t_past == 0) return WATTN_OK;
  if ((int)s.pages.size() > kGatherMaxPages)
    return set_error(WATTN_ERR_UNSUPPORTED, "kv_read_slot: too many pages");
  DeviceGuard g(c->device);
  GatherTable t;
  t.n_rows = s.t_past;
  t.start = s.start;
  t.layer = layer;
  t.n_layers = c->n_layers;
  t.n_heads = c->n_heads;
  t.page_rows = c->page_rows;
  t.which = which;
  for (int i = 0; i < kGatherMaxPages; ++i) t.pages[i] = i < (int)s.pages.size() ? s.pages[i] : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (c->dtype == WATTN_F32) return launch_gather_src<float>(out_dtype, c->pool, out, t, st);
  if (c->dtype == WATTN_F16) return launch_gather_src<__half>(out_dtype, c->pool, out, t, st);
  return launch_gather_src<__nv_bfloat16>(out_dtype, c->pool, out, t, st);
}

int wattn_kv_stats(const wattn_kv_cache *c, int *pages_used, int *pages_total) {
  clear_error();
  if (!c) return set_error(WATTN_ERR_INVALID, "kv_stats: NULL cache");
  if (pages_used) *pages_used = c->n_pages - (int)c->free_pages.size();
  if (pages_total) *pages_total = c->n_pages;
  return WATTN_OK;
}

}  // extern "C"
