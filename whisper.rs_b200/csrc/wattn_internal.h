// wattn_internal.h -- host-side declarations shared by the library's .cu files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "../../include/wattn.h"

namespace wattn {

// Launches a kernel with programmatic stream serialisation: its CTAs may be
// scheduled while the previous kernel in the stream finishes, and they wait
// for it in grid_dep_wait() before touching global memory (every kernel
// launched this way calls it first). Copies and memsets in the stream keep
// their full ordering.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// As launch_pdl, with the grid in clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, unsigned cluster_x, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Records `msg` (printf-style) as the calling thread's last error and
// returns `status`.
int set_error(int status, const char *fmt, ...);
void clear_error();

// Status word of the current device (device address), for kernel params.
int *device_status_ptr();

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry
// point (no link-time dependency on libcuda).
int encode_tmap(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t rank, const void *base,
                const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                CUtensorMapSwizzle swizzle);

inline int elem_size(int dt) { return dt == WATTN_F32 ? 4 : 2; }
// Whether p suits element-by-element access in dtype dt (aligned to the
// element size; NULL passes). Every pointer a kernel reads or writes one
// element at a time is checked with it on the host, so a misaligned caller
// pointer is an argument error rather than a device fault.
inline bool elem_aligned(const void *p, int dt) {
  return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(elem_size(dt) - 1)) == 0;
}
inline bool valid_dtype(int dt) { return dt == WATTN_F32 || dt == WATTN_F16 || dt == WATTN_BF16; }
inline CUtensorMapDataType tmap_dtype(int dt) {
  return dt == WATTN_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : dt == WATTN_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Checks the last CUDA error after a launch; returns WATTN_OK or WATTN_ERR_CUDA.
int check_launch(const char *what);

// Argument rules of wattn_decode_fwd (sizes, dtypes, strides, alignment);
// records the message and returns the status of the first rule broken.
int validate_decode_args(const void *q, const void *k, const void *v, const void *o, int q_dt,
                         int kv_dt, int out_dt, int n_groups, int group_size, int t_kv,
                         int n_heads, int d_head, int64_t q_rs, int64_t kv_rs, int64_t kv_gs,
                         int64_t o_rs, float scale);

// ----------------------------------------------------------- kernel launchers
// All pointers device, strides in elements; arguments already validated.

// Split workspaces (decode and attention) share one layout:
// [counters, kCounterBytes][partials]. The counter region has a fixed size,
// so partials written by one call never land where a later call of another
// shape keeps its counters; every launch leaves the counters it used at zero.
constexpr int kMaxSplitCounters = 65536;
constexpr size_t kCounterBytes = (size_t)kMaxSplitCounters * sizeof(int);

inline size_t round_up_256(size_t x) { return (x + 255) & ~(size_t)255; }

// tcgen05 tensor-core attention, 16-bit inputs (attn_tc.cu). Its workspace
// (split_ws: a caller's 256-byte aligned buffer of split_ws_bytes, or, with
// split_ws NULL, the calling thread's) holds the key-tile split schedule's
// counters and partials (this call zeroes the counters it uses in a
// caller's buffer; without room for the partials whole units are dealt
// round-robin) and, for bf16 inputs, V's f16 copy with its block maxima,
// for which a caller's buffer must have attn_workspace_bytes() bytes.
int launch_attn_tc(const void *q, const void *k, const void *v, void *o, int in_dtype,
                   int out_dtype, int batch, int t_q, int t_kv, int n_heads, int64_t q_rs,
                   int64_t kv_rs, int64_t o_rs, int64_t q_bs, int64_t kv_bs, int64_t o_bs,
                   float scale, int causal, int q_pos_offset, cudaStream_t stream,
                   void *split_ws = nullptr, size_t split_ws_bytes = 0);
// Key tiles per CTA of the split schedule for n_units units of nkv key tiles
// each on n_sm CTAs, or 0 when whole units dealt round-robin finish sooner.
int plan_attn_split(long long n_units, int nkv, int n_sm, int causal);
// Workspace of the split schedule on a device of n_sm SMs (its upper bound).
size_t attn_split_workspace_bytes(int n_sm);
// Whole workspace of one launch_attn_tc call on a device of n_sm SMs.
size_t attn_workspace_bytes(int in_dtype, int batch, int t_kv, int n_heads, int n_sm);

// f32 attention on the tensor cores, 3xTF32 (attn_f32.cu). Its workspace
// (ws: a caller's 256-byte aligned buffer of ws_bytes, which must then have
// attn_f32_workspace_bytes() bytes, or, with ws NULL, the calling thread's)
// holds the split K and V^T operands, the key-split partials and counters.
int launch_attn_f32(const float *q, const float *k, const float *v, float *o, int batch,
                    int t_q, int t_kv, int n_heads, int64_t q_rs, int64_t kv_rs, int64_t o_rs,
                    int64_t q_bs, int64_t kv_bs, int64_t o_bs, float scale, int causal,
                    int q_pos_offset, cudaStream_t stream, void *ws = nullptr,
                    size_t ws_bytes = 0);
// Workspace of one launch_attn_f32 call on a device of n_sm SMs (causal or not).
size_t attn_f32_workspace_bytes(int batch, int t_q, int t_kv, int n_heads, int n_sm);

// y[m][n] = x[m][k] W[n][k]^T (+ bias[n]) on the tensor cores (linear_tc.cu);
// x and W 16-bit of the same type, 16-byte aligned, row strides whose byte
// size is a multiple of 16.
// residual (f32, row stride y_rs, may be y itself) is added when non-null.
int launch_linear(const void *x, const void *w, const float *bias, void *y, int in_dtype,
                  int out_dtype, int m, int n, int k, int64_t x_rs, int64_t w_rs, int64_t y_rs,
                  cudaStream_t stream, const float *residual = nullptr);
// LayerNorm of f32 rows [rows][d] into 16-bit rows (linear_tc.cu).
int launch_layer_norm(const float *x, const float *gamma, const float *beta, void *y, int out_dtype,
                      int rows, int d, float eps, cudaStream_t stream);

// Zero-fills a strided [batch][t][n_heads*64] output (t_kv == 0 case).
int launch_zero_rows(void *o, int out_dtype, int batch, int t, int width, int64_t o_rs,
                     int64_t o_bs, cudaStream_t stream);

// Split-KV decode over dense K/V (decode.cu). Counters of one launch are
// indexed (row group, head) and must fit the fixed counter region.
struct DecodePlan {
  int chunk;      // keys per split (multiple of 64)
  int n_splits;   // splits per (row chunk, head)
  int row_chunks; // ceil(group_size / rows per CTA)
  size_t workspace_bytes;
};
DecodePlan plan_decode(int n_groups, int group_size, int t_kv, int n_heads, int q_dtype,
                       int kv_dtype);
// Alignment-head capture of a dense decode launch: for every query row r
// and head h with slot_of_head[h] >= 0, the softmax over the t_kv keys is
// written to out[((row0 + r) * n_selected + slot_of_head[h]) * t_kv + key].
struct CaptureSpec {
  float *out;  // device
  int n_selected, row0;
  int slot_of_head[64];
};
int launch_decode(const void *q, const void *k, const void *v, void *o, int q_dtype,
                  int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                  int n_heads, int64_t q_rs, int64_t kv_rs, int64_t kv_gs, int64_t o_rs,
                  float scale, void *workspace, size_t workspace_bytes, cudaStream_t stream,
                  const CaptureSpec *cap = nullptr);

// ----------------------------------------------------------- paged decode
constexpr int kDecSubRows = 64;     // keys per decode sub-tile (TMA box rows)
constexpr int kDecTailRows = 16;    // box rows of the paged tail loads
constexpr int kPagedMaxRows = 384;  // query rows per paged launch
constexpr int kPagedMaxPages = 16;  // pages per row in one launch

// Kernel-parameter table of one paged decode launch (passed by value, about
// 29 KB, within the 32 KB kernel-parameter limit): for each entry, the query
// / output row it serves (row_of, relative to the launch's first row), that
// row's slot pages and the physical key range [kv_lo, kv_hi) it attends.
// Entries are sorted by descending key count, so the items a persistent grid
// deals out round by round are of similar length.
struct PagedTable {
  int n_rows;
  int layer, n_layers, page_rows;
  int row_of[kPagedMaxRows];
  int kv_lo[kPagedMaxRows];
  int kv_hi[kPagedMaxRows];
  int pages[kPagedMaxRows][kPagedMaxPages];
};

// `map_k` / `map_v` view the page pool as 2-D [rows][64], map_k with boxes
// of kDecSubRows rows and map_v with boxes of kDecTailRows rows (for the
// last, partly attended sub-tile of a row's keys).
int launch_decode_paged(const CUtensorMap &map_k, const CUtensorMap &map_v, const void *q,
                        void *o, int q_dtype, int kv_dtype, int out_dtype, int n_heads,
                        int64_t q_rs, int64_t o_rs, float scale, const PagedTable &pt,
                        int max_keys, void *workspace, size_t workspace_bytes,
                        cudaStream_t stream);
// Upper bound of the workspace of a paged launch of n_rows rows whose key
// ranges span at most max_keys rows.
size_t paged_workspace_bytes(int n_rows, int n_heads, int max_keys);

// Library-owned, zero-initialised decode workspace of the calling thread on
// the current device (grown on demand). Returns NULL on allocation failure.
void *thread_workspace(size_t bytes, cudaStream_t stream);

}  // namespace wattn
