// decode_noalloc.cu -- split-KV decode that allocates nothing.
//
// wattn_decode_fwd needs scratch memory for its split partials and merge
// counters: either a workspace the caller allocated, or one the library
// allocates with cudaMalloc on first use. Some callers can do neither: code
// that runs where allocation is forbidden or unsafe (inside a real-time audio
// callback, under an allocator that must stay frozen after start-up, or in a
// host that hands out only pre-registered device buffers) still needs to
// decode. This entry point gives them the same kernel with its scratch in a
// fixed array compiled into the library.
//
// The array below lives in every GPU's copy of the library's device module
// from the moment the module is loaded until the process exits. Host code
// cannot use its name as a device address (on the host it names a stand-in
// object), so the device address is looked up once per device with
// cudaGetSymbolAddress and then passed to the kernel. All calls on a device
// share the array and it keeps what the last call left there: the counters
// are cleared at the start of every call, and two calls whose kernels
// overlap on the GPU (different streams, or different host threads) race on
// it and give wrong results. The looked-up address belongs to the device's
// current CUDA context: after cudaDeviceReset on a device this entry point
// must not be called there again in the same process.

#include <mutex>

#include "wattn_common.cuh"
#include "wattn_internal.h"

namespace wattn {
namespace {

// Scratch of the no-allocation decode: merge counters, then split partials.
constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // 8 MiB per GPU
constexpr int kMaxDevicesNoAlloc = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevicesNoAlloc] = {nullptr};

// Device address of this device's scratch array, looked up on the first call
// made with that device current.
int scratch_address(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevicesNoAlloc)
    return set_error(WATTN_ERR_CUDA, "decode_fwd_noalloc: no usable current device");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return set_error(WATTN_ERR_CUDA, "decode_fwd_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return WATTN_OK;
}

}  // namespace
}  // namespace wattn

using namespace wattn;

extern "C" int wattn_decode_fwd_noalloc(const void *q, const void *k, const void *v, void *o,
                                        int q_dtype, int kv_dtype, int out_dtype, int n_groups,
                                        int group_size, int t_kv, int n_heads, int d_head,
                                        int64_t q_row_stride, int64_t kv_row_stride,
                                        int64_t kv_group_stride, int64_t o_row_stride,
                                        float scale, void *stream) {
  clear_error();
  // The argument rules of wattn_decode_fwd, all of them (sizes, dtypes,
  // strides, the alignment of q, k and v), checked before anything runs.
  int rc = validate_decode_args(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size,
                                t_kv, n_heads, d_head, q_row_stride, kv_row_stride,
                                kv_group_stride, o_row_stride, scale);
  if (rc != WATTN_OK) return rc;
  if (n_groups == 0) return WATTN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (t_kv == 0)
    return launch_zero_rows(o, out_dtype, 1, n_groups * group_size, n_heads * kHeadDim,
                            o_row_stride, 0, st);
  const DecodePlan pl = plan_decode(n_groups, group_size, t_kv, n_heads, q_dtype, kv_dtype);
  if (pl.n_splits > 1 && pl.workspace_bytes > kNoAllocScratchBytes)
    return set_error(WATTN_ERR_RANGE,
                     "decode_fwd_noalloc: this call needs %zu bytes of scratch; the built-in "
                     "array holds %zu (use wattn_decode_fwd with a workspace)",
                     pl.workspace_bytes, kNoAllocScratchBytes);
  void *scratch = nullptr;
  if ((rc = scratch_address(&scratch)) != WATTN_OK) return rc;
  // The merge counters must start at zero; a call that was cut short (a
  // bounded wait that ran out) may have left some set.
  const size_t counters = (size_t)n_groups * pl.row_chunks * n_heads * sizeof(int);
  if (pl.n_splits > 1 && cudaMemsetAsync(scratch, 0, counters, st) != cudaSuccess)
    return check_launch("decode_fwd_noalloc: clearing counters");
  return launch_decode(q, k, v, o, q_dtype, kv_dtype, out_dtype, n_groups, group_size, t_kv,
                       n_heads, q_row_stride, kv_row_stride, kv_group_stride, o_row_stride, scale,
                       scratch, kNoAllocScratchBytes, st);
}
