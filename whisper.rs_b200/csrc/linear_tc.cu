// linear_tc.cu -- y = x W^T (+ bias) on the sm_100a tensor cores.
//
// The projection of Weight::linear (crates/tensor/src/weight.rs:121,
// ops/matmul.rs:4-110: output[t][r] = sum_c x[t][c] * W[r][c] + bias[r]) for
// 16-bit x and W with f32 accumulation. It produces the decoder's
// cross-attention K and V on the device (precompute_cross_attn,
// crates/whisper/src/decoder.rs:423-447), straight into the layout the decode
// kernels read, so the encoder output never leaves the GPU.
//
// Both operands are K-major, the layout tcgen05 reads. A persistent grid
// (one CTA per SM) walks 128 x 256 tiles of y: a TMA warp streams 64-deep
// k-tiles of x (128 rows) and W (256 rows) through a 4-stage ring (128-byte
// swizzle) without pausing between tiles; an MMA warp issues tcgen05.mma
// M=128, N=256, K=16 (the shape that runs at the tensor-core peak) into one
// of two 256-column TMEM accumulators; four epilogue warps, one per TMEM lane
// quarter, add the bias and store the previous tile from the other
// accumulator meanwhile. Ragged edges: TMA fills out-of-range rows and k with
// zeros, the epilogue masks the stores.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>

namespace wattn {
namespace {

constexpr int kLinBM = 128;
constexpr int kLinBN = 256;
constexpr int kLinBK = 64;                      // one 128-byte swizzle atom of 16-bit
constexpr int kLinStages = 4;
constexpr int kLinABytes = kLinBM * kLinBK * 2;  // 16 KB
constexpr int kLinBBytes = kLinBN * kLinBK * 2;  // 32 KB
constexpr int kLinTmaWarp = 0, kLinMmaWarp = 1;
constexpr int kLinThreads = 6 * 32;              // + four epilogue warps
constexpr uint32_t kLinTmemCols = 512;           // two 256-column accumulators

struct LinSmem {
  uint8_t a[kLinStages][kLinABytes];
  uint8_t b[kLinStages][kLinBBytes];
  uint64_t full[kLinStages], empty[kLinStages];
  uint64_t acc_full[2];   // accumulator b holds a finished tile (MMA commit)
  uint64_t acc_empty[2];  // the epilogue has read accumulator b (one arrival per warp)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct LinParams {
  void *y;
  const float *bias;      // f32 [n] or nullptr
  const float *residual;  // f32 [m][n] (row stride y_rs) added to y, or nullptr; may be y
  int64_t y_rs;
  int m, n, k;
  int tiles_n, n_tiles;  // tiles along n; all tiles (row-tile major)
  int *status;
};

#define LIN_SITE(role, bar, j) ((3 << 24) | ((role) << 16) | ((bar) << 8) | ((j) & 0xff))

template <int IN_DT, int OUT_DT>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap map_x,
                     const __grid_constant__ CUtensorMap map_w, const LinParams p) {
  using OutT = typename Elem<OUT_DT>::T;
  extern __shared__ uint8_t lin_smem_raw[];
  LinSmem &s = *reinterpret_cast<LinSmem *>(
      (reinterpret_cast<uintptr_t>(lin_smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.k + kLinBK - 1) / kLinBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kLinStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s.acc_full[b], 1);
      mbar_init(&s.acc_empty[b], 4);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == kLinMmaWarp) {
    __syncwarp();
    tmem_alloc(&s.tmem_base, kLinTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // (launched with programmatic serialisation: the set-up above overlaps the
  // previous kernel's end; global memory only after it has completed)
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t tmem = s.tmem_base;
  volatile int *abort = &s.abort;

  if (warp == kLinTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_w);
      uint32_t c = 0;  // ring position over all tiles of this CTA
      int last = -1;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
        const int m0 = (t / p.tiles_n) * kLinBM, n0 = (t % p.tiles_n) * kLinBN;
        for (int kt = 0; kt < nk; ++kt, ++c) {
          const int st = c % kLinStages;
          const uint32_t ph = (c / kLinStages) & 1;
          if (!mbar_wait(&s.empty[st], ph ^ 1, abort, p.status, LIN_SITE(1, 1, kt))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[st], kLinABytes + kLinBBytes);
          tma_load_2d(s.a[st], &map_x, &s.full[st], kt * kLinBK, m0);
          tma_load_2d(s.b[st], &map_w, &s.full[st], kt * kLinBK, n0);
          last = (int)c;
        }
      }
      if (*abort && last >= 0) {
        // Let the loads in flight land before shared memory is released.
        volatile int no_abort = 0;
        mbar_wait(&s.full[last % kLinStages], (last / kLinStages) & 1, &no_abort, p.status,
                  LIN_SITE(1, 2, last));
      }
    }
  } else if (warp == kLinMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t ab = IN_DT == WATTN_BF16 ? 1u : 0u;
      constexpr uint32_t idesc = idesc_f16(ab, kLinBM, kLinBN, 0, 0);
      const uint32_t a0 = smem_u32(s.a[0]), b0 = smem_u32(s.b[0]);
      uint32_t c = 0;
      int i = 0;  // tiles of this CTA so far
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x, ++i) {
        const int b = i & 1;
        // Accumulator b was last used by tile i - 2: its epilogue must be done.
        if (i >= 2 && !mbar_wait(&s.acc_empty[b], ((i >> 1) + 1) & 1, abort, p.status,
                                 LIN_SITE(2, 1, i)))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + b * 256;
        for (int kt = 0; kt < nk; ++kt, ++c) {
          const int st = c % kLinStages;
          const uint32_t ph = (c / kLinStages) & 1;
          if (!mbar_wait(&s.full[st], ph, abort, p.status, LIN_SITE(2, 0, kt))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kLinBK / 16; ++kk)
            umma_ss(acc, smem_desc_sw128(a0 + st * kLinABytes + kk * 32, 16, 1024),
                    smem_desc_sw128(b0 + st * kLinBBytes + kk * 32, 16, 1024), idesc,
                    kt > 0 || kk > 0);
          umma_commit(&s.empty[st]);
        }
        if (!ok) break;
        umma_commit(&s.acc_full[b]);
      }
      // Drain: every MMA issued above completes before TMEM is freed
      // (bounded, ignores abort).
      volatile int no_abort = 0;
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0, &no_abort, p.status, LIN_SITE(2, 2, 0));
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      const int m0 = (t / p.tiles_n) * kLinBM, n0 = (t % p.tiles_n) * kLinBN;
      const bool got = mbar_wait(&s.acc_full[b], (i >> 1) & 1, abort, p.status, LIN_SITE(3, 0, i));
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t t_row = tmem + b * 256 + (uint32_t(q * 32) << 16);
      OutT *yrow = reinterpret_cast<OutT *>(p.y) + (int64_t)row * p.y_rs;
#pragma unroll 1
      for (int ch = 0; ch < kLinBN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld32(t_row + ch * 32, r);
        tmem_wait_ld();
        reg_fence(r);
        const int c0 = n0 + ch * 32;
        if (row < p.m && c0 < p.n) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = c0 + e;
            v[e] = __uint_as_float(r[e]) +
                   ((p.bias != nullptr && col < p.n) ? __ldg(p.bias + col) : 0.f);
          }
          if (p.residual != nullptr) {  // y may alias it: each element is read before it is written
            const float *res = p.residual + (int64_t)row * p.y_rs + c0;
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c0 + e < p.n) v[e] += res[e];
          }
          OutT *dst = yrow + c0;
          if (c0 + 32 <= p.n && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            if constexpr (sizeof(OutT) == 4) {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                reinterpret_cast<float4 *>(dst)[e] =
                    make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                reinterpret_cast<uint4 *>(dst)[e] = make_uint4(
                    pack2<OutT>(v[8 * e], v[8 * e + 1]), pack2<OutT>(v[8 * e + 2], v[8 * e + 3]),
                    pack2<OutT>(v[8 * e + 4], v[8 * e + 5]),
                    pack2<OutT>(v[8 * e + 6], v[8 * e + 7]));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c0 + e < p.n) dst[e] = from_f32<OutT>(v[e]);
          }
        }
      }
      // Accumulator b may take the tile after next.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kLinMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kLinTmemCols);
  }
}

template <int IN_DT, int OUT_DT>
int launch_linear_typed(const CUtensorMap &mx, const CUtensorMap &mw, const LinParams &p,
                        cudaStream_t stream) {
  auto kern = linear_tc_kernel<IN_DT, OUT_DT>;
  const int smem = (int)sizeof(LinSmem) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(linear_tc)");
  // Persistent grid: one CTA per SM (the ring's shared memory allows no second).
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return check_launch("linear_tc: device query");
  if (launch_pdl(kern, dim3(std::min(p.n_tiles, n_sm)), dim3(kLinThreads), smem, stream, mx, mw,
                 p) != cudaSuccess)
    return check_launch("linear_tc (launch)");
  return check_launch("linear_tc");
}

}  // namespace

int launch_linear(const void *x, const void *w, const float *bias, void *y, int in_dtype,
                  int out_dtype, int m, int n, int k, int64_t x_rs, int64_t w_rs, int64_t y_rs,
                  cudaStream_t stream, const float *residual) {
  if (m == 0 || n == 0) return WATTN_OK;
  const long long tiles_m = (m + kLinBM - 1) / kLinBM, tiles_n = (n + kLinBN - 1) / kLinBN;
  if (tiles_m * tiles_n > 2147483647LL)
    return set_error(WATTN_ERR_INVALID, "linear: %lld tiles exceed 2^31", tiles_m * tiles_n);
  CUtensorMap mx, mw;
  const uint64_t dx[2] = {(uint64_t)k, (uint64_t)m}, sx[1] = {(uint64_t)x_rs * 2};
  const uint64_t dw[2] = {(uint64_t)k, (uint64_t)n}, sw[1] = {(uint64_t)w_rs * 2};
  const uint32_t bx[2] = {kLinBK, kLinBM}, bw[2] = {kLinBK, kLinBN};
  int rc = encode_tmap(&mx, tmap_dtype(in_dtype), 2, x, dx, sx, bx, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != WATTN_OK) return rc;
  rc = encode_tmap(&mw, tmap_dtype(in_dtype), 2, w, dw, sw, bw, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != WATTN_OK) return rc;
  LinParams p;
  p.y = y;
  p.bias = bias;
  p.residual = residual;
  p.y_rs = y_rs;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_n = (int)tiles_n;
  p.n_tiles = (int)(tiles_m * tiles_n);
  p.status = device_status_ptr();
  if (p.status == nullptr) return WATTN_ERR_CUDA;
#define WATTN_LIN_CASE(ID, OD) \
  if (in_dtype == ID && out_dtype == OD) return launch_linear_typed<ID, OD>(mx, mw, p, stream);
  WATTN_LIN_CASE(WATTN_F16, WATTN_F32)
  WATTN_LIN_CASE(WATTN_F16, WATTN_F16)
  WATTN_LIN_CASE(WATTN_F16, WATTN_BF16)
  WATTN_LIN_CASE(WATTN_BF16, WATTN_F32)
  WATTN_LIN_CASE(WATTN_BF16, WATTN_F16)
  WATTN_LIN_CASE(WATTN_BF16, WATTN_BF16)
#undef WATTN_LIN_CASE
  return set_error(WATTN_ERR_INVALID, "linear: 16-bit inputs only");
}

// ---------------------------------------------------------------- layer norm
namespace {

// layer_norm_row (crates/tensor/src/ops/norm.rs:67-98, the scalar order):
// mean, population variance around it, y = (x - mean) / sqrt(var + eps) *
// gamma + beta; one warp per row, f32 statistics, 16-bit output for the
// projection that follows.
template <typename OutT>
__global__ void __launch_bounds__(256)
    layer_norm_kernel(const float *x, const float *gamma, const float *beta, OutT *y, int rows,
                      int d, float eps) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *xr = x + (int64_t)row * d;
  float sum = 0.f;
  for (int i = lane; i < d; i += 32) sum += xr[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)d;
  float sq = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float t = xr[i] - mean;
    sq = fmaf(t, t, sq);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float inv_std = 1.0f / sqrtf(sq / (float)d + eps);
  OutT *yr = y + (int64_t)row * d;
  for (int i = lane; i < d; i += 32)
    yr[i] = from_f32<OutT>((xr[i] - mean) * inv_std * __ldg(gamma + i) + __ldg(beta + i));
}

}  // namespace

int launch_layer_norm(const float *x, const float *gamma, const float *beta, void *y, int out_dtype,
                      int rows, int d, float eps, cudaStream_t stream) {
  if (rows == 0) return WATTN_OK;
  const dim3 grid((rows + 7) / 8);
  if (out_dtype == WATTN_F16)
    launch_pdl(layer_norm_kernel<__half>, grid, dim3(256), 0, stream, x, gamma, beta, (__half *)y,
               rows, d, eps);
  else if (out_dtype == WATTN_BF16)
    launch_pdl(layer_norm_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream, x, gamma, beta,
               (__nv_bfloat16 *)y, rows, d, eps);
  else
    return set_error(WATTN_ERR_INVALID, "layer_norm: 16-bit output only");
  return check_launch("layer_norm");
}

}  // namespace wattn
