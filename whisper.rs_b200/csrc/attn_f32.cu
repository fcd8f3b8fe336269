// attn_f32.cu -- f32 attention on the CUDA cores.
//
// The reference computes attention in f32 end to end (flash_attention_2,
// crates/tensor/src/ops/attention.rs:68-242, with matrixmultiply sgemm for
// both products). This kernel keeps f32 inputs, products and accumulators,
// so it meets the reference's own 1e-5 tolerance
// (crates/tensor/tests/test_flash_attention_tiled.rs:123-130).
//
// One CTA (128 threads) owns 64 query rows of one (utterance, head) and walks
// the keys in 64-key tiles with the online-softmax recurrence of
// attention.rs:173-201, in the exp2 domain (q is pre-scaled by
// scale*log2(e)). Thread (ty, tx) = (tid/8, tid%8) holds a 4 x 8 block of the
// score tile (rows 4ty.., keys 4tx..4tx+3 and 32+4tx..32+4tx+3) and the same
// block of the output (rows 4ty.., the same dims); the 8 threads of a row
// reduce with shuffles. Q and K are kept d-major in shared memory so both
// products read float4s. With the two 4-column halves 32 columns apart, the
// 8 threads of one quarter-warp read 8 consecutive float4s of a K or V row
// (every bank once); 8 contiguous columns per thread put threads tx and
// tx+4 on the same banks (a two-way conflict on every such read, measured
// with ncu as 43 % of the kernel's shared-memory wavefronts).
//
// Small problems (few query blocks x heads for the SMs, e.g. Whisper-tiny's
// one utterance of 6 heads: 144 CTAs) split the keys: each of up to three
// CTAs per query block walks a run of key tiles and writes its unnormalised
// partial (64 sums, m, l per row) to a workspace, and attn_merge_f32_kernel
// combines the parts by the same log-sum-exp rule, in f32.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>

namespace wattn {
namespace {

constexpr int kBM = 64, kBN = 64, kPad = 4, kThreads = 128;

struct F32Params {
  const float *q, *k, *v;
  float *o;
  int64_t q_rs, kv_rs, o_rs, q_bs, kv_bs, o_bs;
  int t_q, t_kv;
  float scale_log2;
  int causal, q_pos_offset;
  int n_splits, split_tiles;  // key splits per query block, key tiles per split
  float *part;                // [batch][head][t_q][n_splits][kPartFloats] when split
};

// One row's partial: 64 sums, m, l, padded to 68 floats so that every row
// starts on a 16-byte boundary (the sums are stored as float4s).
constexpr int kPartFloats = 68;

struct F32Smem {
  float qt[64][kBM + kPad];   // [d][row], pre-scaled by scale * log2(e)
  float kt[64][kBN + kPad];   // [d][key]
  float vs[kBN][64 + kPad];   // [key][d]
  float ps[kBM][kBN + kPad];  // [row][key]
};

__global__ void __launch_bounds__(kThreads) attn_fwd_f32_kernel(const F32Params p) {
  extern __shared__ float4 f32_smem[];
  F32Smem &sm = *reinterpret_cast<F32Smem *>(f32_smem);
  auto &qt = sm.qt;
  auto &kt = sm.kt;
  auto &vs = sm.vs;
  auto &ps = sm.ps;

  const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
  const int head = blockIdx.y, b = blockIdx.z;
  const int split = blockIdx.x % p.n_splits;
  const int q0 = (blockIdx.x / p.n_splits) * kBM;
  const float *qb = p.q + (int64_t)b * p.q_bs + head * kHeadDim;
  const float *kb = p.k + (int64_t)b * p.kv_bs + head * kHeadDim;
  const float *vb = p.v + (int64_t)b * p.kv_bs + head * kHeadDim;

  // Q tile, transposed; warp w loads dims 4*(w + 4i).. of 32 consecutive rows.
  for (int i = 0; i < 8; ++i) {
    const int r = (tid & 31) + 32 * (i & 1), d4 = (tid >> 5) + 4 * (i >> 1);
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < p.t_q) x = *reinterpret_cast<const float4 *>(qb + (int64_t)(q0 + r) * p.q_rs + 4 * d4);
    qt[4 * d4 + 0][r] = x.x * p.scale_log2;
    qt[4 * d4 + 1][r] = x.y * p.scale_log2;
    qt[4 * d4 + 2][r] = x.z * p.scale_log2;
    qt[4 * d4 + 3][r] = x.w * p.scale_log2;
  }

  float m[4], l[4], acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
  }
  int kv_end = p.t_kv;
  if (p.causal) kv_end = min(kv_end, min(q0 + kBM, p.t_q) + p.q_pos_offset);
  const int kv_beg = split * p.split_tiles * kBN;
  if (p.n_splits > 1) kv_end = min(kv_end, kv_beg + p.split_tiles * kBN);

  for (int j0 = kv_beg; j0 < kv_end; j0 += kBN) {
    __syncthreads();  // previous tile fully consumed
    for (int i = 0; i < 8; ++i) {
      const int r = (tid & 31) + 32 * (i & 1), d4 = (tid >> 5) + 4 * (i >> 1);
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j0 + r < p.t_kv) x = *reinterpret_cast<const float4 *>(kb + (int64_t)(j0 + r) * p.kv_rs + 4 * d4);
      kt[4 * d4 + 0][r] = x.x;
      kt[4 * d4 + 1][r] = x.y;
      kt[4 * d4 + 2][r] = x.z;
      kt[4 * d4 + 3][r] = x.w;
    }
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + kThreads * i, r = idx >> 4, d4 = idx & 15;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j0 + r < p.t_kv) x = *reinterpret_cast<const float4 *>(vb + (int64_t)(j0 + r) * p.kv_rs + 4 * d4);
      *reinterpret_cast<float4 *>(&vs[r][4 * d4]) = x;
    }
    __syncthreads();

    // S = (Q * scale * log2 e) K^T for the 4 x 8 block.
    float s[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) s[i][c] = 0.f;
#pragma unroll 8
    for (int d = 0; d < 64; ++d) {
      const float4 a = *reinterpret_cast<const float4 *>(&qt[d][4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&kt[d][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&kt[d][32 + 4 * tx]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) s[i][c] = fmaf(av[i], bv[c], s[i][c]);
    }

    // Mask ragged / causal columns, then the online-softmax update per row.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qrow = q0 + 4 * ty + i;
      const int lim = (p.causal ? min(p.t_kv, qrow + p.q_pos_offset + 1) : p.t_kv) - j0;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if ((c < 4 ? 4 * tx + c : 28 + 4 * tx + c) >= lim) s[i][c] = -INFINITY;
        mx = fmaxf(mx, s[i][c]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_new = fmaxf(m[i], mx);
      const float mu = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m[i] - mu);  // 0 when m[i] = -inf
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        s[i][c] = ex2(s[i][c] - mu);
        sum += s[i][c];
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      l[i] = l[i] * alpha + sum;
      m[i] = m_new;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[i][c] *= alpha;
      *reinterpret_cast<float4 *>(&ps[4 * ty + i][4 * tx]) =
          make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
      *reinterpret_cast<float4 *>(&ps[4 * ty + i][32 + 4 * tx]) =
          make_float4(s[i][4], s[i][5], s[i][6], s[i][7]);
    }
    __syncthreads();

    // O += P V for rows 4ty.., dims 4tx.. and 32+4tx..
#pragma unroll 4
    for (int kk = 0; kk < kBN; kk += 4) {
      float4 pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = *reinterpret_cast<const float4 *>(&ps[4 * ty + i][kk]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 v0 = *reinterpret_cast<const float4 *>(&vs[kk + u][4 * tx]);
        const float4 v1 = *reinterpret_cast<const float4 *>(&vs[kk + u][32 + 4 * tx]);
        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float pv = u == 0 ? pr[i].x : u == 1 ? pr[i].y : u == 2 ? pr[i].z : pr[i].w;
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[i][c] = fmaf(pv, vv[c], acc[i][c]);
        }
      }
    }
  }

  if (p.n_splits > 1) {
    // This split's partial rows: the sums unnormalised, with m and l.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qrow = q0 + 4 * ty + i;
      if (qrow >= p.t_q) continue;
      float *dst = p.part + ((((int64_t)b * gridDim.y + head) * p.t_q + qrow) * p.n_splits + split) *
                                kPartFloats;
      *reinterpret_cast<float4 *>(dst + 4 * tx) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      *reinterpret_cast<float4 *>(dst + 32 + 4 * tx) =
          make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      if (tx == 0) {
        dst[64] = m[i];
        dst[65] = l[i];
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qrow = q0 + 4 * ty + i;
    if (qrow >= p.t_q) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    float *dst = p.o + (int64_t)b * p.o_bs + (int64_t)qrow * p.o_rs + head * kHeadDim + 4 * tx;
    *reinterpret_cast<float4 *>(dst) =
        make_float4(acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv);
    *reinterpret_cast<float4 *>(dst + 32) =
        make_float4(acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv);
  }
}

// One output row of one head from its splits' partials (64 threads, one
// dim each): the parts' offsets m are rescaled to the largest of the parts
// that saw keys, as the online softmax does between key tiles
// (attention.rs:173-201), and the sum is divided by the merged normaliser.
__global__ void __launch_bounds__(64) attn_merge_f32_kernel(const F32Params p) {
  const int row = blockIdx.x, head = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  const float *part =
      p.part + (((int64_t)b * gridDim.y + head) * p.t_q + row) * p.n_splits * kPartFloats;
  float mx = -INFINITY;
  for (int sp = 0; sp < p.n_splits; ++sp)
    if (part[sp * kPartFloats + 65] > 0.f) mx = fmaxf(mx, part[sp * kPartFloats + 64]);
  float acc = 0.f, l = 0.f;
  for (int sp = 0; sp < p.n_splits; ++sp) {
    const float *ps = part + sp * kPartFloats;
    if (!(ps[65] > 0.f)) continue;
    const float w = ex2(ps[64] - mx);
    acc = fmaf(w, ps[d], acc);
    l = fmaf(w, ps[65], l);
  }
  p.o[(int64_t)b * p.o_bs + (int64_t)row * p.o_rs + head * kHeadDim + d] = l > 0.f ? acc / l : 0.f;
}

template <typename T>
__global__ void zero_rows_kernel(T *o, int t, int width, int64_t o_rs, int64_t o_bs) {
  const int row = blockIdx.x, b = blockIdx.y;
  if (row >= t) return;
  T *dst = o + (int64_t)b * o_bs + (int64_t)row * o_rs;
  for (int c = threadIdx.x; c < width; c += blockDim.x) dst[c] = from_f32<T>(0.f);
}

}  // namespace

int launch_attn_f32(const float *q, const float *k, const float *v, float *o, int batch,
                    int t_q, int t_kv, int n_heads, int64_t q_rs, int64_t kv_rs, int64_t o_rs,
                    int64_t q_bs, int64_t kv_bs, int64_t o_bs, float scale, int causal,
                    int q_pos_offset, cudaStream_t stream) {
  F32Params p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = o;
  p.q_rs = q_rs;
  p.kv_rs = kv_rs;
  p.o_rs = o_rs;
  p.q_bs = q_bs;
  p.kv_bs = kv_bs;
  p.o_bs = o_bs;
  p.t_q = t_q;
  p.t_kv = t_kv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.q_pos_offset = q_pos_offset;
  const int n_qblk = (t_q + kBM - 1) / kBM;
  // Key splits while the query blocks x heads fill less than half of the
  // SMs' three resident CTAs (shared memory allows three), at least four key
  // tiles per split; causal calls are not split.
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return check_launch("attn_fwd_f32: device query");
  const long long base = (long long)n_qblk * n_heads * batch;
  const int kv_tiles = (t_kv + kBN - 1) / kBN;
  int n_splits = 1;
  if (!causal && base > 0 && 2 * base <= 3LL * n_sm)
    n_splits = (int)std::min<long long>(std::min<long long>(3, (3LL * n_sm) / base), kv_tiles / 4);
  if (n_splits < 1) n_splits = 1;
  p.split_tiles = (kv_tiles + n_splits - 1) / n_splits;
  n_splits = (kv_tiles + p.split_tiles - 1) / p.split_tiles;
  p.n_splits = std::max(n_splits, 1);
  p.part = nullptr;
  if (p.n_splits > 1) {
    // The calling thread's workspace; its first kCounterBytes are the split
    // counters of the other kernels, which stay zero between calls, so the
    // partials go after them.
    const size_t need = (size_t)base * kBM * p.n_splits * kPartFloats * sizeof(float);
    uint8_t *ws = reinterpret_cast<uint8_t *>(thread_workspace(kCounterBytes + need, stream));
    if (ws != nullptr)
      p.part = reinterpret_cast<float *>(ws + kCounterBytes);
    else
      p.n_splits = 1;  // no workspace: one pass over the keys
  }
  dim3 grid(n_qblk * p.n_splits, n_heads, batch);
  const int smem = (int)sizeof(F32Smem);
  if (cudaFuncSetAttribute(attn_fwd_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(attn_fwd_f32)");
  attn_fwd_f32_kernel<<<grid, kThreads, smem, stream>>>(p);
  if (p.n_splits > 1) {
    int rc = check_launch("attn_fwd_f32");
    if (rc != WATTN_OK) return rc;
    attn_merge_f32_kernel<<<dim3(t_q, n_heads, batch), 64, 0, stream>>>(p);
    return check_launch("attn_merge_f32");
  }
  return check_launch("attn_fwd_f32");
}

int launch_zero_rows(void *o, int out_dtype, int batch, int t, int width, int64_t o_rs,
                     int64_t o_bs, cudaStream_t stream) {
  dim3 grid(t, batch);
  if (out_dtype == WATTN_F32)
    zero_rows_kernel<float><<<grid, 128, 0, stream>>>((float *)o, t, width, o_rs, o_bs);
  else if (out_dtype == WATTN_F16)
    zero_rows_kernel<__half><<<grid, 128, 0, stream>>>((__half *)o, t, width, o_rs, o_bs);
  else
    zero_rows_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>((__nv_bfloat16 *)o, t, width,
                                                              o_rs, o_bs);
  return check_launch("zero_rows");
}

}  // namespace wattn
