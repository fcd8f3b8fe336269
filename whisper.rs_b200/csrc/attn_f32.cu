// attn_f32.cu -- f32 attention on the tensor cores (3xTF32).
//
// The reference computes attention in f32 end to end (flash_attention_2,
// crates/tensor/src/ops/attention.rs:68-242, with matrixmultiply sgemm for
// both products) and its tests hold the result to 1e-5
// (crates/tensor/tests/test_flash_attention_tiled.rs:123-130). This path
// keeps f32 inputs, f32 softmax and f32 accumulators, and computes both
// products on the tensor cores with the 3xTF32 split (Ootomo and Yokota,
// "Recovering single precision accuracy from Tensor Cores while surpassing
// the FP32 theoretical peak performance", IJHPCA 2022): every f32 operand x
// is split into x_hi = tf32(x) and x_lo = x - x_hi, and each product a*b is
// computed as a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with three tcgen05.mma of
// kind::tf32. The dropped a_lo*b_lo and the 10-bit mantissa the tensor core
// keeps of each lo part leave about 2^-21 of relative error per product, the
// order of f32 accumulation itself.
//
// Two launches:
//  * f32_split_kernel (bandwidth-bound): K as [bh][t][64] and V transposed
//    as [bh][64][t] (K-major over the keys, for the PV product), each as a
//    hi and a lo array; it also zeroes the split counters of the launch.
//  * attn_f32tc_kernel: one CTA per 128 query rows of one (utterance, head)
//    and run of 64-key tiles. Four softmax warps (one query row per thread,
//    the row's TMEM lane) load, scale (scale * log2 e: scores come out in
//    the exp2 domain) and split their Q rows into tensor memory, where they
//    are the A operand of S = Q K^T; a TMA warp streams the split K and V^T
//    tiles through a 3-stage ring; an MMA warp issues S for the next tile
//    before PV of the current one. P is split by the softmax warps into two
//    double-buffered TMEM regions, so that the softmax of tile j+1 overlaps
//    PV of tile j. Tensor memory (512 columns): S [0,64), O [64,128),
//    Q_hi [128,192), Q_lo [192,256), P buffer b: hi [256+128b, 320+128b),
//    lo [320+128b, 384+128b).
//
// Small problems (few query blocks x heads for the SMs, e.g. Whisper-tiny's
// one utterance of 6 heads: 72 blocks) split the keys: each CTA of a query
// block walks a run of key tiles and writes its unnormalised partial (64
// sums, m, l per row); the last CTA of the block to finish (a counter per
// block) combines the parts by the online-softmax rule of
// attention.rs:173-201 and writes the output.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>
#include <climits>

namespace wattn {
namespace {

constexpr int kTcRows = 128;    // query rows per CTA (UMMA M)
constexpr int kTcKeys = 64;     // keys per tile (UMMA N of S, K of PV)
constexpr int kTcStages = 3;    // K / V^T ring
constexpr int kTcThreads = 6 * 32;  // softmax warps 0-3, TMA warp 4, MMA warp 5
constexpr int kTcTmaWarp = 4, kTcMmaWarp = 5;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 64, kColQh = 128, kColQl = 192, kColP = 256;

// One row's partial: 64 sums, m, l, padded to 68 floats so that every row
// starts on a 16-byte boundary (the sums are stored as float4s).
constexpr int kPartFloats = 68;

// x_hi of a non-negative finite x below 2^127 (the softmax weights, <= 256):
// tf32 to nearest, ties away from zero, with integer operations (the ALU
// pipe, leaving the SFU to the exponentials).
WATTN_DEVINL uint32_t tf32_hi_bits(float x) { return (__float_as_uint(x) + 0x1000u) & 0xffffe000u; }

// ------------------------------------------------------------ split pre-pass
// Thread i handles 4 consecutive elements of a 64-wide row (a float4) of K
// or of V, in that order over one flat index space; the V parts go out
// transposed, walked with the key fastest so that a warp's writes are
// consecutive.
struct SplitParams {
  const float *k, *v;
  int64_t kv_rs, kv_bs;
  int batch, n_heads, t_kv, t_kv_pad;
  float *kh, *kl, *vh, *vl;
  int *cnt;  // split counters of the attention launch, zeroed here
  int n_cnt;
  const float *q;  // Q rows, prefetched into L2 for the attention launch
  int64_t q_rs, q_bs;
  int t_q;
};

__global__ void __launch_bounds__(256) f32_split_kernel(const SplitParams p) {
  grid_dep_wait();
  grid_dep_launch();
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (tid < p.n_cnt) p.cnt[tid] = 0;
  {
    // Q's 128-byte lines into L2: the attention CTAs start by reading
    // their Q rows, a latency every CTA would otherwise wait out on DRAM.
    const int lines_per_row = p.n_heads * 2;
    const long long n_lines = (long long)p.batch * p.t_q * lines_per_row;
    for (long long i = tid; i < n_lines; i += (long long)gridDim.x * blockDim.x) {
      const long long row = i / lines_per_row;
      const int b = (int)(row / p.t_q), t = (int)(row - (long long)b * p.t_q);
      const float *line = p.q + b * p.q_bs + (int64_t)t * p.q_rs + (i - row * lines_per_row) * 32;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
  }
  const long long bh_n = (long long)p.batch * p.n_heads;
  const long long nk = bh_n * p.t_kv * 16;
  for (long long i = tid; i < 2 * nk; i += (long long)gridDim.x * blockDim.x) {
    const bool is_v = i >= nk;
    const long long r = is_v ? i - nk : i;
    long long bh;
    int t, d4;
    if (!is_v) {
      d4 = (int)(r & 15);
      const long long bt = r >> 4;
      bh = bt / p.t_kv;
      t = (int)(bt - bh * p.t_kv);
    } else {
      const long long bd = r / p.t_kv;
      t = (int)(r - bd * p.t_kv);
      bh = bd >> 4;
      d4 = (int)(bd & 15);
    }
    const int b = (int)(bh / p.n_heads), h = (int)(bh - (long long)b * p.n_heads);
    const float *src = (is_v ? p.v : p.k) + b * p.kv_bs + (int64_t)t * p.kv_rs;
    const float4 x = __ldg(reinterpret_cast<const float4 *>(src + h * kHeadDim + 4 * d4));
    const float xv[4] = {x.x, x.y, x.z, x.w};
    float hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hi[e] = round_tf32(xv[e]);
      lo[e] = round_tf32(xv[e] - hi[e]);
    }
    if (!is_v) {
      const int64_t off = ((int64_t)bh * p.t_kv + t) * kHeadDim + 4 * d4;
      *reinterpret_cast<float4 *>(p.kh + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<float4 *>(p.kl + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t off = ((int64_t)bh * kHeadDim + 4 * d4 + e) * p.t_kv_pad + t;
        p.vh[off] = hi[e];
        p.vl[off] = lo[e];
      }
    }
  }
}

// ------------------------------------------------------------ attention
struct TcParams {
  const float *q;  // raw Q rows (the softmax warps scale and split them)
  int64_t q_rs, q_bs;
  float qc;  // scale * log2(e)
  float *o;
  int64_t o_rs, o_bs;
  int t_q, t_kv, n_heads, n_qblk;
  int causal, q_pos_offset;
  int n_splits, split_tiles;  // key splits per query block, 64-key tiles per split
  float *part;                // [batch][head][t_q][n_splits][kPartFloats] when split
  int *cnt;                   // one counter per query block when split (zero on entry)
  int *status;
};

struct TcSmem {
  // [stage][32-value block][rows x 32 values]: K rows (keys) over dims
  // 0-31 and 32-63; V^T rows (dims) over keys 0-31 and 32-63.
  float kh[kTcStages][2][kTcKeys * 32], kl[kTcStages][2][kTcKeys * 32];
  float vh[kTcStages][2][64 * 32], vl[kTcStages][2][64 * 32];
  uint64_t kv_full[kTcStages], kv_empty[kTcStages];
  uint64_t q_full, s_full, s_free, p_full[2], pv_done[2], drain;
  uint32_t tmem_base;
  int abort, last;
};

// Wait sites (kernel 3): role << 16 | barrier << 8 | iteration.
#define TF_SITE(role, bar, j) ((3 << 24) | ((role) << 16) | ((bar) << 8) | ((j) & 0xff))

WATTN_DEVINL void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kTcThreads, 1)
    attn_f32tc_kernel(const __grid_constant__ CUtensorMap map_kh,
                      const __grid_constant__ CUtensorMap map_kl,
                      const __grid_constant__ CUtensorMap map_vh,
                      const __grid_constant__ CUtensorMap map_vl, const TcParams p) {
  extern __shared__ uint8_t tc_smem_raw[];
  TcSmem &s = *reinterpret_cast<TcSmem *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) &
                                          ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, b = blockIdx.z;
  const int split = blockIdx.x % p.n_splits, qblk = blockIdx.x / p.n_splits;
  const int q0 = qblk * kTcRows;
  const int bh = b * p.n_heads + head;
  int kv_end = p.t_kv;
  if (p.causal) kv_end = min(kv_end, min(q0 + kTcRows, p.t_q) + p.q_pos_offset);
  const int kv_beg = split * p.split_tiles * kTcKeys;
  if (p.n_splits > 1) kv_end = min(kv_end, kv_beg + p.split_tiles * kTcKeys);
  const int n_tiles = kv_end > kv_beg ? (kv_end - kv_beg + kTcKeys - 1) / kTcKeys : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    mbar_init(&s.q_full, kTcRows);
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_free, kTcRows);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.p_full[i], kTcRows);
      mbar_init(&s.pv_done[i], 1);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    s.last = 0;
    fence_barrier_init();
  }
  if (warp == kTcMmaWarp) {
    __syncwarp();
    tmem_alloc(&s.tmem_base, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t tmem = s.tmem_base;
  volatile int *abort = &s.abort;

  if (warp == kTcTmaWarp) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&map_kh);
      tma_prefetch_desc(&map_vh);
      int last = -1;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kTcStages;
        if (j >= kTcStages &&
            !mbar_wait(&s.kv_empty[st], ((j / kTcStages) - 1) & 1, abort, p.status,
                       TF_SITE(1, 1, j)))
          break;
        const int key0 = kv_beg + j * kTcKeys;
        mbar_arrive_expect_tx(&s.kv_full[st], 8 * kTcKeys * 32 * 4);
        for (int blk = 0; blk < 2; ++blk) {
          tma_load_3d(s.kh[st][blk], &map_kh, &s.kv_full[st], 32 * blk, key0, bh);
          tma_load_3d(s.kl[st][blk], &map_kl, &s.kv_full[st], 32 * blk, key0, bh);
          tma_load_3d(s.vh[st][blk], &map_vh, &s.kv_full[st], key0 + 32 * blk, 0, bh);
          tma_load_3d(s.vl[st][blk], &map_vl, &s.kv_full[st], key0 + 32 * blk, 0, bh);
        }
        last = j;
      }
      if (*abort && last >= 0) {
        // let the loads in flight land before the shared memory is released
        volatile int no_abort = 0;
        mbar_wait(&s.kv_full[last % kTcStages], (last / kTcStages) & 1, &no_abort, p.status,
                  TF_SITE(1, 3, last));
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc = idesc_tf32(kTcRows, 64);  // M=128, N=64 (keys, or dims)
      const uint32_t t_s = tmem + kColS, t_o = tmem + kColO, t_qh = tmem + kColQh,
                     t_ql = tmem + kColQl;
      // K-major SW128 B operands: rows of 128 bytes (32 values), 8-row atoms
      // of 1024 bytes; the 64 values of a row sit in two 32-column blocks.
      // Step ks (8 values, 32 bytes) of the 64: block ks / 4, +32 bytes per
      // step within it. The descriptors are made once and moved by adding
      // to their address field (16-byte units). A operands (Q, P) are TMEM
      // rows, 8 columns per step. Measured on B200: an M128 N64 K8 step
      // takes ~44 SM cycles when issued back to back alone (as does an f16
      // M128 N64 K16 one; N128 ~64, N256 ~128), and 60-80 here beside the
      // softmax warps: 48 steps per key tile set the kernel's pace.
      constexpr uint32_t kStage16 = sizeof(s.kh[0]) >> 4, kBlk16 = sizeof(s.kh[0][0]) >> 4;
      const uint64_t d_kh = smem_desc_sw128(smem_u32(s.kh[0][0]), 16, 1024),
                     d_kl = smem_desc_sw128(smem_u32(s.kl[0][0]), 16, 1024),
                     d_vh = smem_desc_sw128(smem_u32(s.vh[0][0]), 16, 1024),
                     d_vl = smem_desc_sw128(smem_u32(s.vl[0][0]), 16, 1024);
      auto step = [](uint64_t d, int ks) -> uint64_t {
        return d + (ks < 4 ? 0u : kBlk16) + 2 * (ks & 3);
      };
      bool ok = mbar_wait(&s.q_full, 0, abort, p.status, TF_SITE(2, 0, 0));
      // S = Q_hi K_lo + Q_lo K_hi + Q_hi K_hi: the two small products first,
      // into an empty accumulator, then the large one (measured on config 1:
      // max-abs error 2.6e-6 against the f32 oracle, 3.6e-6 the other way
      // round, at the same speed); the same order for each tile's PV.
      auto s_step = [&](int j) -> bool {
        const int st = j % kTcStages;
        const uint64_t kh = d_kh + st * kStage16, kl = d_kl + st * kStage16;
        if (!mbar_wait(&s.kv_full[st], (j / kTcStages) & 1, abort, p.status, TF_SITE(2, 1, j)))
          return false;
        if (j > 0 && !mbar_wait(&s.s_free, (j - 1) & 1, abort, p.status, TF_SITE(2, 2, j)))
          return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_s, t_qh + 8 * ks, step(kl, ks), idesc, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_s, t_ql + 8 * ks, step(kh, ks), idesc, 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_s, t_qh + 8 * ks, step(kh, ks), idesc, 1);
        umma_commit(&s.s_full);
        return true;
      };
      if (ok) {
        tc_fence_after();
        ok = s_step(0);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % kTcStages, pb = j & 1;
        const uint64_t vh = d_vh + st * kStage16, vl = d_vl + st * kStage16;
        if (j + 1 < n_tiles && !s_step(j + 1)) break;
        if (!mbar_wait(&s.p_full[pb], (j >> 1) & 1, abort, p.status, TF_SITE(2, 3, j))) break;
        tc_fence_after();
        // O += P_hi V_lo + P_lo V_hi + P_hi V_hi
        const uint32_t t_ph = tmem + kColP + 128 * pb, t_pl = t_ph + 64;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_o, t_ph + 8 * ks, step(vl, ks), idesc,
                       j > 0 || ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_o, t_pl + 8 * ks, step(vh, ks), idesc, 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_ts_tf32(t_o, t_ph + 8 * ks, step(vh, ks), idesc, 1);
        umma_commit(&s.pv_done[pb]);
        umma_commit(&s.kv_empty[st]);
      }
      volatile int no_abort = 0;
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0, &no_abort, p.status, TF_SITE(2, 4, 0));
    }
  } else {
    // ---------------------------------------------------------- softmax
    // Thread = query row (its TMEM lane); scores in the exp2 domain.
    const int row = warp * 32 + lane, qrow = q0 + row;
    const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
    const uint32_t t_s = lane_base + kColS, t_o = lane_base + kColO;
    {
      // the Q row, scaled and split (rows past t_q are zeros)
      const float *src = p.q + (int64_t)b * p.q_bs + (int64_t)qrow * p.q_rs + head * kHeadDim;
      const bool in = qrow < p.t_q;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const float4 x = in ? __ldg(reinterpret_cast<const float4 *>(src + 16 * c + 4 * e4))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
          const float xv[4] = {x.x * p.qc, x.y * p.qc, x.z * p.qc, x.w * p.qc};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float h = round_tf32(xv[e]);
            hi[4 * e4 + e] = __float_as_uint(h);
            lo[4 * e4 + e] = __float_as_uint(xv[e] - h);
          }
        }
        tmem_st16(lane_base + kColQh + 16 * c, hi);
        tmem_st16(lane_base + kColQl + 16 * c, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&s.q_full);
    }
    const int lim_row = p.causal ? min(p.t_kv, qrow + p.q_pos_offset + 1) : p.t_kv;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int pb = j & 1;
      const bool got = mbar_wait(&s.s_full, j & 1, abort, p.status, TF_SITE(3, 0, j));
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[2][32];
      tmem_ld32(t_s, r[0]);
      tmem_ld32(t_s + 32, r[1]);
      tmem_wait_ld();
      reg_fence(r[0]);
      reg_fence(r[1]);
      tc_fence_before();
      mbar_arrive(&s.s_free);
      const int lim = lim_row - (kv_beg + j * kTcKeys);  // visible keys of this tile
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float v = i < lim ? __uint_as_float(r[i >> 5][i & 31]) : -INFINITY;
        r[i >> 5][i & 31] = __float_as_uint(v);
        mx4[i & 3] = fmaxf(mx4[i & 3], v);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // Lazy rescale (the online softmax of attention.rs:173-201, with the
      // offset moved only when the max grows by more than 2^8: p then stays
      // <= 256 and the result is exact either way).
      const bool need = mx > m + 8.f;
      const bool warp_need = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2(m - mx) : 1.f;  // 0 on the first tile (m = -inf)
      if (need) {
        l *= alpha;
        m = mx;
      }
      const float mu = (m == -INFINITY) ? 0.f : m;
      // P buffer pb is free once PV(j-2) is complete.
      if (j >= 2) {
        const bool fr = mbar_wait(&s.pv_done[pb], ((j >> 1) - 1) & 1, abort, p.status,
                                  TF_SITE(3, 1, j));
        if (!__all_sync(0xffffffffu, fr)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const uint32_t t_ph = lane_base + kColP + 128 * pb, t_pl = t_ph + 64;
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t ch[32], cl[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pv = ex2(__uint_as_float(r[h2][i]) - mu);
          sum4[i & 3] += pv;
          const uint32_t hb = tf32_hi_bits(pv);
          ch[i] = hb;
          cl[i] = __float_as_uint(pv - __uint_as_float(hb));
        }
        tmem_st32(t_ph + 32 * h2, ch);
        tmem_st32(t_pl + 32 * h2, cl);
      }
      l += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      // O is rescaled once PV(j-1) is complete.
      if (j > 0 && warp_need) {
        const bool done = mbar_wait(&s.pv_done[pb ^ 1], ((j - 1) >> 1) & 1, abort, p.status,
                                    TF_SITE(3, 2, j));
        if (!__all_sync(0xffffffffu, done)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t o[2][32];
        tmem_ld32(t_o, o[0]);
        tmem_ld32(t_o + 32, o[1]);
        tmem_wait_ld();
        reg_fence(o[0]);
        reg_fence(o[1]);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[h2][i] = __float_as_uint(__uint_as_float(o[h2][i]) * alpha);
        tmem_st32(t_o, o[0]);
        tmem_st32(t_o + 32, o[1]);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&s.p_full[pb]);
    }
    // ---------------------------------------------------------- epilogue
    bool have = false;  // this thread's O row, m and l are complete
    uint32_t o[2][32];
    if (ok && n_tiles > 0) {
      const bool fin = mbar_wait(&s.pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, abort,
                                 p.status, TF_SITE(3, 3, n_tiles));
      if (__all_sync(0xffffffffu, fin)) {
        tc_fence_after();
        tmem_ld32(t_o, o[0]);
        tmem_ld32(t_o + 32, o[1]);
        tmem_wait_ld();
        reg_fence(o[0]);
        reg_fence(o[1]);
        have = true;
      }
    }
    const bool row_out = have && qrow < p.t_q;
    float *dst = p.o + (int64_t)b * p.o_bs + (int64_t)qrow * p.o_rs + head * kHeadDim;
    if (p.n_splits == 1) {
      if (row_out) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4 *>(dst + 4 * c) =
              make_float4(__uint_as_float(o[c >> 3][(4 * c) & 31]) * inv,
                          __uint_as_float(o[c >> 3][(4 * c + 1) & 31]) * inv,
                          __uint_as_float(o[c >> 3][(4 * c + 2) & 31]) * inv,
                          __uint_as_float(o[c >> 3][(4 * c + 3) & 31]) * inv);
      }
    } else {
      // This split's partial row (sums unnormalised, m, l); the last CTA of
      // the query block to get here merges all parts. Every softmax thread
      // takes both barriers, whatever its state, so that none waits alone.
      float *part_row =
          p.part + (((int64_t)bh * p.t_q + qrow) * p.n_splits) * kPartFloats;
      if (row_out) {
        float *mine = part_row + split * kPartFloats;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4 *>(mine + 4 * c) =
              make_float4(__uint_as_float(o[c >> 3][(4 * c) & 31]),
                          __uint_as_float(o[c >> 3][(4 * c + 1) & 31]),
                          __uint_as_float(o[c >> 3][(4 * c + 2) & 31]),
                          __uint_as_float(o[c >> 3][(4 * c + 3) & 31]));
        mine[64] = m;
        mine[65] = l;
      }
      __threadfence();
      softmax_sync();
      if (threadIdx.x == 0) {
        int is_last = 0;
        if (!*abort) {
          int *cnt = p.cnt + (int64_t)bh * p.n_qblk + qblk;
          is_last = atomicAdd(cnt, 1) == p.n_splits - 1;
          if (is_last) *cnt = 0;  // ready for the next launch on this workspace
          __threadfence();
        }
        s.last = is_last;
      }
      softmax_sync();
      if (s.last && row_out) {
        float mx = l > 0.f ? m : -INFINITY;
        for (int sp = 0; sp < p.n_splits; ++sp)
          if (sp != split && __ldcg(part_row + sp * kPartFloats + 65) > 0.f)
            mx = fmaxf(mx, __ldcg(part_row + sp * kPartFloats + 64));
        const float w0 = l > 0.f ? ex2(m - mx) : 0.f;
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = __uint_as_float(o[i >> 5][i & 31]) * w0;
        float lt = l * w0;
        for (int sp = 0; sp < p.n_splits; ++sp) {
          const float *ps = part_row + sp * kPartFloats;
          if (sp == split) continue;
          const float pl = __ldcg(ps + 65);
          if (!(pl > 0.f)) continue;
          const float w = ex2(__ldcg(ps + 64) - mx);
          lt = fmaf(w, pl, lt);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float4 x = __ldcg(reinterpret_cast<const float4 *>(ps + 4 * c));
            acc[4 * c] = fmaf(w, x.x, acc[4 * c]);
            acc[4 * c + 1] = fmaf(w, x.y, acc[4 * c + 1]);
            acc[4 * c + 2] = fmaf(w, x.z, acc[4 * c + 2]);
            acc[4 * c + 3] = fmaf(w, x.w, acc[4 * c + 3]);
          }
        }
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4 *>(dst + 4 * c) =
              make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv,
                          acc[4 * c + 3] * inv);
      }
    }
  }

  // Teardown: after the last TMEM access of every warp, free the columns.
  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

template <typename T>
__global__ void zero_rows_kernel(T *o, int t, int width, int64_t o_rs, int64_t o_bs) {
  const int row = blockIdx.x, b = blockIdx.y;
  if (row >= t) return;
  T *dst = o + (int64_t)b * o_bs + (int64_t)row * o_rs;
  for (int c = threadIdx.x; c < width; c += blockDim.x) dst[c] = from_f32<T>(0.f);
}

// Launch plan of one call. Workspace: [counters][partials][K hi, lo][V^T hi, lo].
struct F32Plan {
  int n_qblk, n_splits, split_tiles, t_kv_pad;
  size_t part_bytes, kb, vb, total;
};

F32Plan plan_f32(int batch, int t_q, int t_kv, int n_heads, int causal, int n_sm) {
  F32Plan pl;
  const long long bh = (long long)batch * n_heads;
  pl.n_qblk = (t_q + kTcRows - 1) / kTcRows;
  const int kv_tiles = (t_kv + kTcKeys - 1) / kTcKeys;
  const long long base = (long long)pl.n_qblk * bh;
  // Key splits while the query blocks leave SMs idle (one CTA per SM by
  // shared memory and tensor memory), at least two key tiles per split;
  // causal calls are not split.
  int n_splits = 1;
  if (!causal && base < n_sm)
    n_splits = (int)std::min<long long>(std::max<long long>(1, n_sm / base), kv_tiles / 2);
  n_splits = std::max(n_splits, 1);
  pl.split_tiles = (kv_tiles + n_splits - 1) / n_splits;
  pl.n_splits = std::max(1, (kv_tiles + pl.split_tiles - 1) / pl.split_tiles);
  pl.t_kv_pad = (t_kv + 3) & ~3;
  pl.part_bytes =
      pl.n_splits > 1 ? round_up_256((size_t)bh * t_q * pl.n_splits * kPartFloats * sizeof(float))
                      : 0;
  pl.kb = round_up_256((size_t)bh * t_kv * kHeadDim * 4);
  pl.vb = round_up_256((size_t)bh * kHeadDim * pl.t_kv_pad * 4);
  pl.total = kCounterBytes + pl.part_bytes + 2 * pl.kb + 2 * pl.vb;
  return pl;
}

}  // namespace

size_t attn_f32_workspace_bytes(int batch, int t_q, int t_kv, int n_heads, int n_sm) {
  return plan_f32(batch, t_q, t_kv, n_heads, 0, n_sm).total;
}

int launch_attn_f32(const float *q, const float *k, const float *v, float *o, int batch,
                    int t_q, int t_kv, int n_heads, int64_t q_rs, int64_t kv_rs, int64_t o_rs,
                    int64_t q_bs, int64_t kv_bs, int64_t o_bs, float scale, int causal,
                    int q_pos_offset, cudaStream_t stream, void *ws, size_t ws_bytes) {
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return check_launch("attn_f32: device query");
  const long long bh = (long long)batch * n_heads;
  const F32Plan pl = plan_f32(batch, t_q, t_kv, n_heads, causal, n_sm);
  if ((long long)pl.n_qblk * pl.n_splits > INT_MAX || batch > 65535 || n_heads > 65535)
    return set_error(WATTN_ERR_INVALID, "attention: too many rows");
  if (ws != nullptr && ws_bytes < pl.total)
    return set_error(WATTN_ERR_INVALID,
                     "attention: a workspace of %zu bytes is needed for f32 inputs (%zu given)",
                     pl.total, ws_bytes);
  uint8_t *wsb = reinterpret_cast<uint8_t *>(ws != nullptr ? ws : thread_workspace(pl.total, stream));
  if (wsb == nullptr) return set_error(WATTN_ERR_NOMEM, "attention workspace allocation failed");
  uint8_t *cur = wsb + kCounterBytes;
  TcParams tp;
  tp.part = pl.n_splits > 1 ? reinterpret_cast<float *>(cur) : nullptr;
  cur += pl.part_bytes;
  SplitParams sp;
  sp.k = k;
  sp.v = v;
  sp.kv_rs = kv_rs;
  sp.kv_bs = kv_bs;
  sp.batch = batch;
  sp.n_heads = n_heads;
  sp.t_kv = t_kv;
  sp.t_kv_pad = pl.t_kv_pad;
  sp.kh = reinterpret_cast<float *>(cur);
  sp.kl = reinterpret_cast<float *>(cur + pl.kb);
  sp.vh = reinterpret_cast<float *>(cur + 2 * pl.kb);
  sp.vl = reinterpret_cast<float *>(cur + 2 * pl.kb + pl.vb);
  sp.cnt = reinterpret_cast<int *>(wsb);
  sp.n_cnt = pl.n_splits > 1 ? (int)(bh * pl.n_qblk) : 0;  // < n_sm when split
  sp.q = q;
  sp.q_rs = q_rs;
  sp.q_bs = q_bs;
  sp.t_q = t_q;
  const long long items = bh * t_kv * 32;
  const int split_blocks = (int)std::max<long long>(
      1, std::min<long long>((items + 255) / 256, (long long)n_sm * 8));
  if (launch_pdl(f32_split_kernel, dim3(split_blocks), dim3(256), 0, stream, sp) != cudaSuccess)
    return check_launch("f32_split (launch)");
  // Tensor maps: K as [bh][t][64] (boxes of 32 values x 64 keys), V^T as
  // [bh][64][t_kv] (boxes of 32 keys x 64 dims); rows past the extents read
  // as zero.
  CUtensorMap mkh, mkl, mvh, mvl;
  int rc;
  {
    const uint64_t dk[3] = {64, (uint64_t)t_kv, (uint64_t)bh};
    const uint64_t sk[2] = {64 * 4, (uint64_t)t_kv * 64 * 4};
    const uint32_t boxk[3] = {32, (uint32_t)kTcKeys, 1};
    const uint64_t dv[3] = {(uint64_t)t_kv, 64, (uint64_t)bh};
    const uint64_t sv[2] = {(uint64_t)pl.t_kv_pad * 4, (uint64_t)pl.t_kv_pad * 64 * 4};
    const uint32_t boxv[3] = {32, 64, 1};
    const auto f = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = encode_tmap(&mkh, f, 3, sp.kh, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mkl, f, 3, sp.kl, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvh, f, 3, sp.vh, dv, sv, boxv, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvl, f, 3, sp.vl, dv, sv, boxv, sw)) != WATTN_OK) return rc;
  }
  tp.q = q;
  tp.q_rs = q_rs;
  tp.q_bs = q_bs;
  tp.qc = scale * 1.4426950408889634f;
  tp.o = o;
  tp.o_rs = o_rs;
  tp.o_bs = o_bs;
  tp.t_q = t_q;
  tp.t_kv = t_kv;
  tp.n_heads = n_heads;
  tp.n_qblk = pl.n_qblk;
  tp.causal = causal;
  tp.q_pos_offset = q_pos_offset;
  tp.n_splits = pl.n_splits;
  tp.split_tiles = pl.split_tiles;
  tp.cnt = sp.cnt;
  tp.status = device_status_ptr();
  if (tp.status == nullptr) return WATTN_ERR_CUDA;
  const int smem = (int)sizeof(TcSmem) + 1024;
  if (cudaFuncSetAttribute(attn_f32tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(attn_f32tc)");
  if (launch_pdl(attn_f32tc_kernel, dim3(pl.n_qblk * pl.n_splits, n_heads, batch),
                 dim3(kTcThreads), smem, stream, mkh, mkl, mvh, mvl, tp) != cudaSuccess)
    return check_launch("attn_f32tc (launch)");
  return check_launch("attn_f32tc");
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
