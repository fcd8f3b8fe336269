// attn_f32.cu -- f32 attention on the tensor cores (split-f16 products).
//
// The reference computes attention in f32 end to end (flash_attention_2,
// crates/tensor/src/ops/attention.rs:68-242, with matrixmultiply sgemm for
// both products) and its tests hold the result to 1e-5
// (crates/tensor/tests/test_flash_attention_tiled.rs:123-130). This path
// keeps f32 inputs, f32 softmax and f32 accumulators and computes both
// products on the tensor cores with the split-operand method of Ootomo and
// Yokota ("Recovering single precision accuracy from Tensor Cores while
// surpassing the FP32 theoretical peak performance", IJHPCA 2022), here in
// f16: every operand x (brought into f16's range by a power of two, below)
// is split into x_hi, x rounded to 11 significant bits, and x_lo = x - x_hi,
// both stored as f16, and each product a*b is computed as a_hi*b_lo +
// a_lo*b_hi + a_hi*b_hi with three tcgen05.mma of kind::f16 and f32
// accumulation. The dropped a_lo*b_lo and the 11 bits kept of each lo part
// leave about 2^-22 of relative error per product, the order of f32
// accumulation itself; f16 operands run at twice the rate of tf32 ones, and
// a K=16 step of f16 costs the tensor core what a K=8 step of tf32 does.
//
// Range: the exponent of an f16 spans 2^-14..2^15, so Q (times scale *
// log2 e), K and V are each scaled by a power of two that puts their
// largest magnitude in [2^13, 2^14) (the scale is undone exactly on the
// scores and on the output). Values far below a tensor's largest fall into
// f16's subnormals, where the split keeps an absolute error of at most
// 2^-25 of that scale: in the scores and the output these weigh 2^-39 of
// the largest term. The softmax weights p (<= 256 with the lazy rescale
// below) are split after a scale of 2^6 for the same reason.
//
// Three launches:
//  * f32_absmax_kernel: per-block maxima of |Q|, |K| and |V|.
//  * f32_split_kernel: the scales (from the block maxima), K as [bh][t][64]
//    and V transposed as [bh][64][t] (K-major over the keys, for the PV
//    product), each as a hi and a lo f16 array.
//  * attn_f32tc_kernel: one CTA per 128 query rows of one (utterance, head)
//    and run of 128-key tiles. Four softmax warps (one query row per
//    thread, the row's TMEM lane) load, scale and split their Q rows into
//    tensor memory, where they are the A operand of S = Q K^T; a TMA warp
//    streams the split K and V^T tiles through a 3-stage ring; an MMA warp
//    issues S for the next tile before PV of the current one. P is split
//    by the softmax warps into two double-buffered TMEM regions, so that
//    the softmax of tile j+1 overlaps PV of tile j. Tensor memory (512
//    columns, 16-bit operands two to a column): S [0,128), O [128,192),
//    Q_hi [192,224), Q_lo [224,256), P buffer b: hi [256+128b, 320+128b),
//    lo [320+128b, 384+128b).
//
// Small problems (few query blocks x heads for the SMs, e.g. Whisper-tiny's
// one utterance of 6 heads: 72 blocks) split the keys over a cluster of up
// to four CTAs per query block: each walks a run of key tiles, the others
// hand their unnormalised partial rows (64 sums, m, l) to the first through
// distributed shared memory, and it combines the parts by the
// online-softmax rule of attention.rs:173-201.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>
#include <climits>
#include <mutex>

namespace wattn {
namespace {

constexpr int kTcRows = 128;    // query rows per CTA (UMMA M)
constexpr int kTcKeys = 128;    // keys per tile (UMMA N of S, K of PV)
constexpr int kTcStages = 3;    // K / V^T ring
// Softmax warps 0-7 (warp w: TMEM lane quarter w % 4, key half w / 4),
// TMA warp 8, MMA warps 9 (scores) and 10 (PV).
constexpr int kTcSoftmaxThreads = 256;
constexpr int kTcThreads = 11 * 32;
constexpr int kTcTmaWarp = 8, kTcMmaWarp = 9, kTcPvWarp = 10;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 128, kColQh = 192, kColQl = 224, kColP = 256;
constexpr int kMaxSplits = 4;       // cluster size limit of the key splits
constexpr int kPartFloats = 68;     // a partial row in the landing area: 64 sums, m, l, pad
constexpr float kPScaleLog2 = 6.f;  // softmax weights are split as p * 2^6

// x rounded to 11 significant bits (to nearest, ties away from zero) with
// integer operations, for finite x below 2^127: the hi part of the split,
// exact in f16 wherever f16 holds x's exponent.
WATTN_DEVINL float round11(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

// (hi, lo) of the split of two values, packed two f16 to a word (the first
// value in the low half).
WATTN_DEVINL void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
  const float ha = round11(a), hb = round11(b);
  hi = pack2<__half>(ha, hb);
  lo = pack2<__half>(a - ha, b - hb);
}

// The split of two non-negative values (the softmax weights) with the hi
// part truncated to 11 significant bits: one logic operation each instead
// of a rounding add and mask (the ALU pipe limits the softmax). lo = x - hi
// is exact and below 2^-10 x; its f16 keeps 11 bits of it, 2^-21 of x.
WATTN_DEVINL void split2_trunc(float a, float b, uint32_t &hi, uint32_t &lo) {
  const float ha = __uint_as_float(__float_as_uint(a) & 0xffffe000u),
              hb = __uint_as_float(__float_as_uint(b) & 0xffffe000u);
  hi = pack2<__half>(ha, hb);
  lo = pack2<__half>(a - ha, b - hb);
}

// The power of two 2^e that puts a largest magnitude mx in [2^13, 2^14)
// (1 for 0, infinities and NaN, which then propagate as f32 would).
WATTN_DEVINL int range_exp(float mx) {
  if (!(mx > 0.f) || !(mx < INFINITY)) return 0;
  int e;
  frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
  return 14 - e;
}

// ------------------------------------------------------------ pre-pass
// One block per (utterance x head, 128-key tile, K or V): the tile's
// largest magnitude sets its range exponent (written for the attention
// kernel), then the tile goes out split: K as [bh][t][64] rows, V
// transposed through shared memory as [bh][64][t_kv_pad] rows.
struct PrepParams {
  const float *k, *v;
  int64_t kv_rs, kv_bs;
  int n_heads, t_kv, t_kv_pad, n_kv_tiles;
  __half *kh, *kl, *vh, *vl;
  int *ek, *ev;  // [bh][n_kv_tiles] range exponents of the K and V tiles
  const float *q;  // Q rows, prefetched into L2 for the attention kernel
  int64_t q_rs, q_bs;
  int t_q;
};

WATTN_DEVINL float absmax4(float4 x, float m) {
  return fmaxf(fmaxf(m, fmaxf(fabsf(x.x), fabsf(x.y))), fmaxf(fabsf(x.z), fabsf(x.w)));
}

// 2^e as a float, e clamped to [-100, 100] (a tile whose largest magnitude
// is below 2^-86 keeps part of f16's range unused; all of it is then far
// below anything the tolerance can see).
WATTN_DEVINL float pow2(int e) { return __int_as_float((127 + max(-100, min(100, e))) << 23); }

// Range exponent of a largest magnitude, clamped to pow2's range.
WATTN_DEVINL int range_exp_c(float mx) { return max(-100, min(100, range_exp(mx))); }

// Largest of v over the block (256 threads); red is 8 floats of shared memory.
WATTN_DEVINL float block_max256(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  return m;
}

__global__ void __launch_bounds__(256) f32_split_kernel(const PrepParams p) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ float red[8];
  __shared__ __half tv[2][64][kTcKeys + 8];  // V^T tile, hi and lo ([dim][key], padded rows)
  {
    // Q's 128-byte lines into L2: every attention CTA starts by reading its
    // Q rows, a latency each would otherwise wait out on DRAM.
    const int lines_per_row = p.n_heads * 2;
    const long long n_lines = (long long)(gridDim.x / (2 * p.n_kv_tiles) / p.n_heads) * p.t_q *
                              lines_per_row;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n_lines; i += gridDim.x * 256LL) {
      const long long row = i / lines_per_row;
      const int bq = (int)(row / p.t_q), t = (int)(row - (long long)bq * p.t_q);
      const float *line = p.q + bq * p.q_bs + (int64_t)t * p.q_rs + (i - row * lines_per_row) * 32;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
  }
  const int tile = blockIdx.x % p.n_kv_tiles;
  const bool is_v = (blockIdx.x / p.n_kv_tiles) & 1;
  const long long bh = (long long)blockIdx.x / (2LL * p.n_kv_tiles);
  const int b = (int)(bh / p.n_heads), h = (int)(bh - (long long)b * p.n_heads);
  const int key0 = tile * kTcKeys, nk = min(kTcKeys, p.t_kv - key0);
  const float *src = (is_v ? p.v : p.k) + b * p.kv_bs + h * kHeadDim;
  // thread t: float4 column c4 = t % 16 of rows t / 16 + 16 i
  const int c4 = threadIdx.x & 15, r0 = threadIdx.x >> 4;
  float4 x[8];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + 16 * i;
    x[i] = r < nk ? __ldg(reinterpret_cast<const float4 *>(src + (int64_t)(key0 + r) * p.kv_rs) + c4)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    mx = absmax4(x[i], mx);
  }
  const int e = range_exp_c(block_max256(mx, red));
  if (threadIdx.x == 0) (is_v ? p.ev : p.ek)[bh * p.n_kv_tiles + tile] = e;
  const float f = pow2(e);
  if (!is_v) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + 16 * i;
      if (r >= nk) continue;
      uint2 hi, lo;
      split2(x[i].x * f, x[i].y * f, hi.x, lo.x);
      split2(x[i].z * f, x[i].w * f, hi.y, lo.y);
      const int64_t off = (bh * p.t_kv + key0 + r) * kHeadDim + 4 * c4;
      *reinterpret_cast<uint2 *>(p.kh + off) = hi;
      *reinterpret_cast<uint2 *>(p.kl + off) = lo;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + 16 * i;
    const float xv[4] = {x[i].x * f, x[i].y * f, x[i].z * f, x[i].w * f};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float hv = round11(xv[q]);
      tv[0][4 * c4 + q][r] = __float2half_rn(hv);
      tv[1][4 * c4 + q][r] = __float2half_rn(xv[q] - hv);
    }
  }
  __syncthreads();
  // rows of V^T: 64 dims x 16 chunks of 8 keys, for hi and lo
  for (int i = threadIdx.x; i < 2 * 64 * 16; i += 256) {
    const int part = i >> 10, d = (i >> 4) & 63, ch = i & 15;
    if (8 * ch >= nk) continue;  // the chunk's keys lie within t_kv_pad
    const uint4 w = *reinterpret_cast<const uint4 *>(&tv[part][d][8 * ch]);
    *reinterpret_cast<uint4 *>((part ? p.vl : p.vh) + (bh * kHeadDim + d) * p.t_kv_pad + key0 +
                               8 * ch) = w;
  }
}

// ------------------------------------------------------------ attention
struct TcParams {
  const float *q;  // raw Q rows (the softmax warps scale and split them)
  int64_t q_rs, q_bs;
  float qc;        // scale * log2(e)
  float *o;
  int64_t o_rs, o_bs;
  int t_q, t_kv, n_heads;
  int causal, q_pos_offset;
  int n_splits, split_tiles;  // key splits (cluster size) per query block, key tiles per split
  const int *ek, *ev;         // [bh][n_kv_tiles] range exponents of the K and V tiles
  int n_kv_tiles;
  int *status;
};

struct TcSmem {
  // K tiles: [key][64 dims] rows of 128 bytes; V^T tiles: two 64-key
  // halves of [dim][64 keys] rows of 128 bytes. After the main loop the
  // ring is the landing area of the other splits' partial rows.
  __half kh[kTcStages][kTcKeys * 64], kl[kTcStages][kTcKeys * 64];
  __half vh[kTcStages][2][64 * 64], vl[kTcStages][2][64 * 64];
  uint64_t kv_full[kTcStages], kv_empty[kTcStages];
  uint64_t q_full, s_full, s_free, p_full[2], pv_done[2], drain;
  uint64_t land;  // the first CTA of a cluster: the other splits' partial rows have landed
  float xmax[2][2][kTcRows];  // [tile parity][key half][row]: the halves' row maxima
  float xsum[2][kTcRows];     // [key half][row]: the halves' row sums, at the end
  float xq[8];                // the softmax warps' largest |Q * qc|
  uint32_t tmem_base;
  int abort;
};
// After the main loop the ring holds, from its start, the landing area of
// the other splits' partial rows ([split - 1][row][kPartFloats] floats; a
// CTA other than the first stages its own there) and, at kStageOffset, the
// output tile for the TMA store ([half][row][32 floats], 128-byte swizzle).
constexpr uint32_t kPartBytes = kTcRows * kPartFloats * sizeof(float);
constexpr uint32_t kStageOffset = 112 * 1024;
static_assert((kMaxSplits - 1) * kPartBytes <= kStageOffset, "landing area below the output tile");
static_assert(kStageOffset + 2 * kTcRows * 32 * sizeof(float) <=
                  sizeof(TcSmem::kh) + sizeof(TcSmem::kl) + sizeof(TcSmem::vh) + sizeof(TcSmem::vl),
              "output tile inside the ring");

// Wait sites (kernel 3): role << 16 | barrier << 8 | iteration.
#define TF_SITE(role, bar, j) ((3 << 24) | ((role) << 16) | ((bar) << 8) | ((j) & 0xff))

// Barrier of the 256 softmax threads (named barrier 1), returning whether
// `pred` held in all of them.
WATTN_DEVINL bool softmax_sync_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

WATTN_DEVINL void tma_store_3d(const CUtensorMap *map, const void *src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// `bytes` of this CTA's shared memory at src to the cluster shared-memory
// address dst (another CTA's), completing on the mbarrier at cluster
// address bar.
WATTN_DEVINL void bulk_copy_to_cluster(uint32_t dst, const void *src, uint32_t bytes,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst),
      "r"(smem_u32(src)), "r"(bytes), "r"(bar)
      : "memory");
}

WATTN_DEVINL void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
WATTN_DEVINL uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attn_f32tc_kernel(const __grid_constant__ CUtensorMap map_kh,
                      const __grid_constant__ CUtensorMap map_kl,
                      const __grid_constant__ CUtensorMap map_vh,
                      const __grid_constant__ CUtensorMap map_vl,
                      const __grid_constant__ CUtensorMap map_o, const TcParams p) {
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
    mbar_init(&s.q_full, kTcSoftmaxThreads);
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_free, kTcSoftmaxThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.p_full[i], kTcSoftmaxThreads);
      mbar_init(&s.pv_done[i], 1);
    }
    mbar_init(&s.drain, 2);
    mbar_init(&s.land, 1);
    s.abort = 0;
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
  // The softmax threads' results (row m and l, the half's 32 output
  // columns), read by the split merge below.
  const int quarter = warp & 3, half = (warp >> 2) & 1;
  const int row = quarter * 32 + lane, qrow = q0 + row;
  float m = -INFINITY, l = 0.f;
  int ev_min = 100;  // O is accumulated at the scale 2^ev_min (below)
  bool have = false;
  uint32_t o[32];

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
        mbar_arrive_expect_tx(&s.kv_full[st], (uint32_t)(sizeof(s.kh[0]) * 2 + sizeof(s.vh[0]) * 2));
        tma_load_3d(s.kh[st], &map_kh, &s.kv_full[st], 0, key0, bh);
        tma_load_3d(s.kl[st], &map_kl, &s.kv_full[st], 0, key0, bh);
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_3d(s.vh[st][hf], &map_vh, &s.kv_full[st], key0 + 64 * hf, 0, bh);
          tma_load_3d(s.vl[st][hf], &map_vl, &s.kv_full[st], key0 + 64 * hf, 0, bh);
        }
        last = j;
      }
      if (*abort && last >= 0) {
        // let the loads in flight land before the shared memory is reused
        volatile int no_abort = 0;
        mbar_wait(&s.kv_full[last % kTcStages], (last / kTcStages) & 1, &no_abort, p.status,
                  TF_SITE(1, 3, last));
      }
    }
  } else if (warp == kTcMmaWarp || warp == kTcPvWarp) {
    // ---------------------------------------------------------- MMA issuers
    // Two threads issue the products, warp 9 the scores S(j) and warp 10
    // the PV(j) products, side by side: one thread issuing both took 75-85
    // cycles per instruction beside the softmax warps, above the tensor
    // core's own time for these shapes. Each thread's commits track its own
    // products; PV(j) needs P(j), so S(j) is complete when PV(j) is issued,
    // and PV(j)'s commit also frees the stage for the TMA warp.
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_f16(0, kTcRows, kTcKeys, 0, 0);  // M=128, N=128 keys
      constexpr uint32_t idesc_o = idesc_f16(0, kTcRows, 64, 0, 0);       // M=128, N=64 dims
      const uint32_t t_s = tmem + kColS, t_o = tmem + kColO, t_qh = tmem + kColQh,
                     t_ql = tmem + kColQl;
      // K-major SW128 B operands, rows of 128 bytes (64 f16), 8-row atoms of
      // 1024 bytes. K: a K=16 step (32 bytes) is +2 in the descriptor's
      // address field (16-byte units), 4 steps per row. V^T: 8 steps over the
      // 128 keys, 4 in each 64-key half. A operands (Q, P) are TMEM rows, two
      // f16 to a column, 8 columns per step. Descriptors are made once and
      // moved by adding to the address field.
      constexpr uint32_t kStage16 = sizeof(s.kh[0]) >> 4, kHalf16 = sizeof(s.vh[0][0]) >> 4;
      static_assert(sizeof(s.kh[0]) == sizeof(s.vh[0]), "stage strides");
      if (warp == kTcMmaWarp) {
        const uint64_t d_kh = smem_desc_sw128(smem_u32(s.kh[0]), 16, 1024),
                       d_kl = smem_desc_sw128(smem_u32(s.kl[0]), 16, 1024);
        bool ok = mbar_wait(&s.q_full, 0, abort, p.status, TF_SITE(2, 0, 0));
        if (ok) tc_fence_after();
        // S = Q_hi K_lo + Q_lo K_hi + Q_hi K_hi: the two small products
        // first, into an empty accumulator, then the large one (on the tf32
        // form of this kernel that order measured 2.6e-6 max-abs error on
        // config 1 against 3.6e-6 the other way round); the same for PV.
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int st = j % kTcStages;
          const uint64_t kh = d_kh + st * kStage16, kl = d_kl + st * kStage16;
          if (!mbar_wait(&s.kv_full[st], (j / kTcStages) & 1, abort, p.status, TF_SITE(2, 1, j)))
            break;
          // S(j) overwrites S(j-1): the softmax must have read it
          if (j > 0 && !mbar_wait(&s.s_free, (j - 1) & 1, abort, p.status, TF_SITE(2, 2, j)))
            break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(t_s, t_qh + 8 * kk, kl + 2 * kk, idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_ts(t_s, t_ql + 8 * kk, kh + 2 * kk, idesc_s, 1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_ts(t_s, t_qh + 8 * kk, kh + 2 * kk, idesc_s, 1);
          umma_commit(&s.s_full);
        }
      } else {
        const uint64_t d_vh = smem_desc_sw128(smem_u32(s.vh[0][0]), 16, 1024),
                       d_vl = smem_desc_sw128(smem_u32(s.vl[0][0]), 16, 1024);
        auto vstep = [](uint64_t d, int kk) -> uint64_t {
          return d + (kk < 4 ? 0u : kHalf16) + 2 * (kk & 3);
        };
        for (int j = 0; j < n_tiles; ++j) {
          const int st = j % kTcStages, pb = j & 1;
          const uint64_t vh = d_vh + st * kStage16, vl = d_vl + st * kStage16;
          if (!mbar_wait(&s.p_full[pb], (j >> 1) & 1, abort, p.status, TF_SITE(2, 3, j))) break;
          tc_fence_after();
          // O += P_hi V_lo + P_lo V_hi + P_hi V_hi
          const uint32_t t_ph = tmem + kColP + 128 * pb, t_pl = t_ph + 64;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ts(t_o, t_ph + 8 * kk, vstep(vl, kk), idesc_o, j > 0 || kk > 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_ts(t_o, t_pl + 8 * kk, vstep(vh, kk), idesc_o, 1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_ts(t_o, t_ph + 8 * kk, vstep(vh, kk), idesc_o, 1);
          umma_commit(&s.pv_done[pb]);
          umma_commit(&s.kv_empty[st]);
        }
      }
      // both issuers' products complete before TMEM is freed
      volatile int no_abort = 0;
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0, &no_abort, p.status, TF_SITE(2, 4, 0));
    }
  } else {
    // ---------------------------------------------------------- softmax
    // Thread = query row (its TMEM lane) x key half: warps w and w + 4 share
    // the rows of lane quarter w and take keys 0-63 and 64-127 of each tile,
    // so that two softmax warps share each scheduler (one per scheduler was
    // latency-bound at ~25 cycles per key). The halves trade row maxima
    // through shared memory at a barrier of the 256 softmax threads per
    // tile; the barrier also ANDs every thread's wait results, so that the
    // threads leave the loop together and none waits at a barrier alone.
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t t_s = lane_base + kColS + 64 * half, t_o = lane_base + kColO + 32 * half;
    // Range exponents: e_q of this CTA's Q rows (every CTA of a cluster
    // has the same rows), the key tiles' from the pre-pass. V's tiles come
    // with their own exponents e_v(t); P is weighted by 2^(ev_min - e_v(t))
    // so that one accumulator holds every tile at the scale 2^ev_min.
    int e_q;
    {
      const int tile0 = kv_beg / kTcKeys;
      const int *ev = p.ev + (int64_t)bh * p.n_kv_tiles + tile0;
      for (int i = lane; i < n_tiles; i += 32) ev_min = min(ev_min, __ldg(ev + i));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ev_min = min(ev_min, __shfl_xor_sync(0xffffffffu, ev_min, o));
    }
    const int *ek_row = p.ek + (int64_t)bh * p.n_kv_tiles + kv_beg / kTcKeys;
    const int *ev_row = p.ev + (int64_t)bh * p.n_kv_tiles + kv_beg / kTcKeys;
    {
      // this half's 32 dims of the Q row (rows past t_q are zeros), times
      // scale * log2 e, scaled into f16's range and split
      const float *src = p.q + (int64_t)b * p.q_bs + (int64_t)qrow * p.q_rs + head * kHeadDim +
                         32 * half;
      const bool in = qrow < p.t_q;
      float4 x[8];
      float mq = 0.f;
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        x[e4] = in ? __ldg(reinterpret_cast<const float4 *>(src + 4 * e4))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
        x[e4] = make_float4(x[e4].x * p.qc, x[e4].y * p.qc, x[e4].z * p.qc, x[e4].w * p.qc);
        mq = absmax4(x[e4], mq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      if (lane == 0) s.xq[warp] = mq;
      softmax_sync_and(true);
#pragma unroll
      for (int w = 0; w < 8; ++w) mq = fmaxf(mq, s.xq[w]);
      e_q = range_exp_c(mq);
      const float fq = pow2(e_q);
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        split2(x[e4].x * fq, x[e4].y * fq, hi[2 * e4], lo[2 * e4]);
        split2(x[e4].z * fq, x[e4].w * fq, hi[2 * e4 + 1], lo[2 * e4 + 1]);
      }
      tmem_st16(lane_base + kColQh + 16 * half, hi);
      tmem_st16(lane_base + kColQl + 16 * half, lo);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&s.q_full);
    }
    const int lim_row = p.causal ? min(p.t_kv, qrow + p.q_pos_offset + 1) : p.t_kv;
    bool ok = true;
    int ek_next = n_tiles > 0 ? __ldg(ek_row) : 0, ev_next = n_tiles > 0 ? __ldg(ev_row) : 0;
    for (int j = 0; j < n_tiles; ++j) {
      const int pb = j & 1;
      const int ek_j = ek_next, ev_j = ev_next;
      if (j + 1 < n_tiles) {
        ek_next = __ldg(ek_row + j + 1);
        ev_next = __ldg(ev_row + j + 1);
      }
      // scores in the exp2 domain: acc * 2^-(e_q + e_k(j)), at least 2^-126
      // (only scores below 2^-92 differ, all of which weigh 1), so that a
      // masked -inf stays -inf
      const float fs = fmaxf(pow2(-e_q) * pow2(-ek_j), 0x1p-126f);
      bool got = ok && mbar_wait(&s.s_full, j & 1, abort, p.status, TF_SITE(3, 0, j));
      got = __all_sync(0xffffffffu, got);
      uint32_t r[2][32];
      float mxh = -INFINITY;
      // visible keys of this half-tile
      const int lim = lim_row - (kv_beg + j * kTcKeys) - 64 * half;
      if (got) {
        tc_fence_after();
        tmem_ld32(t_s, r[0]);
        tmem_ld32(t_s + 32, r[1]);
        tmem_wait_ld();
        reg_fence(r[0]);
        reg_fence(r[1]);
        tc_fence_before();
        mbar_arrive(&s.s_free);
        // keys past the row's visible ones become -inf (weight 0); only
        // partial tiles (the last, causal rows) pay for the selects
        if (__any_sync(0xffffffffu, lim < 64)) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= lim) r[i >> 5][i & 31] = __float_as_uint(-INFINITY);
        }
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 64; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(r[i >> 5][i & 31]));
        mxh = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      s.xmax[pb][half][row] = mxh;
      if (!softmax_sync_and(got)) {
        ok = false;
        break;
      }
      float mx = fmaxf(mxh, s.xmax[pb][half ^ 1][row]);
      if (mx != -INFINITY) mx *= fs;
      // Lazy rescale (the online softmax of attention.rs:173-201, with the
      // offset moved only when the max grows by more than 2^8: p then stays
      // <= 256 and the result is exact either way). Both halves of a row
      // take the same steps.
      const bool need = mx > m + 8.f;
      const bool warp_need = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2(m - mx) : 1.f;  // 0 on the first tile (m = -inf)
      if (need) {
        l *= alpha;
        m = mx;
      }
      // p * 2^6 * 2^(ev_min - e_v(j)) = exp2(acc * fs + 6 + ev_min - e_v(j) - m)
      const float bias =
          kPScaleLog2 + (float)(ev_min - ev_j) - (m == -INFINITY ? 0.f : m);
      // P buffer pb is free once PV(j-2) is complete.
      bool fine = true;
      if (j >= 2) {
        fine = mbar_wait(&s.pv_done[pb], ((j >> 1) - 1) & 1, abort, p.status, TF_SITE(3, 1, j));
        fine = __all_sync(0xffffffffu, fine);
        if (fine) tc_fence_after();
      }
      if (fine) {
        const uint32_t t_ph = lane_base + kColP + 128 * pb + 32 * half, t_pl = t_ph + 64;
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2) {
            const float p0 = ex2(fmaf(__uint_as_float(r[c][2 * i2]), fs, bias));
            const float p1 = ex2(fmaf(__uint_as_float(r[c][2 * i2 + 1]), fs, bias));
            sum4[i2 & 3] += p0 + p1;
            split2_trunc(p0, p1, hi[i2], lo[i2]);
          }
          tmem_st16(t_ph + 16 * c, hi);
          tmem_st16(t_pl + 16 * c, lo);
        }
        // l sums p * 2^6 (the V weight taken back out)
        l += ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3])) * pow2(ev_j - ev_min);
        // O (this half's 32 columns) is rescaled once PV(j-1) is complete.
        if (j > 0 && warp_need) {
          fine = mbar_wait(&s.pv_done[pb ^ 1], ((j - 1) >> 1) & 1, abort, p.status,
                           TF_SITE(3, 2, j));
          fine = __all_sync(0xffffffffu, fine);
          if (fine) {
            tc_fence_after();
            uint32_t ov[32];
            tmem_ld32(t_o, ov);
            tmem_wait_ld();
            reg_fence(ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st32(t_o, ov);
          }
        }
        tmem_wait_st();
      }
      if (!fine) ok = false;  // the next tile's barrier ends the loop for all
      tc_fence_before();
      mbar_arrive(&s.p_full[pb]);
    }
    bool fin = ok && n_tiles > 0 &&
               mbar_wait(&s.pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, abort,
                         p.status, TF_SITE(3, 3, n_tiles));
    fin = __all_sync(0xffffffffu, fin);
    if (fin) {
      tc_fence_after();
      tmem_ld32(t_o, o);
      tmem_wait_ld();
      reg_fence(o);
    }
    // the row's l: the two halves' sums
    s.xsum[half][row] = l;
    have = softmax_sync_and(fin);
    l += s.xsum[half ^ 1][row];
  }

  // ------------------------------------------------------------ epilogue
  // The output tile goes out through the TMA (rows past t_q are not
  // written): each softmax thread puts its half-row into the swizzled
  // staging tile, then one thread stores the two 32-column halves. Every
  // softmax thread takes the named barriers, whatever its state.
  uint8_t *ring = reinterpret_cast<uint8_t *>(&s.kh[0][0]);
  float *land = reinterpret_cast<float *>(ring);
  auto store_out = [&](const float (&v)[32], bool valid) {
    if (valid) {
      uint8_t *tile = ring + kStageOffset + half * (kTcRows * 128) + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4 *>(tile + ((c ^ (row & 7)) << 4)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
    fence_proxy_async_smem();
    const bool any = softmax_sync_and(!valid) == false;  // some thread has a row to write
    if (threadIdx.x == 0 && any) {
      for (int h = 0; h < 2; ++h)
        tma_store_3d(&map_o, ring + kStageOffset + h * (kTcRows * 128), head * kHeadDim + 32 * h,
                     q0, b);
      bulk_commit_group();
      bulk_wait_read_all();
    }
  };
  if (p.n_splits == 1) {
    if (warp < kTcTmaWarp) {
      // O = O' 2^-e_v / l (l sums the same p * 2^6 that O' does)
      const float inv = l > 0.f ? pow2(-ev_min) / l : 0.f;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
      store_out(v, have);
    }
  } else {
    // Key splits: the CTAs of a query block form a cluster. After the first
    // cluster barrier every CTA is past its main loop (loads landed,
    // products done), so the rings are free: each CTA but the first stages
    // its partial rows (sums, m, l; l = 0 for a row without a result) in
    // its own ring and sends them with one bulk copy to the first CTA's
    // landing area, which counts the bytes on its `land` barrier. The
    // second cluster barrier holds the senders until the first CTA has
    // everything. Every thread of every CTA takes both barriers.
    if (split == 0 && threadIdx.x == 0)
      mbar_arrive_expect_tx(&s.land, (uint32_t)(p.n_splits - 1) * kPartBytes);
    __syncwarp();
    cluster_sync_all();
    if (split > 0 && warp < kTcTmaWarp) {
      // the sums at their true scale (each split has its own ev_min)
      float *mine = land + row * kPartFloats;
      const float sc = pow2(-ev_min);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4 *>(mine + 32 * half + 4 * c) =
            make_float4(__uint_as_float(o[4 * c]) * sc, __uint_as_float(o[4 * c + 1]) * sc,
                        __uint_as_float(o[4 * c + 2]) * sc, __uint_as_float(o[4 * c + 3]) * sc);
      if (half == 0) *reinterpret_cast<float4 *>(mine + 64) = make_float4(m, have ? l : 0.f, 0.f, 0.f);
      fence_proxy_async_smem();
      softmax_sync_and(true);
      if (threadIdx.x == 0)
        bulk_copy_to_cluster(cluster_map(smem_u32(ring + (split - 1) * kPartBytes), 0), ring,
                             kPartBytes, cluster_map(smem_u32(&s.land), 0));
    }
    bool landed = true;
    if (split == 0 && warp < kTcTmaWarp) {
      landed = mbar_wait(&s.land, 0, abort, p.status, TF_SITE(3, 4, 0));
      landed = softmax_sync_and(landed);
    }
    __syncwarp();
    cluster_sync_all();
    if (split == 0 && warp < kTcTmaWarp) {
      float mx = l > 0.f ? m : -INFINITY;
      for (int sp = 1; sp < p.n_splits; ++sp) {
        const float *ps = land + ((sp - 1) * kTcRows + row) * kPartFloats;
        if (ps[65] > 0.f) mx = fmaxf(mx, ps[64]);
      }
      const float w0 = l > 0.f ? ex2(m - mx) : 0.f;
      const float w0s = w0 * pow2(-ev_min);
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(o[i]) * w0s;
      float lt = l * w0;
      for (int sp = 1; sp < p.n_splits; ++sp) {
        const float *ps = land + ((sp - 1) * kTcRows + row) * kPartFloats;
        const float pl = ps[65];
        if (!(pl > 0.f)) continue;
        const float w = ex2(ps[64] - mx);
        lt = fmaf(w, pl, lt);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 x = *reinterpret_cast<const float4 *>(ps + 32 * half + 4 * c);
          acc[4 * c] = fmaf(w, x.x, acc[4 * c]);
          acc[4 * c + 1] = fmaf(w, x.y, acc[4 * c + 1]);
          acc[4 * c + 2] = fmaf(w, x.z, acc[4 * c + 2]);
          acc[4 * c + 3] = fmaf(w, x.w, acc[4 * c + 3]);
        }
      }
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] *= inv;
      store_out(acc, have && landed);
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

constexpr int kPlanDevices = 64;

// Clusters of n CTAs of the attention kernel that fit on the device at once
// (one CTA per SM; a cluster's CTAs share a GPC), per device, measured once.
int max_clusters(int n, int dev) {
  static std::mutex mu;
  static int cache[kPlanDevices][kMaxSplits + 1];
  static bool done[kPlanDevices][kMaxSplits + 1];
  if (dev < 0 || dev >= kPlanDevices || n < 1 || n > kMaxSplits) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (!done[dev][n]) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n, 1, 1);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = sizeof(TcSmem) + 1024;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaFuncSetAttribute(attn_f32tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)cfg.dynamicSmemBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&c, attn_f32tc_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    cache[dev][n] = c;
    done[dev][n] = true;
  }
  return cache[dev][n];
}

// Launch plan of one call. Workspace: [counter region (left to the other
// kernels)][K tile exponents][V tile exponents][K hi, lo][V^T hi, lo].
struct F32Plan {
  int n_qblk, n_splits, split_tiles, t_kv_pad, n_kv_tiles;
  size_t eb, kb, vb, total;
};

F32Plan plan_f32(int batch, int t_q, int t_kv, int n_heads, int causal, int n_sm, int dev,
                 bool clusters) {
  F32Plan pl;
  const long long bh = (long long)batch * n_heads;
  pl.n_qblk = (t_q + kTcRows - 1) / kTcRows;
  const int kv_tiles = (t_kv + kTcKeys - 1) / kTcKeys;
  const long long base = (long long)pl.n_qblk * bh;
  // Key splits while the query blocks leave SMs idle (one CTA per SM by
  // shared memory and tensor memory), at least two key tiles per split and
  // at most kMaxSplits; all clusters must fit on the device at once.
  // Causal calls are not split.
  int n_splits = 1;
  if (!causal && base < n_sm)
    n_splits = (int)std::min<long long>(std::min<long long>(n_sm / base, kv_tiles / 2), kMaxSplits);
  n_splits = std::max(n_splits, 1);
  if (clusters)
    while (n_splits > 1 && base > max_clusters(n_splits, dev)) --n_splits;
  pl.split_tiles = (kv_tiles + n_splits - 1) / n_splits;
  pl.n_splits = std::max(1, (kv_tiles + pl.split_tiles - 1) / pl.split_tiles);
  pl.t_kv_pad = (t_kv + 7) & ~7;  // V^T rows: 16-byte multiples
  pl.n_kv_tiles = kv_tiles;
  pl.eb = round_up_256((size_t)bh * kv_tiles * sizeof(int));
  pl.kb = round_up_256((size_t)bh * t_kv * kHeadDim * 2);
  pl.vb = round_up_256((size_t)bh * kHeadDim * pl.t_kv_pad * 2);
  pl.total = kCounterBytes + 2 * pl.eb + 2 * pl.kb + 2 * pl.vb;
  return pl;
}

}  // namespace

size_t attn_f32_workspace_bytes(int batch, int t_q, int t_kv, int n_heads, int n_sm) {
  return plan_f32(batch, t_q, t_kv, n_heads, 0, n_sm, 0, false).total;
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
  const F32Plan pl = plan_f32(batch, t_q, t_kv, n_heads, causal, n_sm, dev, true);
  if ((long long)pl.n_qblk * pl.n_splits > INT_MAX || batch > 65535 || n_heads > 65535)
    return set_error(WATTN_ERR_INVALID, "attention: too many rows");
  if (ws != nullptr && ws_bytes < pl.total)
    return set_error(WATTN_ERR_INVALID,
                     "attention: a workspace of %zu bytes is needed for f32 inputs (%zu given)",
                     pl.total, ws_bytes);
  uint8_t *wsb = reinterpret_cast<uint8_t *>(ws != nullptr ? ws : thread_workspace(pl.total, stream));
  if (wsb == nullptr) return set_error(WATTN_ERR_NOMEM, "attention workspace allocation failed");
  uint8_t *cur = wsb + kCounterBytes;
  PrepParams pp;
  pp.k = k;
  pp.v = v;
  pp.kv_rs = kv_rs;
  pp.kv_bs = kv_bs;
  pp.n_heads = n_heads;
  pp.t_kv = t_kv;
  pp.t_kv_pad = pl.t_kv_pad;
  pp.n_kv_tiles = pl.n_kv_tiles;
  pp.q = q;
  pp.q_rs = q_rs;
  pp.q_bs = q_bs;
  pp.t_q = t_q;
  pp.ek = reinterpret_cast<int *>(cur);
  pp.ev = reinterpret_cast<int *>(cur + pl.eb);
  cur += 2 * pl.eb;
  pp.kh = reinterpret_cast<__half *>(cur);
  pp.kl = reinterpret_cast<__half *>(cur + pl.kb);
  pp.vh = reinterpret_cast<__half *>(cur + 2 * pl.kb);
  pp.vl = reinterpret_cast<__half *>(cur + 2 * pl.kb + pl.vb);
  const long long split_blocks = bh * 2 * pl.n_kv_tiles;
  if (split_blocks > INT_MAX) return set_error(WATTN_ERR_INVALID, "attention: too many key tiles");
  if (launch_pdl(f32_split_kernel, dim3((unsigned)split_blocks), dim3(256), 0, stream, pp) !=
      cudaSuccess)
    return check_launch("f32_split (launch)");
  // Tensor maps: K as [bh][t][64] f16 (boxes of 64 values x 128 keys), V^T
  // as [bh][64][t_kv] f16 (boxes of 64 keys x 64 dims); rows past the
  // extents read as zero.
  CUtensorMap mkh, mkl, mvh, mvl, mo;
  int rc;
  {
    const uint64_t dk[3] = {64, (uint64_t)t_kv, (uint64_t)bh};
    const uint64_t sk[2] = {64 * 2, (uint64_t)t_kv * 64 * 2};
    const uint32_t boxk[3] = {64, (uint32_t)kTcKeys, 1};
    const uint64_t dv[3] = {(uint64_t)t_kv, 64, (uint64_t)bh};
    const uint64_t sv[2] = {(uint64_t)pl.t_kv_pad * 2, (uint64_t)pl.t_kv_pad * 64 * 2};
    const uint32_t boxv[3] = {64, 64, 1};
    const auto f = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = encode_tmap(&mkh, f, 3, pp.kh, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mkl, f, 3, pp.kl, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvh, f, 3, pp.vh, dv, sv, boxv, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvl, f, 3, pp.vl, dv, sv, boxv, sw)) != WATTN_OK) return rc;
    // the output: [batch][t_q][n_heads * 64] f32, stored in 32-column halves
    const uint64_t dout[3] = {(uint64_t)n_heads * 64, (uint64_t)t_q, (uint64_t)batch};
    const uint64_t sout[2] = {(uint64_t)o_rs * 4,
                              (uint64_t)(batch > 1 ? o_bs : (int64_t)t_q * o_rs) * 4};
    const uint32_t boxo[3] = {32, (uint32_t)kTcRows, 1};
    if ((rc = encode_tmap(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, o, dout, sout, boxo, sw)) !=
        WATTN_OK)
      return rc;
  }
  TcParams tp;
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
  tp.causal = causal;
  tp.q_pos_offset = q_pos_offset;
  tp.n_splits = pl.n_splits;
  tp.split_tiles = pl.split_tiles;
  tp.ek = pp.ek;
  tp.ev = pp.ev;
  tp.n_kv_tiles = pl.n_kv_tiles;
  tp.status = device_status_ptr();
  if (tp.status == nullptr) return WATTN_ERR_CUDA;
  const int smem = (int)sizeof(TcSmem) + 1024;
  if (cudaFuncSetAttribute(attn_f32tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(attn_f32tc)");
  const dim3 grid(pl.n_qblk * pl.n_splits, n_heads, batch);
  const cudaError_t e =
      pl.n_splits > 1
          ? launch_pdl_cluster(attn_f32tc_kernel, grid, dim3(kTcThreads), smem, stream,
                               (unsigned)pl.n_splits, mkh, mkl, mvh, mvl, mo, tp)
          : launch_pdl(attn_f32tc_kernel, grid, dim3(kTcThreads), smem, stream, mkh, mkl, mvh,
                       mvl, mo, tp);
  if (e != cudaSuccess) return check_launch("attn_f32tc (launch)");
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
