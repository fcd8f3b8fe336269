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
// Range: the exponent of an f16 spans 2^-14..2^15, so each 128-key tile of
// K and of V, and each 128-row block of Q (times scale * log2 e), is scaled
// by a power of two that puts its largest magnitude in [2^13, 2^14); the
// scales are undone exactly on the scores and, through the weights, on the
// output. Values far below a tile's largest fall into f16's subnormals,
// where the split keeps an absolute error of at most 2^-25 of that scale:
// in the scores and the output these weigh 2^-39 of the largest term. The
// softmax weights p (<= 256 with the lazy rescale below) are split after a
// scale of 2^6 for the same reason.
//
// Two launches:
//  * f32_split_kernel: per 128-key tile of K and of V, the range exponent
//    and the tile split into [bh][t][64] rows of hi and lo f16; per 128-row
//    query block, Q's range exponent.
//  * attn_f32tc_kernel: one CTA per 128 query rows of one (utterance, head)
//    and run of 128-key tiles. Eight softmax warps (a query row per TMEM
//    lane, a key half per warp) load, scale and split their Q rows into
//    tensor memory, where they are the A operand of S = Q K^T; a TMA warp
//    streams the split K and V tiles through a 3-stage ring; one MMA warp
//    issues the S products and another the PV products (V as an MN-major
//    operand). P is split by the softmax warps into two double-buffered
//    TMEM regions, so that the softmax of tile j+1 overlaps PV of tile j.
//    Tensor memory (512 columns, 16-bit operands two to a column): S
//    [0,128), O [128,192), Q_hi [192,224), Q_lo [224,256), P buffer b: hi
//    [256+128b, 320+128b), lo [320+128b, 384+128b).
//
// Small problems (few query blocks x heads for the SMs, e.g. Whisper-tiny's
// one utterance of 6 heads: 72 blocks) split the keys over a cluster of up
// to three CTAs per query block: each walks a run of key tiles, then each
// lane quarter of rows is merged by one of the CTAs, which receives the
// others' unnormalised partial rows (32 sums per half, m, l) through
// distributed shared memory and combines them by the online-softmax rule
// of attention.rs:173-201.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>
#include <climits>
#include <mutex>

namespace wattn {
namespace {

constexpr int kTcRows = 128;    // query rows per CTA (UMMA M)
constexpr int kTcKeys = 128;    // keys per tile (UMMA N of S, K of PV)
constexpr int kTcStages = 3;    // K / V ring
// Softmax warps 0-7 (warp w: TMEM lane quarter w % 4, key half w / 4),
// TMA warp 8, MMA warps 9 (scores) and 10 (PV).
constexpr int kTcSoftmaxThreads = 256;
constexpr int kTcThreads = 11 * 32;
constexpr int kTcTmaWarp = 8, kTcMmaWarp = 9, kTcPvWarp = 10;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 128, kColQh = 192, kColQl = 224, kColP = 256;
constexpr int kMaxSplits = 3;       // cluster size limit of the key splits
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
// kernel), then the tile goes out split as [bh][t][64] rows of hi and lo
// f16 (K and V alike; PV reads V's tiles as an MN-major operand). Then one
// block per (utterance x head, 128-row query block): Q's range exponent.
struct PrepParams {
  const float *k, *v;
  int64_t kv_rs, kv_bs;
  int n_heads, t_kv, n_kv_tiles;
  __half *kh, *kl, *vh, *vl;
  int *ek, *ev;  // [bh][n_kv_tiles] range exponents of the K and V tiles
  const float *q;  // Q rows: the range exponent per 128-row block
  int64_t q_rs, q_bs;
  int t_q, n_qblk;
  long long bh;    // utterances x heads
  float qc;        // scale * log2(e)
  int *eq;         // [bh][n_qblk] range exponents of |Q * qc|
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
  // thread t: float4 column c4 = t % 16 of rows t / 16 + 16 i
  const int c4 = threadIdx.x & 15, r0 = threadIdx.x >> 4;
  const long long n_kv_blocks = (long long)p.bh * 2 * p.n_kv_tiles;
  if (blockIdx.x >= n_kv_blocks) {
    // A 128-row query block of one head: the range exponent of its
    // |Q * scale * log2 e| (the attention kernel splits Q itself), and its
    // rows pulled into L2 on the way.
    const long long qb = blockIdx.x - n_kv_blocks, bh = qb / p.n_qblk;
    const int qblk = (int)(qb - bh * p.n_qblk);
    const int b = (int)(bh / p.n_heads), h = (int)(bh - (long long)b * p.n_heads);
    const int row0 = qblk * kTcRows, nr = min(kTcRows, p.t_q - row0);
    const float *src = p.q + b * p.q_bs + h * kHeadDim;
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + 16 * i;
      if (r < nr)
        mx = absmax4(__ldg(reinterpret_cast<const float4 *>(src + (int64_t)(row0 + r) * p.q_rs) + c4),
                     mx);
    }
    const int e = range_exp_c(block_max256(mx, red) * p.qc);
    if (threadIdx.x == 0) p.eq[bh * p.n_qblk + qblk] = e;
    return;
  }
  const int tile = blockIdx.x % p.n_kv_tiles;
  const bool is_v = (blockIdx.x / p.n_kv_tiles) & 1;
  const long long bh = (long long)blockIdx.x / (2LL * p.n_kv_tiles);
  const int b = (int)(bh / p.n_heads), h = (int)(bh - (long long)b * p.n_heads);
  const int key0 = tile * kTcKeys, nk = min(kTcKeys, p.t_kv - key0);
  const float *src = (is_v ? p.v : p.k) + b * p.kv_bs + h * kHeadDim;
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
  __half *dh = is_v ? p.vh : p.kh, *dl = is_v ? p.vl : p.kl;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + 16 * i;
    if (r >= nk) continue;
    uint2 hi, lo;
    split2(x[i].x * f, x[i].y * f, hi.x, lo.x);
    split2(x[i].z * f, x[i].w * f, hi.y, lo.y);
    const int64_t off = (bh * p.t_kv + key0 + r) * kHeadDim + 4 * c4;
    *reinterpret_cast<uint2 *>(dh + off) = hi;
    *reinterpret_cast<uint2 *>(dl + off) = lo;
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
  const int *eq;              // [bh][n_qblk] range exponents of the query blocks
  int n_kv_tiles, n_qblk;
  int *status;
};

struct TcSmem {
  // K and V tiles: [key][64 dims] rows of 128 bytes (128-byte swizzle).
  __half kh[kTcStages][kTcKeys * 64], kl[kTcStages][kTcKeys * 64];
  __half vh[kTcStages][kTcKeys * 64], vl[kTcStages][kTcKeys * 64];
  uint64_t kv_full[kTcStages], kv_empty[kTcStages];
  uint64_t q_full, s_full, s_free, p_full[2], pv_done[2], drain;
  uint64_t land;  // the first CTA of a cluster: the other splits' partial rows have landed
  float xmax[2][2][kTcRows];  // [tile parity][key half][row]: the halves' row maxima
  float xsum[2][kTcRows];     // [key half][row]: the halves' row sums, at the end
  uint32_t tmem_base;
  int abort;
};
// After the main loop the ring holds, from its start, the partial rows of
// the key splits ([split][row][kPartFloats] floats: a CTA stages its own in
// its slot and receives the others' in theirs) and, at kStageOffset, the
// output tile for the TMA stores ([half][lane quarter][32 rows][32 floats],
// 128-byte swizzle).
constexpr uint32_t kRowBytes = kPartFloats * sizeof(float);
constexpr uint32_t kPartBytes = kTcRows * kRowBytes;
constexpr uint32_t kStageOffset = 112 * 1024;
static_assert(kMaxSplits * kPartBytes <= kStageOffset, "partial rows below the output tile");
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

// Barrier of the two softmax warps that share lane quarter q (named barrier
// 2 + q, 64 threads), returning whether `pred` held in both.
WATTN_DEVINL bool pair_sync_and(bool pred, int q) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(2 + q)
      : "memory");
  return r != 0;
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
  // The softmax threads' Q half-rows are read before the dependency wait:
  // the pre-pass does not write Q, and every kernel ahead of it in the
  // stream has completed when this grid's CTAs start (the pre-pass waits
  // for them before it lets this grid launch), so the load's latency hides
  // behind the set-up and the wait.
  const int quarter = warp & 3, half = (warp >> 2) & 1;
  const int row = quarter * 32 + lane, qrow = q0 + row;
  float4 x[8];
  if (warp < kTcTmaWarp) {
    const float *src = p.q + (int64_t)b * p.q_bs + (int64_t)qrow * p.q_rs + head * kHeadDim +
                       32 * half;
    const bool q_in = qrow < p.t_q;
#pragma unroll
    for (int e4 = 0; e4 < 8; ++e4)
      x[e4] = q_in ? __ldg(reinterpret_cast<const float4 *>(src + 4 * e4))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
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
        tma_load_3d(s.vh[st], &map_vh, &s.kv_full[st], 0, key0, bh);
        tma_load_3d(s.vl[st], &map_vl, &s.kv_full[st], 0, key0, bh);
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
      // PV: V's tile is [key][dim], so B is MN-major (the dims contiguous)
      constexpr uint32_t idesc_o = idesc_f16(0, kTcRows, 64, 0, 1);       // M=128, N=64 dims
      const uint32_t t_s = tmem + kColS, t_o = tmem + kColO, t_qh = tmem + kColQh,
                     t_ql = tmem + kColQl;
      // SW128 B operands, rows of 128 bytes (64 f16), 8-row atoms of 1024
      // bytes. K (K-major): a K=16 step (32 bytes) is +2 in the
      // descriptor's address field (16-byte units), 4 steps per row. V
      // (MN-major, one 64-dim column of atoms): a K=16 step is 16 key rows,
      // +128. A operands (Q, P) are TMEM rows, two f16 to a column, 8
      // columns per step. Descriptors are made once and moved by adding to
      // the address field.
      constexpr uint32_t kStage16 = sizeof(s.kh[0]) >> 4;
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
        const uint64_t d_vh = smem_desc_sw128(smem_u32(s.vh[0]), 16384, 1024),
                       d_vl = smem_desc_sw128(smem_u32(s.vl[0]), 16384, 1024);
        auto vstep = [](uint64_t d, int kk) -> uint64_t { return d + 128 * kk; };
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
    // latency-bound at ~25 cycles per key). The two warps of a quarter trade
    // row maxima through shared memory at a barrier of their own per tile;
    // the barrier also ANDs their wait results, so that they leave the loop
    // together and neither waits at a barrier alone (the other pairs learn
    // of a failed wait through the abort flag, at their next wait).
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t t_s = lane_base + kColS + 64 * half, t_o = lane_base + kColO + 32 * half;
    // Range exponents from the pre-pass: e_q of this query block (every CTA
    // of a cluster has the same rows) and the key tiles'. V's tiles come
    // with their own exponents e_v(t); P is weighted by 2^(ev_min - e_v(t))
    // so that one accumulator holds every tile at the scale 2^ev_min.
    const int *ek_row = p.ek + (int64_t)bh * p.n_kv_tiles + kv_beg / kTcKeys;
    const int *ev_row = p.ev + (int64_t)bh * p.n_kv_tiles + kv_beg / kTcKeys;
    const int e_q = __ldg(p.eq + (int64_t)bh * p.n_qblk + qblk);
    for (int i = lane; i < n_tiles; i += 32) ev_min = min(ev_min, __ldg(ev_row + i));
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1)
      ev_min = min(ev_min, __shfl_xor_sync(0xffffffffu, ev_min, sh));
    {
      // this half's 32 dims of the Q row (rows past t_q are zeros), times
      // scale * log2 e, scaled into f16's range and split
      const float fq = p.qc * pow2(e_q);
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
        for (int i = 0; i < 64; i += 8)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mx4[k] = fmax3(mx4[k], __uint_as_float(r[(i + 2 * k) >> 5][(i + 2 * k) & 31]),
                           __uint_as_float(r[(i + 2 * k + 1) >> 5][(i + 2 * k + 1) & 31]));
        mxh = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      s.xmax[pb][half][row] = mxh;
      if (!pair_sync_and(got, quarter)) {
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
  // Each softmax warp stores its own 32 rows x 32 columns through the TMA
  // (rows past t_q are not written): the lanes put their half-rows into the
  // warp's swizzled staging box, then lane 0 issues the store.
  uint8_t *ring = reinterpret_cast<uint8_t *>(&s.kh[0][0]);
  auto store_out = [&](const float (&v)[32]) {
    uint8_t *box = ring + kStageOffset + (half * 4 + quarter) * (32 * 128);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4 *>(box + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(&map_o, box, head * kHeadDim + 32 * half, q0 + 32 * quarter, b);
      bulk_commit_group();
      bulk_wait_read_all();
    }
  };
  if (p.n_splits == 1) {
    if (warp < kTcTmaWarp && have) {
      // O = O' 2^-e_v / l (l sums the same p * 2^6 that O' does)
      const float inv = l > 0.f ? pow2(-ev_min) / l : 0.f;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
      store_out(v);
    }
  } else {
    // Key splits: the CTAs of a query block form a cluster, and each lane
    // quarter of rows is merged by one of them (owner(q) = q * S / 4), so
    // the merges and the stores are shared out. After the first cluster
    // barrier every CTA is past its main loop (loads landed, products
    // done) and its ring is free: each stages the partial rows (sums at
    // their true scale, m, l; l = 0 for a row without a result) of the
    // quarters it does not own in its own slot and sends each quarter's 32
    // rows with one bulk copy into the owner's ring, same slot, counted on
    // the owner's `land` barrier. The second cluster barrier holds every
    // CTA until all of them have what they merge. Every thread of every
    // CTA takes both barriers.
    const int S = p.n_splits;
    const int owner = quarter * S / 4;
    if (threadIdx.x == 0) {
      uint32_t owned = 0;
      for (int q = 0; q < 4; ++q) owned += (q * S / 4 == split) ? 32u : 0u;
      mbar_arrive_expect_tx(&s.land, (uint32_t)(S - 1) * owned * kRowBytes);
    }
    // This CTA's own ring is free once its last products are done (have:
    // every softmax thread saw them), so its outgoing rows are staged before
    // the cluster barrier, which also orders the staging for the copies.
    if (warp < kTcTmaWarp && owner != split && have) {
      float *mine = reinterpret_cast<float *>(ring + split * kPartBytes) + row * kPartFloats;
      const float sc = pow2(-ev_min);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4 *>(mine + 32 * half + 4 * c) =
            make_float4(__uint_as_float(o[4 * c]) * sc, __uint_as_float(o[4 * c + 1]) * sc,
                        __uint_as_float(o[4 * c + 2]) * sc, __uint_as_float(o[4 * c + 3]) * sc);
      if (half == 0) *reinterpret_cast<float4 *>(mine + 64) = make_float4(m, l, 0.f, 0.f);
      fence_proxy_async_smem();
    }
    __syncwarp();
    cluster_sync_all();
    bool landed = true;
    if (warp < kTcTmaWarp) {
      if (owner != split) {
        if (!have && half == 0) {
          // no result (a wait gave up): the rows go out marked empty, l = 0
          float *mine = reinterpret_cast<float *>(ring + split * kPartBytes) + row * kPartFloats;
          *reinterpret_cast<float4 *>(mine + 64) = make_float4(m, 0.f, 0.f, 0.f);
          fence_proxy_async_smem();
        }
        if (!have) pair_sync_and(true, quarter);
        if (half == 0 && lane == 0) {
          const uint32_t off = split * kPartBytes + quarter * 32 * kRowBytes;
          bulk_copy_to_cluster(cluster_map(smem_u32(ring + off), owner), ring + off,
                               32 * kRowBytes, cluster_map(smem_u32(&s.land), owner));
        }
      } else {
        landed = mbar_wait(&s.land, 0, abort, p.status, TF_SITE(3, 4, 0));
        landed = __all_sync(0xffffffffu, landed);
        if (landed && have) {
          float mx = l > 0.f ? m : -INFINITY;
          for (int sp = 0; sp < S; ++sp) {
            if (sp == split) continue;
            const float *ps = reinterpret_cast<const float *>(ring + sp * kPartBytes) + row * kPartFloats;
            if (ps[65] > 0.f) mx = fmaxf(mx, ps[64]);
          }
          const float w0 = l > 0.f ? ex2(m - mx) : 0.f;
          const float w0s = w0 * pow2(-ev_min);
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(o[i]) * w0s;
          float lt = l * w0;
          for (int sp = 0; sp < S; ++sp) {
            if (sp == split) continue;
            const float *ps = reinterpret_cast<const float *>(ring + sp * kPartBytes) + row * kPartFloats;
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
          store_out(acc);
        }
      }
    }
    __syncwarp();
    cluster_sync_all();
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
// kernels)][K tile exponents][V tile exponents][Q block exponents][K hi,
// lo][V hi, lo].
struct F32Plan {
  int n_qblk, n_splits, split_tiles, n_kv_tiles;
  size_t eb, qeb, kb, vb, total;
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
  pl.n_kv_tiles = kv_tiles;
  pl.eb = round_up_256((size_t)bh * kv_tiles * sizeof(int));
  pl.qeb = round_up_256((size_t)bh * pl.n_qblk * sizeof(int));
  pl.kb = round_up_256((size_t)bh * t_kv * kHeadDim * 2);
  pl.vb = pl.kb;
  pl.total = kCounterBytes + 2 * pl.eb + pl.qeb + 2 * pl.kb + 2 * pl.vb;
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
  pp.n_kv_tiles = pl.n_kv_tiles;
  pp.q = q;
  pp.q_rs = q_rs;
  pp.q_bs = q_bs;
  pp.t_q = t_q;
  pp.n_qblk = pl.n_qblk;
  pp.bh = bh;
  pp.qc = scale * 1.4426950408889634f;
  pp.ek = reinterpret_cast<int *>(cur);
  pp.ev = reinterpret_cast<int *>(cur + pl.eb);
  pp.eq = reinterpret_cast<int *>(cur + 2 * pl.eb);
  cur += 2 * pl.eb + pl.qeb;
  pp.kh = reinterpret_cast<__half *>(cur);
  pp.kl = reinterpret_cast<__half *>(cur + pl.kb);
  pp.vh = reinterpret_cast<__half *>(cur + 2 * pl.kb);
  pp.vl = reinterpret_cast<__half *>(cur + 2 * pl.kb + pl.vb);
  // Tensor maps: K and V as [bh][t][64] f16 (boxes of 64 values x 128
  // keys); rows past the extents read as zero.
  CUtensorMap mkh, mkl, mvh, mvl, mo;
  int rc;
  {
    const uint64_t dk[3] = {64, (uint64_t)t_kv, (uint64_t)bh};
    const uint64_t sk[2] = {64 * 2, (uint64_t)t_kv * 64 * 2};
    const uint32_t boxk[3] = {64, (uint32_t)kTcKeys, 1};
    const auto f = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = encode_tmap(&mkh, f, 3, pp.kh, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mkl, f, 3, pp.kl, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvh, f, 3, pp.vh, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    if ((rc = encode_tmap(&mvl, f, 3, pp.vl, dk, sk, boxk, sw)) != WATTN_OK) return rc;
    // the output: [batch][t_q][n_heads * 64] f32, stored in boxes of 32 rows
    // x 32 columns
    const uint64_t dout[3] = {(uint64_t)n_heads * 64, (uint64_t)t_q, (uint64_t)batch};
    const uint64_t sout[2] = {(uint64_t)o_rs * 4,
                              (uint64_t)(batch > 1 ? o_bs : (int64_t)t_q * o_rs) * 4};
    const uint32_t boxo[3] = {32, 32, 1};  // one softmax warp's rows and half
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
  tp.eq = pp.eq;
  tp.n_kv_tiles = pl.n_kv_tiles;
  tp.n_qblk = pl.n_qblk;
  tp.status = device_status_ptr();
  if (tp.status == nullptr) return WATTN_ERR_CUDA;
  const int smem = (int)sizeof(TcSmem) + 1024;
  if (cudaFuncSetAttribute(attn_f32tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(attn_f32tc)");
  // Everything the host prepares (tensor maps, attributes) is ready before
  // the first launch, so that the two launches go out back to back and the
  // attention grid is queued while the pre-pass runs.
  const long long split_blocks = bh * (2LL * pl.n_kv_tiles + pl.n_qblk);
  if (split_blocks > INT_MAX) return set_error(WATTN_ERR_INVALID, "attention: too many key tiles");
  if (launch_pdl(f32_split_kernel, dim3((unsigned)split_blocks), dim3(256), 0, stream, pp) !=
      cudaSuccess)
    return check_launch("f32_split (launch)");
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
