// decode.cu -- memory-bound split-KV decode attention.
//
// Replaces single_token_mha_d64 (crates/tensor/src/ops/attention.rs:246-434)
// for the decoder's cross-attention (decoder.rs:698, one query row per beam
// over the 1500 encoder states) and, over the paged cache, the causal
// self-attention of multi_head_attention_with_cache (decoder.rs:835-892).
//
// Structure (one CTA = 4 warps per (split of the keys, head, group of <= 8
// query rows)):
//   * thread 0 issues every TMA load of the split up front: 64-key K and V
//     sub-tiles, 128-byte swizzled, one mbarrier each, so all of a CTA's
//     bytes are in flight at once and two or three CTAs per SM keep HBM busy;
//   * scores: two lanes per key (32 dims each) against every query row of the
//     group, q pre-scaled by scale*log2(e) and broadcast from shared memory.
//     The query rows of one group share each K/V byte loaded (the beams of an
//     utterance share its cross-attention K/V), so the bytes per row fall
//     with the group size;
//   * exact softmax over the split (max, exp2, sum), then P V with each lane
//     owning two output dims;
//   * splits are merged by a log-sum-exp reduction done by the last CTA of
//     each (row group, head) to finish (a device counter in the workspace,
//     reset by that CTA), so there is no second kernel launch.
// The reference skips values whose probability is below 1e-7
// (attention.rs:366,425); this kernel does not (the skip changes a result by
// at most t_kv * 1e-7 * max|v|).

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <type_traits>

namespace wattn {

constexpr int kDecSub = 64;        // keys per sub-tile (TMA box rows)
constexpr int kDecRows = 8;        // query rows per CTA
constexpr int kDecThreads = 128;
constexpr int kDecMaxSubs = 4;     // sub-tiles per split (chunk <= 256 keys; 128 for f32)
constexpr int kPartStride = 66;    // floats per partial: acc[64], m, l
// Workspace layout, the same for every call: [counters][partials]. The
// counter region has a fixed size, so partials written by one call can never
// land where a later call of another shape keeps its counters; every call
// leaves the counters it used at zero.
constexpr size_t kCounterBytes = (size_t)kMaxSplitCounters * sizeof(int);
static_assert(kDecSub == kDecSubRows, "paged sub-tiles and TMA boxes must agree");

namespace {

template <int KV_DT> struct KvGeom {
  static constexpr int es = KV_DT == WATTN_F32 ? 4 : 2;
  static constexpr int blocks = (64 * es) / 128;   // 128-byte column blocks per row
  static constexpr int block_elems = 128 / es;     // elements per block row
  static constexpr int sub_bytes = kDecSub * 128 * blocks;
  static constexpr int max_subs = KV_DT == WATTN_F32 ? 2 : kDecMaxSubs;
};

struct DecParams {
  const void *q;
  void *o;
  int64_t q_rs, o_rs;
  int group_size, t_kv, n_heads;
  int row_chunks, n_splits, chunk;
  float scale_log2;
  float *part;   // [rows][n_heads][n_splits][kPartStride]
  int *count;    // [row groups][n_heads]
  int *status;
};

template <int KV_DT>
struct DecSmem {
  static constexpr int S = KvGeom<KV_DT>::max_subs;
  uint8_t k[S][KvGeom<KV_DT>::sub_bytes];
  uint8_t v[S][KvGeom<KV_DT>::sub_bytes];
  float q[kDecRows][64];
  float sc[kDecRows][S * kDecSub];
  float m[kDecRows], l[kDecRows];
  uint64_t kbar[S], vbar[S];
  int abort;
  int last;
};

// Shared memory of the tensor-core path: no score or query buffers (the
// scores stay in mma fragments), so three CTAs fit on an SM.
template <int KV_DT>
struct DecSmemMma {
  static constexpr int S = KvGeom<KV_DT>::max_subs;
  uint8_t k[S][KvGeom<KV_DT>::sub_bytes];
  uint8_t v[S][KvGeom<KV_DT>::sub_bytes];
  float m[kDecRows], l[kDecRows];
  float wm[4][kDecRows], wl[4][kDecRows];  // per-warp max / normaliser
  uint64_t kbar[S], vbar[S];
  int abort;
  int last;
};

// Warp-level tensor-core helpers (mma.sync m16n8k16, f32 accumulation).
template <typename T>
WATTN_DEVINL void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (sizeof(T) == 2 && __is_same(T, __nv_bfloat16)) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Four 8x8 16-bit matrices from shared memory; lane i addresses row i % 8 of
// matrix i / 8. The .trans form delivers them transposed.
WATTN_DEVINL void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
WATTN_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                            uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled tile.
WATTN_DEVINL int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Dot products of one key half-row (32 dims) with every query row.
template <int KV_DT>
WATTN_DEVINL void half_dots(const uint8_t *ktile, int krow, int half, const float (*q)[64],
                            int nr, float *dot) {
#pragma unroll
  for (int r = 0; r < kDecRows; ++r) dot[r] = 0.f;
  if constexpr (KV_DT == WATTN_F32) {
    const uint8_t *blk = ktile + half * (kDecSub * 128);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 kv = *reinterpret_cast<const float4 *>(blk + swz(krow, c));
      const int d = half * 32 + 4 * c;
#pragma unroll
      for (int r = 0; r < kDecRows; ++r) {
        if (r < nr) {
          const float4 qv = *reinterpret_cast<const float4 *>(&q[r][d]);
          dot[r] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, dot[r]))));
        }
      }
    }
  } else {
    using T = typename Elem<KV_DT>::T;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int c = half * 4 + cc;
      const uint4 w = *reinterpret_cast<const uint4 *>(ktile + swz(krow, c));
      const float2 k01 = unpack2<T>(w.x), k23 = unpack2<T>(w.y), k45 = unpack2<T>(w.z),
                   k67 = unpack2<T>(w.w);
      const int d = 8 * c;
#pragma unroll
      for (int r = 0; r < kDecRows; ++r) {
        if (r < nr) {
          const float4 qa = *reinterpret_cast<const float4 *>(&q[r][d]);
          const float4 qb = *reinterpret_cast<const float4 *>(&q[r][d + 4]);
          float acc = dot[r];
          acc = fmaf(qa.x, k01.x, acc);
          acc = fmaf(qa.y, k01.y, acc);
          acc = fmaf(qa.z, k23.x, acc);
          acc = fmaf(qa.w, k23.y, acc);
          acc = fmaf(qb.x, k45.x, acc);
          acc = fmaf(qb.y, k45.y, acc);
          acc = fmaf(qb.z, k67.x, acc);
          acc = fmaf(qb.w, k67.y, acc);
          dot[r] = acc;
        }
      }
    }
  }
}

// Two consecutive dims (2*lane, 2*lane+1) of value row `vrow` of a tile.
template <int KV_DT>
WATTN_DEVINL float2 value_pair(const uint8_t *vtile, int vrow, int lane) {
  if constexpr (KV_DT == WATTN_F32) {
    const uint8_t *blk = vtile + (lane >> 4) * (kDecSub * 128);
    const int d = (2 * lane) & 31;  // dim within the 32-float block row
    return *reinterpret_cast<const float2 *>(blk + swz(vrow, d >> 2) + (d & 3) * 4);
  } else {
    using T = typename Elem<KV_DT>::T;
    const uint32_t w =
        *reinterpret_cast<const uint32_t *>(vtile + swz(vrow, lane >> 2) + (lane & 3) * 4);
    return unpack2<T>(w);
  }
}

template <typename OutT>
WATTN_DEVINL void store_out(void *o, int64_t off, float x) {
  reinterpret_cast<OutT *>(o)[off] = from_f32<OutT>(x);
}

// Shared body. PAGED selects how a sub-tile's TMA coordinates are formed.
// Tensor-core path: 16-bit K/V with a query of the same type.
template <int Q_DT, int KV_DT>
constexpr bool kDecUseMma = KV_DT != WATTN_F32 && Q_DT == KV_DT;

template <int Q_DT, int KV_DT, int OUT_DT, bool PAGED>
__device__ void decode_body(const CUtensorMap &map_k, const CUtensorMap &map_v,
                            const DecParams &p, const PagedTable *pt) {
  using QT = typename Elem<Q_DT>::T;
  using OutT = typename Elem<OUT_DT>::T;
  using G = KvGeom<KV_DT>;
  constexpr bool kMma = kDecUseMma<Q_DT, KV_DT>;
  using SmemT = typename std::conditional<kMma, DecSmemMma<KV_DT>, DecSmem<KV_DT>>::type;
  extern __shared__ uint8_t dec_smem_raw[];
  SmemT &s = *reinterpret_cast<SmemT *>(
      (reinterpret_cast<uintptr_t>(dec_smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, head = blockIdx.y;

  // Rows of this CTA and the physical key range they attend.
  int row0, nr, kv_lo, kv_hi, group = 0, cnt_idx;
  if constexpr (PAGED) {
    row0 = blockIdx.z;
    nr = 1;
    kv_lo = pt->kv_lo[row0];
    kv_hi = pt->kv_hi[row0];
    cnt_idx = row0 * p.n_heads + head;
  } else {
    group = blockIdx.z / p.row_chunks;
    const int rc = blockIdx.z % p.row_chunks;
    row0 = group * p.group_size + rc * kDecRows;
    nr = min(kDecRows, p.group_size - rc * kDecRows);
    kv_lo = 0;
    kv_hi = p.t_kv;
    cnt_idx = blockIdx.z * p.n_heads + head;
  }
  const int base = kv_lo & ~(kDecSub - 1);                 // sub-tiles start on 64-row marks
  const int n_splits = (kv_hi - base + p.chunk - 1) / p.chunk;
  const int k_beg = base + split * p.chunk;
  if (k_beg >= kv_hi) return;                              // beyond this row's keys
  const int n_sub = min(p.chunk, kv_hi - k_beg + kDecSub - 1) / kDecSub;

  if (tid == 0) {
    for (int st = 0; st < n_sub; ++st) {
      mbar_init(&s.kbar[st], 1);
      mbar_init(&s.vbar[st], 1);
    }
    s.abort = 0;
    fence_barrier_init();
    for (int st = 0; st < n_sub; ++st) {
      const int key = k_beg + st * kDecSub;
      mbar_arrive_expect_tx(&s.kbar[st], G::sub_bytes);
      mbar_arrive_expect_tx(&s.vbar[st], G::sub_bytes);
      if constexpr (PAGED) {
        // Pool rows: (((page * n_layers + layer) * 2 + kv) * n_heads + head) * page_rows + r
        const int page = pt->pages[row0][key / pt->page_rows];
        const int r_in = key % pt->page_rows;
        const int64_t rk =
            ((((int64_t)page * pt->n_layers + pt->layer) * 2 + 0) * p.n_heads + head) *
                pt->page_rows + r_in;
        const int64_t rv = rk + (int64_t)p.n_heads * pt->page_rows;
#pragma unroll
        for (int bk = 0; bk < G::blocks; ++bk) {
          tma_load_2d(s.k[st] + bk * kDecSub * 128, &map_k, &s.kbar[st], bk * G::block_elems,
                      (int)rk);
          tma_load_2d(s.v[st] + bk * kDecSub * 128, &map_v, &s.vbar[st], bk * G::block_elems,
                      (int)rv);
        }
      } else {
#pragma unroll
        for (int bk = 0; bk < G::blocks; ++bk) {
          tma_load_4d(s.k[st] + bk * kDecSub * 128, &map_k, &s.kbar[st], bk * G::block_elems,
                      head, key, group);
          tma_load_4d(s.v[st] + bk * kDecSub * 128, &map_v, &s.vbar[st], bk * G::block_elems,
                      head, key, group);
        }
      }
    }
  }

  // Per-warp partial outputs, summed over the warps below, in the (now idle)
  // K buffer: [4 warps][kDecRows][64] floats.
  float *red = reinterpret_cast<float *>(&s.k[0][0]);
  if constexpr (kMma) {
    // ---- tensor-core path. Warp w takes keys 16w..16w+15 of every 64-key
    // sub-tile. S = Q K^T and O += P V with mma.sync m16n8k16 (rows = query
    // rows of the group, padded to 16; the scale is applied in f32 to S),
    // online softmax per row in the exp2 domain on the accumulator
    // fragments, then the four warps merge by log-sum-exp.
    const int g = lane >> 2, t4 = lane & 3;
    volatile int *abort = &s.abort;
    uint32_t qa[4][4];
    {
      const uint32_t *qrow = reinterpret_cast<const uint32_t *>(
          reinterpret_cast<const QT *>(p.q) + (int64_t)(row0 + g) * p.q_rs + head * 64);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = g < nr ? qrow[ks * 8 + t4] : 0u;
        qa[ks][2] = g < nr ? qrow[ks * 8 + 4 + t4] : 0u;
        qa[ks][1] = qa[ks][3] = 0u;  // rows 8..15 of the tile: beyond the 8 rows of a CTA
      }
    }
    const float c = p.scale_log2;
    float m_r = -INFINITY, l_r = 0.f;
    float acc[8][4];
#pragma unroll
    for (int db = 0; db < 8; ++db) acc[db][0] = acc[db][1] = acc[db][2] = acc[db][3] = 0.f;
    __syncthreads();  // barrier initialisation visible to every warp
    const int kb = warp * 16;
    for (int st = 0; st < n_sub; ++st) {
      mbar_wait(&s.kbar[st], 0, abort, p.status, (2 << 24) | (1 << 16) | (st << 8));
      const uint32_t ktile = smem_u32(s.k[st]), vtile = smem_u32(s.v[st]);
      float sc[2][4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
        const int key_row = kb + nb * 8 + (lane & 7);
#pragma unroll
        for (int ks2 = 0; ks2 < 2; ++ks2) {
          uint32_t r0, r1, r2, r3;
          const int chunk = 4 * ks2 + (lane >> 3);
          ldsm_x4(ktile + key_row * 128 + ((chunk ^ (key_row & 7)) << 4), r0, r1, r2, r3);
          mma16816<QT>(sc[nb], qa[2 * ks2], r0, r1);
          mma16816<QT>(sc[nb], qa[2 * ks2 + 1], r2, r3);
        }
      }
      // Mask keys outside [kv_lo, kv_hi) (row g holds keys 2*t4, 2*t4+1 of each 8).
      const int key0 = k_beg + st * kDecSub + kb + 2 * t4;
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + nb * 8 + e;
          if (key < kv_lo || key >= kv_hi) sc[nb][e] = -INFINITY;
        }
      float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mc = mx * c;
      if (mc > m_r + 8.0f) {  // lazy rescale, as in the encoder kernel
        const float alpha = ex2(m_r - mc);
        l_r *= alpha;
#pragma unroll
        for (int db = 0; db < 8; ++db) {
          acc[db][0] *= alpha;
          acc[db][1] *= alpha;
        }
        m_r = mc;
      }
      const float mu = (m_r == -INFINITY) ? 0.f : m_r;
      float pe[2][2];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) pe[nb][e] = ex2(fmaf(sc[nb][e], c, -mu));
      uint32_t pa[4];
      pa[0] = pack2<QT>(pe[0][0], pe[0][1]);
      pa[2] = pack2<QT>(pe[1][0], pe[1][1]);
      pa[1] = pa[3] = 0u;
      // Normalise by the rounded weights the tensor core uses.
      {
        const float2 r0 = unpack2<QT>(pa[0]), r2 = unpack2<QT>(pa[2]);
        l_r += (r0.x + r0.y) + (r2.x + r2.y);
      }
      mbar_wait(&s.vbar[st], 0, abort, p.status, (2 << 24) | (2 << 16) | (st << 8));
      {
        const int key_row = kb + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int db2 = 0; db2 < 4; ++db2) {
          uint32_t r0, r1, r2, r3;
          const int chunk = db2 * 2 + (lane >> 4);
          ldsm_x4_t(vtile + key_row * 128 + ((chunk ^ (key_row & 7)) << 4), r0, r1, r2, r3);
          mma16816<QT>(acc[2 * db2], pa, r0, r1);
          mma16816<QT>(acc[2 * db2 + 1], pa, r2, r3);
        }
      }
    }
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
    // Merge the four warps (log-sum-exp) into red / s.m / s.l.
    __syncthreads();  // every warp is done with K: `red` may overwrite it
    if (t4 == 0 && g < kDecRows) s.wm[warp][g] = m_r;
    __syncthreads();
    if (g < nr) {
      const float M = fmaxf(fmaxf(s.wm[0][g], s.wm[1][g]), fmaxf(s.wm[2][g], s.wm[3][g]));
      const float w = (m_r == -INFINITY) ? 0.f : ex2(m_r - M);
#pragma unroll
      for (int db = 0; db < 8; ++db)
        *reinterpret_cast<float2 *>(&red[(warp * kDecRows + g) * 64 + db * 8 + 2 * t4]) =
            make_float2(acc[db][0] * w, acc[db][1] * w);
      if (t4 == 0) {
        s.wl[warp][g] = l_r * w;
        if (warp == 0) s.m[g] = M;
      }
    }
    __syncthreads();
    if (tid < nr) s.l[tid] = s.wl[0][tid] + s.wl[1][tid] + s.wl[2][tid] + s.wl[3][tid];
    __syncthreads();
  } else {
  // Query rows, pre-scaled into the exp2 domain.
  for (int i = tid; i < kDecRows * 64; i += kDecThreads) {
    const int r = i >> 6, d = i & 63;
    float x = 0.f;
    if (r < nr)
      x = to_f32(reinterpret_cast<const QT *>(p.q)[(int64_t)(row0 + r) * p.q_rs + head * 64 + d]);
    s.q[r][d] = x * p.scale_log2;
  }
  __syncthreads();
  volatile int *abort = &s.abort;

  // ---- scores: warp w takes keys 16w.. of every sub-tile, two lanes per key
  const int krow = warp * 16 + (lane >> 1), half = lane & 1;
  for (int st = 0; st < n_sub; ++st) {
    mbar_wait(&s.kbar[st], 0, abort, p.status, (2 << 24) | (1 << 16) | (st << 8));
    float dot[kDecRows];
    half_dots<KV_DT>(s.k[st], krow, half, s.q, nr, dot);
    const int key = k_beg + st * kDecSub + krow;
    const bool valid = key >= kv_lo && key < kv_hi;
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) {
      const float full = dot[r] + __shfl_xor_sync(0xffffffffu, dot[r], 1);
      if (half == 0 && r < nr) s.sc[r][st * kDecSub + krow] = valid ? full : -INFINITY;
    }
  }
  __syncthreads();

  // ---- exact softmax over the split, one warp per row
  const int n_keys = n_sub * kDecSub;
  for (int r = warp; r < nr; r += 4) {
    float mx = -INFINITY;
    for (int j = lane; j < n_keys; j += 32) mx = fmaxf(mx, s.sc[r][j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < n_keys; j += 32) {
      const float pj = ex2(s.sc[r][j] - mx);
      s.sc[r][j] = pj;
      sum += pj;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      s.m[r] = mx;
      s.l[r] = sum;
    }
  }
  __syncthreads();

  // ---- P V: lane owns dims 2*lane, 2*lane+1; warp w takes keys 16w.. of every sub-tile
  float acc[kDecRows][2];
#pragma unroll
  for (int r = 0; r < kDecRows; ++r) acc[r][0] = acc[r][1] = 0.f;
  for (int st = 0; st < n_sub; ++st) {
    mbar_wait(&s.vbar[st], 0, abort, p.status, (2 << 24) | (2 << 16) | (st << 8));
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      const int vrow = warp * 16 + kk;
      const float2 vv = value_pair<KV_DT>(s.v[st], vrow, lane);
#pragma unroll
      for (int r = 0; r < kDecRows; ++r) {
        if (r < nr) {
          const float pj = s.sc[r][st * kDecSub + vrow];
          acc[r][0] = fmaf(pj, vv.x, acc[r][0]);
          acc[r][1] = fmaf(pj, vv.y, acc[r][1]);
        }
      }
    }
  }
  // Cross-warp sum through the (now idle) K buffer.
#pragma unroll
  for (int r = 0; r < kDecRows; ++r)
    if (r < nr) *reinterpret_cast<float2 *>(&red[(warp * kDecRows + r) * 64 + 2 * lane]) =
        make_float2(acc[r][0], acc[r][1]);
  __syncthreads();

  }

  const int64_t part_base = (int64_t)row0 * p.n_heads;  // row-major partial index base
  for (int i = tid; i < nr * 64; i += kDecThreads) {
    const int r = i >> 6, d = i & 63;
    const float a = red[(0 * kDecRows + r) * 64 + d] + red[(1 * kDecRows + r) * 64 + d] +
                    red[(2 * kDecRows + r) * 64 + d] + red[(3 * kDecRows + r) * 64 + d];
    if (n_splits == 1) {
      store_out<OutT>(p.o, (int64_t)(row0 + r) * p.o_rs + head * 64 + d, a / s.l[r]);
    } else {
      float *part = p.part + ((part_base + (int64_t)r * p.n_heads + head) * p.n_splits + split) *
                                 kPartStride;
      part[d] = a;
      if (d == 0) {
        part[64] = s.m[r];
        part[65] = s.l[r];
      }
    }
  }
  if (n_splits == 1) return;

  // ---- last CTA of this (row group, head) merges the splits (log-sum-exp)
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&p.count[cnt_idx], 1);
    s.last = (prev == n_splits - 1);
  }
  __syncthreads();
  if (!s.last) return;
  __threadfence();
  for (int i = tid; i < nr * 64; i += kDecThreads) {
    const int r = i >> 6, d = i & 63;
    const float *part0 =
        p.part + ((part_base + (int64_t)r * p.n_heads + head) * p.n_splits) * kPartStride;
    float M = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(part0 + sp * kPartStride + 64));
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const float w = ex2(__ldcg(part0 + sp * kPartStride + 64) - M);
      L = fmaf(w, __ldcg(part0 + sp * kPartStride + 65), L);
      O = fmaf(w, __ldcg(part0 + sp * kPartStride + d), O);
    }
    store_out<OutT>(p.o, (int64_t)(row0 + r) * p.o_rs + head * 64 + d, O / L);
  }
  if (tid == 0) p.count[cnt_idx] = 0;  // leave the workspace zeroed for the next call
}

template <int Q_DT, int KV_DT, int OUT_DT>
__global__ void __launch_bounds__(kDecThreads)
    decode_dense_kernel(const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const DecParams p) {
  decode_body<Q_DT, KV_DT, OUT_DT, false>(map_k, map_v, p, nullptr);
}

template <int Q_DT, int KV_DT, int OUT_DT>
__global__ void __launch_bounds__(kDecThreads)
    decode_paged_kernel(const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const DecParams p,
                        const __grid_constant__ PagedTable pt) {
  decode_body<Q_DT, KV_DT, OUT_DT, true>(map_k, map_v, p, &pt);
}

template <int Q_DT, int KV_DT> constexpr int dec_smem_bytes() {
  return (kDecUseMma<Q_DT, KV_DT> ? (int)sizeof(DecSmemMma<KV_DT>) : (int)sizeof(DecSmem<KV_DT>)) +
         1024;
}

template <typename K>
int set_smem(K kern, int bytes) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(decode)");
  return WATTN_OK;
}

template <int Q_DT, int KV_DT, int OUT_DT>
int launch_dense_typed(const CUtensorMap &mk, const CUtensorMap &mv, const DecParams &p,
                       int n_groups, cudaStream_t stream) {
  auto kern = decode_dense_kernel<Q_DT, KV_DT, OUT_DT>;
  const int smem = dec_smem_bytes<Q_DT, KV_DT>();
  int rc = set_smem(kern, smem);
  if (rc != WATTN_OK) return rc;
  dim3 grid(p.n_splits, p.n_heads, n_groups * p.row_chunks);
  kern<<<grid, kDecThreads, smem, stream>>>(mk, mv, p);
  return check_launch("decode_dense");
}

template <int Q_DT, int KV_DT, int OUT_DT>
int launch_paged_typed(const CUtensorMap &mk, const CUtensorMap &mv, const DecParams &p,
                       const PagedTable &pt, int max_splits, cudaStream_t stream) {
  auto kern = decode_paged_kernel<Q_DT, KV_DT, OUT_DT>;
  const int smem = dec_smem_bytes<Q_DT, KV_DT>();
  int rc = set_smem(kern, smem);
  if (rc != WATTN_OK) return rc;
  dim3 grid(max_splits, p.n_heads, pt.n_rows);
  kern<<<grid, kDecThreads, smem, stream>>>(mk, mv, p, pt);
  return check_launch("decode_paged");
}

// Dispatch over (q, kv, out) element types.
template <bool PAGED>
int dispatch(int q_dt, int kv_dt, int out_dt, const CUtensorMap &mk, const CUtensorMap &mv,
             const DecParams &p, int n_groups, const PagedTable *pt, int max_splits,
             cudaStream_t stream) {
#define WATTN_DEC_CASE(QD, KD, OD)                                                     \
  if (q_dt == QD && kv_dt == KD && out_dt == OD) {                                     \
    if constexpr (PAGED) return launch_paged_typed<QD, KD, OD>(mk, mv, p, *pt, max_splits, stream); \
    else return launch_dense_typed<QD, KD, OD>(mk, mv, p, n_groups, stream);          \
  }
#define WATTN_DEC_KV(QD, OD)              \
  WATTN_DEC_CASE(QD, WATTN_F32, OD)       \
  WATTN_DEC_CASE(QD, WATTN_F16, OD)       \
  WATTN_DEC_CASE(QD, WATTN_BF16, OD)
#define WATTN_DEC_OUT(QD)                 \
  WATTN_DEC_KV(QD, WATTN_F32)             \
  WATTN_DEC_KV(QD, WATTN_F16)             \
  WATTN_DEC_KV(QD, WATTN_BF16)
  WATTN_DEC_OUT(WATTN_F32)
  WATTN_DEC_OUT(WATTN_F16)
  WATTN_DEC_OUT(WATTN_BF16)
#undef WATTN_DEC_OUT
#undef WATTN_DEC_KV
#undef WATTN_DEC_CASE
  return set_error(WATTN_ERR_INVALID, "decode: unsupported dtype combination");
}

int chunk_for(int kv_dtype, int ctas_per_chunk_unit, int t_kv) {
  // Largest chunk (<= 256 keys, 128 for f32 K/V to fit shared memory) that
  // still gives >= ~4 waves of CTAs on 148 SMs.
  const int max_chunk = (kv_dtype == WATTN_F32 ? 2 : kDecMaxSubs) * kDecSub;
  int chunk = max_chunk;
  while (chunk > kDecSub) {
    const long long ctas = (long long)ctas_per_chunk_unit * ((t_kv + chunk - 1) / chunk);
    if (ctas >= 148LL * 2 * 4) break;
    chunk >>= 1;
  }
  return chunk;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

DecodePlan plan_decode(int n_groups, int group_size, int t_kv, int n_heads, int kv_dtype) {
  DecodePlan pl;
  pl.row_chunks = (group_size + kDecRows - 1) / kDecRows;
  pl.chunk = chunk_for(kv_dtype, n_groups * pl.row_chunks * n_heads, t_kv);
  pl.n_splits = t_kv > 0 ? (t_kv + pl.chunk - 1) / pl.chunk : 1;
  const size_t rows = (size_t)n_groups * group_size;
  pl.workspace_bytes = kCounterBytes + rows * n_heads * pl.n_splits * kPartStride * sizeof(float);
  return pl;
}

int launch_decode(const void *q, const void *k, const void *v, void *o, int q_dtype,
                  int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                  int n_heads, int64_t q_rs, int64_t kv_rs, int64_t kv_gs, int64_t o_rs,
                  float scale, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
  const DecodePlan pl = plan_decode(n_groups, group_size, t_kv, n_heads, kv_dtype);
  if (pl.n_splits > 1 && workspace_bytes < pl.workspace_bytes)
    return set_error(WATTN_ERR_INVALID, "decode: workspace of %zu bytes, %zu needed",
                     workspace_bytes, pl.workspace_bytes);
  if ((size_t)n_groups * pl.row_chunks * n_heads > (size_t)kMaxSplitCounters)
    return set_error(WATTN_ERR_INVALID, "decode: %d row groups x %d heads exceed %d per call",
                     n_groups * pl.row_chunks, n_heads, kMaxSplitCounters);
  const uint64_t es = elem_size(kv_dtype);
  const uint64_t dims[4] = {64, (uint64_t)n_heads, (uint64_t)t_kv, (uint64_t)n_groups};
  const uint64_t strides[3] = {64 * es, (uint64_t)kv_rs * es,
                               (uint64_t)(n_groups > 1 ? kv_gs : (int64_t)t_kv * kv_rs) * es};
  const uint32_t box[4] = {(uint32_t)(128 / es), 1, kDecSub, 1};
  CUtensorMap mk, mv;
  int rc = encode_tmap(&mk, tmap_dtype(kv_dtype), 4, k, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != WATTN_OK) return rc;
  rc = encode_tmap(&mv, tmap_dtype(kv_dtype), 4, v, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != WATTN_OK) return rc;
  DecParams p;
  p.q = q;
  p.o = o;
  p.q_rs = q_rs;
  p.o_rs = o_rs;
  p.group_size = group_size;
  p.t_kv = t_kv;
  p.n_heads = n_heads;
  p.row_chunks = pl.row_chunks;
  p.n_splits = pl.n_splits;
  p.chunk = pl.chunk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.count = reinterpret_cast<int *>(workspace);
  p.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(workspace) + kCounterBytes);
  p.status = device_status_ptr();
  if (p.status == nullptr) return WATTN_ERR_CUDA;
  return dispatch<false>(q_dtype, kv_dtype, out_dtype, mk, mv, p, n_groups, nullptr, 0, stream);
}

// Paged launch, used by the KV cache (kv_cache.cu).
int launch_decode_paged(const CUtensorMap &map_k, const CUtensorMap &map_v, const void *q,
                        void *o, int q_dtype, int kv_dtype, int out_dtype, int n_heads,
                        int64_t q_rs, int64_t o_rs, float scale, const PagedTable &pt,
                        int max_keys, void *workspace, size_t workspace_bytes,
                        cudaStream_t stream) {
  DecParams p;
  p.q = q;
  p.o = o;
  p.q_rs = q_rs;
  p.o_rs = o_rs;
  p.group_size = 1;
  p.t_kv = 0;
  p.n_heads = n_heads;
  p.row_chunks = 1;
  p.chunk = chunk_for(kv_dtype, pt.n_rows * n_heads, max_keys);
  p.n_splits = (max_keys + p.chunk - 1) / p.chunk;  // upper bound; rows use their own
  p.scale_log2 = scale * 1.4426950408889634f;
  const size_t need =
      kCounterBytes + (size_t)pt.n_rows * n_heads * p.n_splits * kPartStride * sizeof(float);
  if (need > paged_workspace_bytes(pt.n_rows, n_heads, max_keys))
    return set_error(WATTN_ERR_INVALID, "paged decode: internal workspace bound violated");
  if ((size_t)pt.n_rows * n_heads > (size_t)kMaxSplitCounters)
    return set_error(WATTN_ERR_INVALID, "paged decode: too many rows x heads per launch");
  if (workspace_bytes < need)
    return set_error(WATTN_ERR_INVALID, "paged decode: workspace of %zu bytes, %zu needed",
                     workspace_bytes, need);
  p.count = reinterpret_cast<int *>(workspace);
  p.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(workspace) + kCounterBytes);
  p.status = device_status_ptr();
  if (p.status == nullptr) return WATTN_ERR_CUDA;
  return dispatch<true>(q_dtype, kv_dtype, out_dtype, map_k, map_v, p, 0, &pt, p.n_splits,
                        stream);
}

size_t paged_workspace_bytes(int n_rows, int n_heads, int max_keys) {
  // Every chunk is at least one sub-tile, so splits <= ceil(max_keys / 64).
  const int n_splits = (max_keys + kDecSub - 1) / kDecSub;
  return kCounterBytes + (size_t)n_rows * n_heads * n_splits * kPartStride * sizeof(float);
}

}  // namespace wattn
