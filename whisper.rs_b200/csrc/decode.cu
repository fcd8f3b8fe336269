// decode.cu -- memory-bound split-KV decode attention.
//
// Replaces single_token_mha_d64 (crates/tensor/src/ops/attention.rs:246-434)
// for the decoder's cross-attention (decoder.rs:698, one query row per beam
// over the 1500 encoder states) and, over the paged cache, the causal
// self-attention of multi_head_attention_with_cache (decoder.rs:835-892).
//
// One CTA serves (a split of the keys, a head, a group of <= 8 query rows).
// The query rows of one group share every K/V byte loaded (the beams of an
// utterance share its cross-attention K/V), so the bytes per row fall with
// the group size. K/V arrive as 64-key sub-tiles by TMA, 128-byte swizzled
// (on the streaming path, a dense item's partial last sub-tile by cp.async
// copies of the producer warp instead: copy_partial_sub).
//
// Tensor-core path (16-bit K/V and a query of the same type), a streaming
// kernel: a producer warp keeps a ring of kStrStages sub-tiles full while
// four compute warps consume it, so each CTA has up to four sub-tiles (64 KB)
// in flight for its whole life. Splits are few and long (about three waves of
// CTAs over the GPU): S = Q K^T and O += P V run on mma.sync m16n8k16 with an
// online softmax on the accumulator fragments; the four warps merge by
// log-sum-exp.
//
// CUDA-core path (f32 K/V, or a query type other than the K/V type): thread 0
// issues every load of a short split up front; two lanes per key form the
// scores, an exact softmax over the split follows, then P V with each lane
// owning two output dims.
//
// Either way, splits of one (row group, head) are merged by a log-sum-exp
// reduction in the last CTA to finish (a device counter in the workspace,
// reset by that CTA), so there is no second kernel launch.
// The reference skips values whose probability is below 1e-7
// (attention.rs:366,425); these kernels do not (the skip changes a result by
// at most t_kv * 1e-7 * max|v|).

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>

namespace wattn {

constexpr int kDecSub = 64;        // keys per sub-tile (TMA box rows)
constexpr int kDecRows = 8;        // query rows per CTA
constexpr int kDecThreads = 128;   // CUDA-core path
constexpr int kDecMaxSubs = 4;     // CUDA-core path: sub-tiles per split (chunk <= 256 keys; 128 for f32)
constexpr int kPartStride = 66;    // floats per partial: acc[64], m, l
constexpr int kCapMaxHeads = 64;   // heads an alignment-head capture can select from
constexpr int kStrStages = 4;      // tensor-core path: depth of the K/V ring (sub-tiles)
constexpr int kStrWarps = 4;       // compute warps; one more warp issues the loads
constexpr int kStrThreads = (kStrWarps + 1) * 32;
constexpr int kStrSlots = 148 * 3; // resident tensor-core CTAs on a B200: three per SM
// Splits are made only while the items number below this (measured on B200:
// a split costs a partial write, a fence and an atomic per item, ~5 us, so
// it pays only when a handful of items would leave most SMs idle).
constexpr int kStrSplitTarget = 160;
constexpr int kStrMinSubs = 4;     // sub-tiles per split below which no further split is made
constexpr bool kStrPagedPersist = true;  // paged entries come sorted by length
static_assert(kDecSub == kDecSubRows, "paged sub-tiles and TMA boxes must agree");
// Paged kernels take two tensor maps, DecParams (< 128 bytes) and the table
// by value; CUDA 12.1+ allows 32764 bytes of kernel parameters.
static_assert(2 * sizeof(CUtensorMap) + 256 + sizeof(PagedTable) <= 32764,
              "paged kernel parameters exceed the 32764-byte limit");

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
  // Dense K / V in global memory (the streaming kernel copies a partial last
  // sub-tile itself): element strides of rows and of row groups.
  const void *k, *v;
  int64_t kv_rs, kv_gs;
  int64_t q_rs, o_rs;
  int group_size, t_kv, n_heads;
  int row_chunks, n_splits, chunk;
  int n_items;   // tensor-core path: (split, head, row chunk) items, walked by a persistent grid
  float scale_log2;
  float *part;   // [rows][n_heads][n_splits][kPartStride]
  int *count;    // [row groups][n_heads]
  int *status;
  // Alignment-head capture (dense decode only; cap == nullptr turns it off):
  // the softmax over the keys of each query row r for every head h with
  // cap_slot[h] >= 0 goes to cap[((cap_row0 + r) * cap_nsel + cap_slot[h]) * t_kv + key].
  float *cap;
  int cap_nsel, cap_row0;
  signed char cap_slot[kCapMaxHeads];
};

// Capture slot of `head` in this launch, or -1.
WATTN_DEVINL int cap_slot_of(const DecParams &p, int head) {
  return (p.cap != nullptr && head < kCapMaxHeads) ? p.cap_slot[head] : -1;
}
WATTN_DEVINL float *cap_row(const DecParams &p, int row, int slot) {
  return p.cap + ((int64_t)(p.cap_row0 + row) * p.cap_nsel + slot) * p.t_kv;
}

// Shared memory of the CUDA-core path: every sub-tile of the split at once.
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

// Shared memory of the tensor-core path: the K/V ring (64 KB for 16-bit
// K/V, so three CTAs share an SM) and the cross-warp merge buffers (the
// ring keeps streaming the next item during a merge). The scores stay in
// mma fragments.
template <int KV_DT>
struct StreamSmem {
  uint8_t k[kStrStages][KvGeom<KV_DT>::sub_bytes];
  uint8_t v[kStrStages][KvGeom<KV_DT>::sub_bytes];
  float red[kStrWarps][kDecRows][64];  // per-warp partial outputs of an item
  float m[kDecRows], l[kDecRows];
  float wm[kStrWarps][kDecRows], wl[kStrWarps][kDecRows];  // per-warp max / normaliser
  uint64_t kfull[kStrStages], vfull[kStrStages], empty[kStrStages];
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

// Query rows of one work item and the physical key range [kv_lo, kv_hi)
// they attend; `cnt_idx` is the item's split counter.
struct DecRows {
  int row0, nr, kv_lo, kv_hi, group, cnt_idx;
  int entry;  // paged: the item's entry in the PagedTable
};

// One work item: split `split` of the keys of (row chunk / paged row z,
// head). `k_beg` is its first key and `n_sub` its sub-tiles; an item past
// the end of its row's keys (paged rows shorter than the longest) is empty.
struct DecWork {
  DecRows rw;
  int head, split, n_splits, k_beg, n_sub;
};

template <bool PAGED>
WATTN_DEVINL DecWork dec_work(const DecParams &p, const PagedTable *pt, int split, int head,
                              int z) {
  DecWork w;
  DecRows &r = w.rw;
  if constexpr (PAGED) {
    r.entry = z;
    r.row0 = pt->row_of[z];
    r.nr = 1;
    r.kv_lo = pt->kv_lo[z];
    r.kv_hi = pt->kv_hi[z];
    r.group = 0;
  } else {
    r.group = z / p.row_chunks;
    const int rc = z % p.row_chunks;
    r.row0 = r.group * p.group_size + rc * kDecRows;
    r.nr = min(kDecRows, p.group_size - rc * kDecRows);
    r.kv_lo = 0;
    r.kv_hi = p.t_kv;
    r.entry = 0;
  }
  r.cnt_idx = z * p.n_heads + head;
  w.head = head;
  w.split = split;
  const int base = r.kv_lo & ~(kDecSub - 1);  // sub-tiles start on 64-row marks
  w.n_splits = (r.kv_hi - base + p.chunk - 1) / p.chunk;
  w.k_beg = base + split * p.chunk;
  w.n_sub = w.k_beg < r.kv_hi ? min(p.chunk, r.kv_hi - w.k_beg + kDecSub - 1) / kDecSub : 0;
  return w;
}

// Item `it` of the tensor-core grid: split fastest, then head, then row
// chunk, so the items running at once read neighbouring heads of the same
// K/V rows.
template <bool PAGED>
WATTN_DEVINL DecWork dec_item(const DecParams &p, const PagedTable *pt, int it) {
  const int split = it % p.n_splits;
  const int rest = it / p.n_splits;
  return dec_work<PAGED>(p, pt, split, rest % p.n_heads, rest / p.n_heads);
}

// Barrier of the four compute warps of the tensor-core path (the producer
// warp runs ahead and takes no part).
WATTN_DEVINL void compute_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Issues the TMA loads of the K and V sub-tiles that start at key `key`,
// each completing on its own barrier. Dense: map_k / map_v are the K and V
// tensors. Paged: both view the page pool, map_k with 64-row boxes and
// map_v with kDecTailRows-row boxes; a sub-tile of which only `rows` < 64
// keys are attended loads just the 16-row boxes covering them (the rows
// left unloaded keep finite data of earlier sub-tiles or the initial zeros
// and are masked).
template <int KV_DT, bool PAGED>
WATTN_DEVINL void issue_sub(uint8_t *kdst, uint8_t *vdst, uint64_t *kbar, uint64_t *vbar,
                            const CUtensorMap &map_k, const CUtensorMap &map_v,
                            const DecParams &p, const PagedTable *pt, const DecRows &rw,
                            int head, int key, int rows) {
  using G = KvGeom<KV_DT>;
  if constexpr (PAGED) {
    // Pool rows: (((page * n_layers + layer) * 2 + kv) * n_heads + head) * page_rows + r
    const int page = pt->pages[rw.entry][key / pt->page_rows];
    const int r_in = key % pt->page_rows;
    const int64_t rk =
        ((((int64_t)page * pt->n_layers + pt->layer) * 2 + 0) * p.n_heads + head) *
            pt->page_rows + r_in;
    const int64_t rv = rk + (int64_t)p.n_heads * pt->page_rows;
    if (rows >= kDecSub) {
      mbar_arrive_expect_tx(kbar, G::sub_bytes);
      mbar_arrive_expect_tx(vbar, G::sub_bytes);
#pragma unroll
      for (int bk = 0; bk < G::blocks; ++bk) {
        tma_load_2d(kdst + bk * kDecSub * 128, &map_k, kbar, bk * G::block_elems, (int)rk);
        tma_load_2d(vdst + bk * kDecSub * 128, &map_k, vbar, bk * G::block_elems, (int)rv);
      }
    } else {
      const int n_box = (rows + kDecTailRows - 1) / kDecTailRows;
      const uint32_t bytes = n_box * kDecTailRows * 128 * G::blocks;
      mbar_arrive_expect_tx(kbar, bytes);
      mbar_arrive_expect_tx(vbar, bytes);
      for (int i = 0; i < n_box; ++i) {
        const int off = i * kDecTailRows;
#pragma unroll
        for (int bk = 0; bk < G::blocks; ++bk) {
          tma_load_2d(kdst + bk * kDecSub * 128 + off * 128, &map_v, kbar, bk * G::block_elems,
                      (int)(rk + off));
          tma_load_2d(vdst + bk * kDecSub * 128 + off * 128, &map_v, vbar, bk * G::block_elems,
                      (int)(rv + off));
        }
      }
    }
  } else {
    mbar_arrive_expect_tx(kbar, G::sub_bytes);
    mbar_arrive_expect_tx(vbar, G::sub_bytes);
#pragma unroll
    for (int bk = 0; bk < G::blocks; ++bk) {
      tma_load_4d(kdst + bk * kDecSub * 128, &map_k, kbar, bk * G::block_elems, head, key,
                  rw.group);
      tma_load_4d(vdst + bk * kDecSub * 128, &map_v, vbar, bk * G::block_elems, head, key,
                  rw.group);
    }
  }
}

// Turns the captured scaled scores of one query row into its softmax over
// the row's n keys, p = 2^(v - M) / sum 2^(v - M) (one warp; M is any value
// within 2^8 of the row max, the kernels' running max or the split merge's).
WATTN_DEVINL void cap_softmax_row(float *row, int n, float M, int ln) {
  float sum = 0.f;
  for (int j = ln; j < n; j += 32) sum += ex2(__ldcg(row + j) - M);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;
  for (int j = ln; j < n; j += 32) row[j] = ex2(__ldcg(row + j) - M) * inv;
}

// Sums the four warps' partial outputs in `red` ([4][kDecRows][64]) and
// either stores the rows (one split) or writes this split's partial; the
// last CTA of the (row group, head) to finish then merges every split by
// log-sum-exp. Called by all threads of the CTA.
// NAMED: the CTA's compute warps (threads 0..127) call it, synchronising on
// compute_sync(); otherwise every thread does, on __syncthreads().
template <typename OutT, bool NAMED, bool PAGED>
__device__ void finish_split(const DecParams &p, const float *red, const float *sm,
                             const float *sl, int *s_last, const DecRows &rw, int head, int split,
                             int n_splits) {
  const int tid = threadIdx.x, nt = NAMED ? kStrWarps * 32 : blockDim.x;
  const int64_t part_base = (int64_t)rw.row0 * p.n_heads;  // row-major partial index base
  for (int i = tid; i < rw.nr * 64; i += nt) {
    const int r = i >> 6, d = i & 63;
    const float a = red[(0 * kDecRows + r) * 64 + d] + red[(1 * kDecRows + r) * 64 + d] +
                    red[(2 * kDecRows + r) * 64 + d] + red[(3 * kDecRows + r) * 64 + d];
    if (n_splits == 1) {
      store_out<OutT>(p.o, (int64_t)(rw.row0 + r) * p.o_rs + head * 64 + d, a / sl[r]);
    } else {
      float *part = p.part + ((part_base + (int64_t)r * p.n_heads + head) * p.n_splits + split) *
                                 kPartStride;
      part[d] = a;
      if (d == 0) {
        part[64] = sm[r];
        part[65] = sl[r];
      }
    }
  }
  const int n_warps = nt >> 5, wid = tid >> 5, ln = tid & 31;
  const int cap_slot = PAGED ? -1 : cap_slot_of(p, head);  // no capture on the paged path
  if (n_splits == 1) {
    // The captured scores of this CTA's rows were written before the
    // barriers that precede this call.
    if (cap_slot >= 0)
      for (int r = wid; r < rw.nr; r += n_warps)
        cap_softmax_row(cap_row(p, rw.row0 + r, cap_slot), p.t_kv, sm[r], ln);
    return;
  }

  // Release: the barrier orders every thread's partial before thread 0's
  // fence, and the fence orders them before the count.
  if constexpr (NAMED) compute_sync(); else __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(&p.count[rw.cnt_idx], 1);
    *s_last = (prev == n_splits - 1);
    if (*s_last) __threadfence();  // acquire: the other splits' partials
  }
  if constexpr (NAMED) compute_sync(); else __syncthreads();
  if (!*s_last) return;
  // One warp per row, two dims per lane; the splits' partials are read four
  // at a time with independent loads (they sit in L2).
  for (int r = wid; r < rw.nr; r += n_warps) {
    const float *part0 =
        p.part + ((part_base + (int64_t)r * p.n_heads + head) * p.n_splits) * kPartStride;
    float M = -INFINITY;
    for (int sp = ln; sp < n_splits; sp += 32) M = fmaxf(M, __ldcg(part0 + sp * kPartStride + 64));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f, o0 = 0.f, o1 = 0.f;
    int sp = 0;
    for (; sp + 4 <= n_splits; sp += 4) {
      float mv[4], lv[4];
      float2 av[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float *pp = part0 + (sp + u) * kPartStride;
        mv[u] = __ldcg(pp + 64);
        lv[u] = __ldcg(pp + 65);
        av[u] = __ldcg(reinterpret_cast<const float2 *>(pp + 2 * ln));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = ex2(mv[u] - M);
        L = fmaf(w, lv[u], L);
        o0 = fmaf(w, av[u].x, o0);
        o1 = fmaf(w, av[u].y, o1);
      }
    }
    for (; sp < n_splits; ++sp) {
      const float *pp = part0 + sp * kPartStride;
      const float w = ex2(__ldcg(pp + 64) - M);
      const float2 a = __ldcg(reinterpret_cast<const float2 *>(pp + 2 * ln));
      L = fmaf(w, __ldcg(pp + 65), L);
      o0 = fmaf(w, a.x, o0);
      o1 = fmaf(w, a.y, o1);
    }
    const int64_t off = (int64_t)(rw.row0 + r) * p.o_rs + head * 64 + 2 * ln;
    store_out<OutT>(p.o, off, o0 / L);
    store_out<OutT>(p.o, off + 1, o1 / L);
    // Every split's captured scores are visible here (they precede each
    // split's release of the counter).
    if (cap_slot >= 0) cap_softmax_row(cap_row(p, rw.row0 + r, cap_slot), p.t_kv, M, ln);
  }
  if (tid == 0) p.count[rw.cnt_idx] = 0;  // leave the workspace zeroed for the next call
}

// ---------------------------------------------------------------- tensor-core path
// Persistent streaming body. CTA b walks items b, b + gridDim.x, ... (the
// host sizes the grid so each CTA gets the same number of items). Warp
// kStrWarps (lane 0) fills the ring for all of them in order, running ahead
// across item boundaries; compute warp w takes keys 16w..16w+15 of every
// 64-key sub-tile. S = Q K^T and O += P V with mma.sync m16n8k16 (rows = the
// item's query rows, padded to 16; the scale is applied in f32 to S), online
// softmax per row in the exp2 domain, then a log-sum-exp merge of the four
// warps and the split epilogue, while the producer already streams the next
// item's keys.
template <int DT>
WATTN_DEVINL void load_q(uint32_t (&qa)[4][4], const DecParams &p, const DecRows &rw, int head,
                         int g, int t4) {
  using T = typename Elem<DT>::T;
  const uint32_t *qrow = reinterpret_cast<const uint32_t *>(
      reinterpret_cast<const T *>(p.q) + (int64_t)(rw.row0 + g) * p.q_rs + head * 64);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    qa[ks][0] = g < rw.nr ? qrow[ks * 8 + t4] : 0u;
    qa[ks][2] = g < rw.nr ? qrow[ks * 8 + 4 + t4] : 0u;
    qa[ks][1] = qa[ks][3] = 0u;  // rows 8..15 of the tile: beyond the 8 rows of an item
  }
}

// A dense sub-tile of which only `rows` < 64 keys lie inside the key range,
// copied by the whole producer warp into the ring's 128-byte-swizzled layout
// (16-byte chunk c of row r at r * 128 + ((c ^ (r & 7)) << 4)) with 16-byte
// cp.async copies, the rows past the range zero-filled by the copies
// themselves (source size 0). A TMA box reaching past the tensor's last row
// would zero-fill those rows itself; with such boxes in a ring that wraps,
// items whose stages a later item reuses were read wrong now and then (on
// B200: up to a quarter of the calls of 32 x 16 rows over 70 keys beside a
// concurrent kernel), so partial sub-tiles never leave the key range. The
// copies complete on the stage's full barrier (see the producer), so the
// warp goes on at once.
template <int DT>
WATTN_DEVINL void copy_partial_sub(uint8_t *dst, const void *src_base, int64_t row_stride,
                                   int rows, int lane) {
  static_assert(KvGeom<DT>::blocks == 1, "16-bit rows of 128 bytes");
  using T = typename Elem<DT>::T;
  const T *src = reinterpret_cast<const T *>(src_base);
  const uint32_t d0 = smem_u32(dst);
#pragma unroll 4
  for (int i = lane; i < kDecSub * 8; i += 32) {
    const int r = i >> 3, ch = i & 7;
    const bool in = r < rows;
    const T *from = src + (int64_t)(in ? r : 0) * row_stride + ch * 8;  // a valid address either way
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     d0 + r * 128 + ((ch ^ (r & 7)) << 4)),
                 "l"(from), "r"(in ? 16 : 0)
                 : "memory");
  }
}

// Makes `bar`'s current phase wait for this thread's cp.async copies issued
// so far: the pending count goes up by one now and down by one when they
// have landed.
WATTN_DEVINL void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int DT, int OUT_DT, bool PAGED>
__device__ void decode_stream_body(const CUtensorMap &map_k, const CUtensorMap &map_v,
                                   const DecParams &p, const PagedTable *pt) {
  using T = typename Elem<DT>::T;
  using OutT = typename Elem<OUT_DT>::T;
  extern __shared__ uint8_t dec_smem_raw[];
  StreamSmem<DT> &s = *reinterpret_cast<StreamSmem<DT> *>(
      (reinterpret_cast<uintptr_t>(dec_smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if constexpr (PAGED) {
    // Tail sub-tiles load only their attended rows: the V rows they leave
    // must hold finite values (they meet p = 0), so the ring starts zeroed.
    uint4 *v4 = reinterpret_cast<uint4 *>(&s.v[0][0]);
    for (int i = tid; i < (int)(sizeof(s.v) / 16); i += blockDim.x) v4[i] = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (tid == 0) {
    for (int st = 0; st < kStrStages; ++st) {
      mbar_init(&s.kfull[st], 1);
      mbar_init(&s.vfull[st], 1);
      mbar_init(&s.empty[st], kStrWarps);
    }
    s.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int *abort = &s.abort;

  if (warp == kStrWarps) {
    // ---- producer: refills each stage as the compute warps free it; lane 0
    // issues the TMA loads, and a dense item's partial last sub-tile is
    // copied by the whole warp (copy_partial_sub): every lane ties its copies
    // to both full barriers, then lane 0 makes the one expected arrival, so
    // each barrier completes once all the copies have landed.
    uint32_t c = 0;  // position in the ring, over all items of this CTA
    for (int it = blockIdx.x; it < p.n_items; it += gridDim.x) {
      const DecWork w = dec_item<PAGED>(p, pt, it);
      for (int st = 0; st < w.n_sub; ++st, ++c) {
        const int stage = c % kStrStages;
        const uint32_t ph = (c / kStrStages) & 1;
        const bool free_stage = mbar_wait(&s.empty[stage], ph ^ 1, abort, p.status,
                                          (2 << 24) | (3 << 16) | ((c & 0xff) << 8));
        if (!__all_sync(0xffffffffu, free_stage)) return;
        const int key = w.k_beg + st * kDecSub;
        const int rows = w.rw.kv_hi - key;
        if (!PAGED && rows < kDecSub) {
          const int64_t off = (int64_t)w.rw.group * p.kv_gs + (int64_t)key * p.kv_rs + w.head * 64;
          using T = typename Elem<DT>::T;
          copy_partial_sub<DT>(s.k[stage], reinterpret_cast<const T *>(p.k) + off, p.kv_rs, rows,
                               lane);
          copy_partial_sub<DT>(s.v[stage], reinterpret_cast<const T *>(p.v) + off, p.kv_rs, rows,
                               lane);
          cp_async_arrive(&s.kfull[stage]);
          cp_async_arrive(&s.vfull[stage]);
          __syncwarp();  // every lane's pending count is in before the expected arrival
          if (lane == 0) {
            mbar_arrive(&s.kfull[stage]);
            mbar_arrive(&s.vfull[stage]);
          }
        } else if (lane == 0) {
          // a stage last filled by the copies above is rewritten by the TMA
          // (async proxy) only after these writes, seen through the empty
          // barrier, are ordered for it
          if constexpr (!PAGED) fence_proxy_async_smem();
          issue_sub<DT, PAGED>(s.k[stage], s.v[stage], &s.kfull[stage], &s.vfull[stage], map_k,
                               map_v, p, pt, w.rw, w.head, key, rows);
        }
        __syncwarp();
      }
    }
    return;  // the producer warp takes no part in the epilogues
  }

  // ---- compute warps
  const int g = lane >> 2, t4 = lane & 3;
  const float c = p.scale_log2;
  const int kb = warp * 16;
  uint32_t pos = 0;  // position in the ring, as the producer counts it
  // Each item's description and query rows are fetched one item ahead, at
  // the start of the previous item, so their latency (a page-table entry in
  // the constant bank, a query row in HBM) hides behind a whole item.
  uint32_t qa[4][4], qn[4][4];
  DecWork w;
  if (blockIdx.x < p.n_items) {
    w = dec_item<PAGED>(p, pt, blockIdx.x);
    if (w.n_sub > 0) load_q<DT>(qa, p, w.rw, w.head, g, t4);
  }
  for (int it = blockIdx.x; it < p.n_items; it += gridDim.x) {
    const int nx = it + gridDim.x;
    DecWork wn;
    if (nx < p.n_items) {
      wn = dec_item<PAGED>(p, pt, nx);
      if (wn.n_sub > 0) load_q<DT>(qn, p, wn.rw, wn.head, g, t4);
    }
    if (w.n_sub == 0) {  // a paged row with fewer splits than the longest
      w = wn;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int e = 0; e < 4; ++e) qa[ks][e] = qn[ks][e];
      continue;
    }
    float m_r = -INFINITY, l_r = 0.f;
    float acc[8][4];
#pragma unroll
    for (int db = 0; db < 8; ++db) acc[db][0] = acc[db][1] = acc[db][2] = acc[db][3] = 0.f;
    for (int st = 0; st < w.n_sub; ++st, ++pos) {
      const int stage = pos % kStrStages;
      const uint32_t ph = (pos / kStrStages) & 1;
      mbar_wait(&s.kfull[stage], ph, abort, p.status, (2 << 24) | (1 << 16) | ((pos & 0xff) << 8));
      const uint32_t ktile = smem_u32(s.k[stage]), vtile = smem_u32(s.v[stage]);
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
          mma16816<T>(sc[nb], qa[2 * ks2], r0, r1);
          mma16816<T>(sc[nb], qa[2 * ks2 + 1], r2, r3);
        }
      }
      // Mask keys outside [kv_lo, kv_hi) (row g holds keys 2*t4, 2*t4+1 of each 8).
      const int key0 = w.k_beg + st * kDecSub + kb + 2 * t4;
      if constexpr (!PAGED) {
        const int slot = cap_slot_of(p, w.head);
        if (slot >= 0 && g < w.rw.nr) {
          // Alignment-head capture: the scaled scores (exp2 domain) of the
          // attended keys; finish_split turns them into the softmax.
          float *dst = cap_row(p, w.rw.row0 + g, slot);
#pragma unroll
          for (int nb = 0; nb < 2; ++nb)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = key0 + nb * 8 + e;
              if (key < w.rw.kv_hi) dst[key] = sc[nb][e] * c;
            }
        }
      }
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + nb * 8 + e;
          if (key < w.rw.kv_lo || key >= w.rw.kv_hi) sc[nb][e] = -INFINITY;
        }
      float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mc = mx * c;
      if (mc > m_r + 8.0f) {  // lazy rescale: only when the running max grows by > 2^8
        const float alpha = ex2(m_r - mc);
        l_r *= alpha;
#pragma unroll
        for (int db = 0; db < 8; ++db)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[db][e] *= alpha;
        m_r = mc;
      }
      const float mu = (m_r == -INFINITY) ? 0.f : m_r;
      float pe[2][2];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) pe[nb][e] = ex2(fmaf(sc[nb][e], c, -mu));
      // P enters the product as two 16-bit parts: rows 0-7 of the A tile
      // hold the weights rounded to T, rows 8-15 (no query rows there) the
      // rounding residual p - round(p), also in T. Output rows 8-15 then
      // gather the residual's products, added to rows 0-7 at the item's end:
      // P keeps ~16 significant bits with bf16 (the reference's weights
      // are f32, attention.rs:246-434; bf16's 8 alone gave 2.5e-3 max-abs
      // errors on short key ranges) at no extra tensor-core instruction.
      uint32_t pa[4];
      pa[0] = pack2<T>(pe[0][0], pe[0][1]);
      pa[2] = pack2<T>(pe[1][0], pe[1][1]);
      {
        const float2 r0 = unpack2<T>(pa[0]), r2 = unpack2<T>(pa[2]);
        pa[1] = pack2<T>(pe[0][0] - r0.x, pe[0][1] - r0.y);
        pa[3] = pack2<T>(pe[1][0] - r2.x, pe[1][1] - r2.y);
        // the f32 weights, which the two parts carry to ~2^-16
        l_r += (pe[0][0] + pe[0][1]) + (pe[1][0] + pe[1][1]);
      }
      mbar_wait(&s.vfull[stage], ph, abort, p.status, (2 << 24) | (2 << 16) | ((pos & 0xff) << 8));
      {
        const int key_row = kb + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int db2 = 0; db2 < 4; ++db2) {
          uint32_t r0, r1, r2, r3;
          const int chunk = db2 * 2 + (lane >> 4);
          ldsm_x4_t(vtile + key_row * 128 + ((chunk ^ (key_row & 7)) << 4), r0, r1, r2, r3);
          mma16816<T>(acc[2 * db2], pa, r0, r1);
          mma16816<T>(acc[2 * db2 + 1], pa, r2, r3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);  // this warp is done with the stage
    }
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
    // the residual's products (output rows 8-15) join the rounded weights'
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      acc[db][0] += acc[db][2];
      acc[db][1] += acc[db][3];
    }

    // ---- merge the four compute warps (log-sum-exp) into red / s.m / s.l
    compute_sync();  // the previous item's epilogue is done with red, m, l
    if (t4 == 0) s.wm[warp][g] = m_r;
    compute_sync();
    if (g < w.rw.nr) {
      const float M = fmaxf(fmaxf(s.wm[0][g], s.wm[1][g]), fmaxf(s.wm[2][g], s.wm[3][g]));
      const float wt = (m_r == -INFINITY) ? 0.f : ex2(m_r - M);
#pragma unroll
      for (int db = 0; db < 8; ++db)
        *reinterpret_cast<float2 *>(&s.red[warp][g][db * 8 + 2 * t4]) =
            make_float2(acc[db][0] * wt, acc[db][1] * wt);
      if (t4 == 0) {
        s.wl[warp][g] = l_r * wt;
        if (warp == 0) s.m[g] = M;
      }
    }
    compute_sync();
    if (tid < w.rw.nr) s.l[tid] = s.wl[0][tid] + s.wl[1][tid] + s.wl[2][tid] + s.wl[3][tid];
    compute_sync();
    finish_split<OutT, true, PAGED>(p, &s.red[0][0][0], s.m, s.l, &s.last, w.rw, w.head, w.split,
                             w.n_splits);
    w = wn;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
      for (int e = 0; e < 4; ++e) qa[ks][e] = qn[ks][e];
  }
}

// ---------------------------------------------------------------- CUDA-core path
template <int Q_DT, int KV_DT, int OUT_DT, bool PAGED>
__device__ void decode_simt_body(const CUtensorMap &map_k, const CUtensorMap &map_v,
                                 const DecParams &p, const PagedTable *pt) {
  using QT = typename Elem<Q_DT>::T;
  using OutT = typename Elem<OUT_DT>::T;
  extern __shared__ uint8_t dec_smem_raw[];
  DecSmem<KV_DT> &s = *reinterpret_cast<DecSmem<KV_DT> *>(
      (reinterpret_cast<uintptr_t>(dec_smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const DecWork w = dec_work<PAGED>(p, pt, blockIdx.x, blockIdx.y, blockIdx.z);
  if (w.n_sub == 0) return;  // beyond this row's keys
  const DecRows &rw = w.rw;
  const int nr = rw.nr, head = w.head, split = w.split, n_splits = w.n_splits;
  const int k_beg = w.k_beg, n_sub = w.n_sub;

  if (tid == 0) {
    for (int st = 0; st < n_sub; ++st) {
      mbar_init(&s.kbar[st], 1);
      mbar_init(&s.vbar[st], 1);
    }
    s.abort = 0;
    fence_barrier_init();
    for (int st = 0; st < n_sub; ++st)
      issue_sub<KV_DT, PAGED>(s.k[st], s.v[st], &s.kbar[st], &s.vbar[st], map_k, map_v, p, pt,
                              rw, head, k_beg + st * kDecSub, kDecSub);
  }

  // Query rows, pre-scaled into the exp2 domain.
  for (int i = tid; i < kDecRows * 64; i += kDecThreads) {
    const int r = i >> 6, d = i & 63;
    float x = 0.f;
    if (r < nr)
      x = to_f32(
          reinterpret_cast<const QT *>(p.q)[(int64_t)(rw.row0 + r) * p.q_rs + head * 64 + d]);
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
    const bool valid = key >= rw.kv_lo && key < rw.kv_hi;
    const int slot = PAGED ? -1 : cap_slot_of(p, head);
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) {
      const float full = dot[r] + __shfl_xor_sync(0xffffffffu, dot[r], 1);
      if (half == 0 && r < nr) {
        s.sc[r][st * kDecSub + krow] = valid ? full : -INFINITY;
        if (slot >= 0 && valid) cap_row(p, rw.row0 + r, slot)[key] = full;  // alignment-head capture
      }
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
  // Cross-warp sum through the K buffer, idle since the barrier after the scores.
  float *red = reinterpret_cast<float *>(&s.k[0][0]);
#pragma unroll
  for (int r = 0; r < kDecRows; ++r)
    if (r < nr)
      *reinterpret_cast<float2 *>(&red[(warp * kDecRows + r) * 64 + 2 * lane]) =
          make_float2(acc[r][0], acc[r][1]);
  __syncthreads();
  finish_split<OutT, false, PAGED>(p, red, s.m, s.l, &s.last, rw, head, split, n_splits);
}

template <int Q_DT, int KV_DT>
constexpr bool kDecStream = KV_DT != WATTN_F32 && Q_DT == KV_DT;

template <int Q_DT, int KV_DT, int OUT_DT>
__global__ void __launch_bounds__(kDecThreads)
    decode_dense_kernel(const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const DecParams p) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  decode_simt_body<Q_DT, KV_DT, OUT_DT, false>(map_k, map_v, p, nullptr);
}

template <int Q_DT, int KV_DT, int OUT_DT>
__global__ void __launch_bounds__(kDecThreads)
    decode_paged_kernel(const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const DecParams p,
                        const __grid_constant__ PagedTable pt) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  decode_simt_body<Q_DT, KV_DT, OUT_DT, true>(map_k, map_v, p, &pt);
}

template <int DT, int OUT_DT>
__global__ void __launch_bounds__(kStrThreads, 3)  // three CTAs per SM (shared memory allows three)
    decode_stream_dense_kernel(const __grid_constant__ CUtensorMap map_k,
                               const __grid_constant__ CUtensorMap map_v, const DecParams p) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  decode_stream_body<DT, OUT_DT, false>(map_k, map_v, p, nullptr);
}

template <int DT, int OUT_DT>
__global__ void __launch_bounds__(kStrThreads, 3)  // three CTAs per SM (shared memory allows three)
    decode_stream_paged_kernel(const __grid_constant__ CUtensorMap map_k,
                               const __grid_constant__ CUtensorMap map_v, const DecParams p,
                               const __grid_constant__ PagedTable pt) {
  grid_dep_wait();  // (launched with programmatic serialisation)
  grid_dep_launch();
  decode_stream_body<DT, OUT_DT, true>(map_k, map_v, p, &pt);
}

template <typename K>
int set_smem(K kern, int bytes) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(decode)");
  return WATTN_OK;
}

// Grid: (splits, heads, row groups x row chunks) dense; (splits, heads, rows) paged.
template <int Q_DT, int KV_DT, int OUT_DT, bool PAGED>
int launch_typed(const CUtensorMap &mk, const CUtensorMap &mv, const DecParams &p,
                 const PagedTable *pt, dim3 grid, cudaStream_t stream) {
  if constexpr (kDecStream<Q_DT, KV_DT>) {
    constexpr int smem = (int)sizeof(StreamSmem<KV_DT>) + 1024;
    if constexpr (PAGED) {
      auto kern = decode_stream_paged_kernel<KV_DT, OUT_DT>;
      int rc = set_smem(kern, smem);
      if (rc != WATTN_OK) return rc;
      if (launch_pdl(kern, grid, dim3(kStrThreads), smem, stream, mk, mv, p, *pt) != cudaSuccess)
        return check_launch("decode_stream_paged (launch)");
    } else {
      auto kern = decode_stream_dense_kernel<KV_DT, OUT_DT>;
      int rc = set_smem(kern, smem);
      if (rc != WATTN_OK) return rc;
      if (launch_pdl(kern, grid, dim3(kStrThreads), smem, stream, mk, mv, p) != cudaSuccess)
        return check_launch("decode_stream_dense (launch)");
    }
  } else {
    constexpr int smem = (int)sizeof(DecSmem<KV_DT>) + 1024;
    if constexpr (PAGED) {
      auto kern = decode_paged_kernel<Q_DT, KV_DT, OUT_DT>;
      int rc = set_smem(kern, smem);
      if (rc != WATTN_OK) return rc;
      if (launch_pdl(kern, grid, dim3(kDecThreads), smem, stream, mk, mv, p, *pt) != cudaSuccess)
        return check_launch("decode_paged (launch)");
    } else {
      auto kern = decode_dense_kernel<Q_DT, KV_DT, OUT_DT>;
      int rc = set_smem(kern, smem);
      if (rc != WATTN_OK) return rc;
      if (launch_pdl(kern, grid, dim3(kDecThreads), smem, stream, mk, mv, p) != cudaSuccess)
        return check_launch("decode_dense (launch)");
    }
  }
  return check_launch(PAGED ? "decode_paged" : "decode_dense");
}

// Dispatch over (q, kv, out) element types.
template <bool PAGED>
int dispatch(int q_dt, int kv_dt, int out_dt, const CUtensorMap &mk, const CUtensorMap &mv,
             const DecParams &p, const PagedTable *pt, dim3 grid, cudaStream_t stream) {
#define WATTN_DEC_CASE(QD, KD, OD)                                       \
  if (q_dt == QD && kv_dt == KD && out_dt == OD)                         \
    return launch_typed<QD, KD, OD, PAGED>(mk, mv, p, pt, grid, stream);
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

bool uses_stream(int q_dtype, int kv_dtype) {
  return kv_dtype != WATTN_F32 && q_dtype == kv_dtype;
}

// Keys per split. Tensor-core path: no split unless the items number below
// kStrSplitTarget, then about kStrSplitTarget / items splits, each at least
// kStrMinSubs sub-tiles where the keys allow, the splits of a row equal to
// within a sub-tile. CUDA-core path: the largest chunk (<= 256 keys, 128 for
// f32 K/V to fit shared memory) that still gives >= ~4 waves of CTAs on 148
// SMs.
int chunk_for(int q_dtype, int kv_dtype, int ctas_per_chunk_unit, int t_kv) {
  const int subs = std::max(1, (t_kv + kDecSub - 1) / kDecSub);
  if (uses_stream(q_dtype, kv_dtype)) {
    const int units = std::max(1, ctas_per_chunk_unit);
    int splits = std::min(kStrSplitTarget / units, subs / kStrMinSubs);
    splits = std::max(1, splits);
    return ((subs + splits - 1) / splits) * kDecSub;
  }
  const int max_chunk = (kv_dtype == WATTN_F32 ? 2 : kDecMaxSubs) * kDecSub;
  int chunk = max_chunk;
  while (chunk > kDecSub) {
    const long long ctas = (long long)ctas_per_chunk_unit * ((t_kv + chunk - 1) / chunk);
    if (ctas >= 148LL * 2 * 4) break;
    chunk >>= 1;
  }
  return chunk;
}

// Persistent grid of the tensor-core path: the fewest CTAs that give every
// CTA the same number of items (to within one) with at most kStrSlots CTAs
// per round of items.
int stream_grid(long long items) {
  const long long per_cta = (items + kStrSlots - 1) / kStrSlots;
  return (int)((items + per_cta - 1) / per_cta);
}

}  // namespace

DecodePlan plan_decode(int n_groups, int group_size, int t_kv, int n_heads, int q_dtype,
                       int kv_dtype) {
  DecodePlan pl;
  pl.row_chunks = (group_size + kDecRows - 1) / kDecRows;
  pl.chunk = chunk_for(q_dtype, kv_dtype, n_groups * pl.row_chunks * n_heads, t_kv);
  pl.n_splits = t_kv > 0 ? (t_kv + pl.chunk - 1) / pl.chunk : 1;
  const size_t rows = (size_t)n_groups * group_size;
  pl.workspace_bytes = kCounterBytes + rows * n_heads * pl.n_splits * kPartStride * sizeof(float);
  return pl;
}

int launch_decode(const void *q, const void *k, const void *v, void *o, int q_dtype,
                  int kv_dtype, int out_dtype, int n_groups, int group_size, int t_kv,
                  int n_heads, int64_t q_rs, int64_t kv_rs, int64_t kv_gs, int64_t o_rs,
                  float scale, void *workspace, size_t workspace_bytes, cudaStream_t stream,
                  const CaptureSpec *cap) {
  if (cap != nullptr && n_heads > kCapMaxHeads)
    return set_error(WATTN_ERR_UNSUPPORTED, "decode capture: %d heads (at most %d)", n_heads,
                     kCapMaxHeads);
  const DecodePlan pl = plan_decode(n_groups, group_size, t_kv, n_heads, q_dtype, kv_dtype);
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
  p.k = k;
  p.v = v;
  p.kv_rs = kv_rs;
  p.kv_gs = kv_gs;
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
  p.cap = nullptr;
  p.cap_nsel = p.cap_row0 = 0;
  for (int h = 0; h < kCapMaxHeads; ++h) p.cap_slot[h] = -1;
  if (cap != nullptr) {
    p.cap = cap->out;
    p.cap_nsel = cap->n_selected;
    p.cap_row0 = cap->row0;
    for (int h = 0; h < n_heads; ++h) p.cap_slot[h] = (signed char)cap->slot_of_head[h];
  }
  p.n_items = pl.n_splits * n_heads * n_groups * pl.row_chunks;
  const dim3 grid = uses_stream(q_dtype, kv_dtype)
                        ? dim3(stream_grid(p.n_items))
                        : dim3(pl.n_splits, n_heads, n_groups * pl.row_chunks);
  return dispatch<false>(q_dtype, kv_dtype, out_dtype, mk, mv, p, nullptr, grid, stream);
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
  p.k = p.v = nullptr;  // (the paged kernels read the pool through the tensor maps only)
  p.kv_rs = p.kv_gs = 0;
  p.q_rs = q_rs;
  p.o_rs = o_rs;
  p.group_size = 1;
  p.t_kv = 0;
  p.n_heads = n_heads;
  p.row_chunks = 1;
  p.chunk = chunk_for(q_dtype, kv_dtype, pt.n_rows * n_heads, max_keys);
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
  p.cap = nullptr;  // no capture on the paged (self-attention) path
  p.cap_nsel = p.cap_row0 = 0;
  for (int h = 0; h < kCapMaxHeads; ++h) p.cap_slot[h] = -1;
  p.n_items = p.n_splits * n_heads * pt.n_rows;
  const dim3 grid = !uses_stream(q_dtype, kv_dtype) ? dim3(p.n_splits, n_heads, pt.n_rows)
                    : kStrPagedPersist              ? dim3(stream_grid(p.n_items))
                                                    : dim3(p.n_items);
  return dispatch<true>(q_dtype, kv_dtype, out_dtype, map_k, map_v, p, &pt, grid, stream);
}

size_t paged_workspace_bytes(int n_rows, int n_heads, int max_keys) {
  // Every chunk is at least one sub-tile, so splits <= ceil(max_keys / 64).
  const int n_splits = (max_keys + kDecSub - 1) / kDecSub;
  return kCounterBytes + (size_t)n_rows * n_heads * n_splits * kPartStride * sizeof(float);
}

}  // namespace wattn
