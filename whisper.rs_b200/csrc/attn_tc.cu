// attn_tc.cu -- encoder / general attention on the sm_100a tensor cores.
//
// Replaces the tiled online-softmax loop of flash_attention_2
// (crates/tensor/src/ops/attention.rs:111-241) for f16 / bf16 inputs with
// f32 accumulation. Same function, B200 structure:
//
//   * a persistent grid of one CTA per SM walks work units of two 128-row
//     query tiles of one (utterance, head); each tile has its own softmax
//     warpgroup, so while one warpgroup turns S into P the tensor cores work
//     on the other tile. Every barrier phase, the K/V ring and the TMEM
//     buffers carry over from unit to unit, so the next unit's Q and first
//     K/V tiles load and its first scores are computed while the current
//     unit's last softmax and epilogue run;
//   * a TMA warp streams 128-key K and V tiles through a 4-deep ring in
//     shared memory (128-byte swizzle, the layout UMMA reads directly); the
//     query tiles are double-buffered, so the next unit's Q is resident
//     before the current unit ends. A ring stage is handed back by the two
//     softmax warpgroups once they have seen its PV products complete;
//   * one MMA warp per query tile issues that tile's tcgen05.mma: S = Q K^T
//     (M=128, N=128, K=64) into tensor memory, then O += P V (M=128, N=64,
//     K=128) with P read back from tensor memory. S(t, j+1) is issued as
//     soon as the softmax has taken S(t, j) into registers, so the next
//     scores are ready when the softmax finishes the current ones; the two
//     tiles' chains do not wait on each other;
//   * the softmax warpgroup owns one query row per thread: it reads its S
//     row from TMEM, keeps the running max m and normaliser l in registers
//     (exp2 domain), rescales O in TMEM only when the max grows by more than
//     2^8 (the result is exact either way: p never exceeds 256), and writes P
//     as packed 16-bit pairs back to TMEM. The two warpgroups take turns on
//     the exponential loop, warp by warp on each scheduler (whose SFU the
//     two warps share), so one's loads, max and stores hide behind the
//     other's exponentials;
//   * with bf16 inputs, P is rounded to f16 (11 significant bits) rather
//     than bf16 (8), so the PV product keeps close to the reference's f32 P
//     (attention.rs:207-222): a bandwidth-bound pre-pass writes an f16 copy
//     of V (exact for bf16 values in f16's normal range) with the largest
//     |v| of each block of the pass, and the kernel multiplies f16 P by that
//     copy when the largest |v| lies in [2^-6, 65280] (values below 2^-14
//     then err by less than 2^-25); otherwise (one uniform decision per
//     launch) P and V stay bf16;
//   * a unit's 16-bit output tiles are staged in its Q buffer (free once its
//     last scores are done) and leave with one TMA tensor store each, issued
//     by a second lane of the TMA warp, in place of row-by-row stores that
//     each touch 32 rows per warp.
//
// When whole units would leave SMs idle at the end (few utterances or heads
// per GPU), the units' key tiles are instead shared out evenly: each CTA
// takes a run of key tiles, a unit cut by a CTA boundary is computed in
// parts, and the part counted in last merges them (log-sum-exp); a merge
// warp does that while the softmax warps go on.
//
// Tensor memory per CTA (512 columns): tile t uses S at 256t (128 columns),
// P at 256t+128 (64 columns of packed pairs), O at 256t+192 (64 columns).
//
// Reference semantics kept: ragged key tiles are masked (attention.rs:190-192),
// causal rows see keys j <= i + q_pos_offset (:161-165; decoder.rs:864), the
// output is acc / l with 0 for an empty row (:228-240). Head dim is 64.

#include "wattn_common.cuh"
#include "wattn_internal.h"

#include <algorithm>
#include <climits>

namespace wattn {
namespace {

constexpr int kBM = 128;                 // query rows per tile (UMMA M)
constexpr int kBN = 128;                 // keys per tile
constexpr int kTiles = 2;                // query tiles per CTA
constexpr int kStages = 4;               // K/V ring depth
constexpr int kTileBytes = 128 * 128;    // 128 rows x 64 x 16-bit
constexpr int kTmaWarp = 4 * kTiles;      // warp 8
constexpr int kMmaWarp = kTmaWarp + 1;    // warp 9
constexpr int kMergeWarp = kMmaWarp + 1;  // warp 10: counts and merges split units' parts
constexpr int kMma1Warp = kMergeWarp + 1;  // warp 11: issues tile 1's products (warp 9: tile 0's)
constexpr int kThreads = (kMma1Warp + 1) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kAttnPartFloats = 66 * kBM;  // one tile's partial: O [64][128], m [128], l [128]
// One pair of exponentials in every kFmaExp2Every is computed on the FMA
// pipe (exp2_fma2) instead of the SFU (0: all on the SFU). With the two
// warpgroups taking turns, one warp per scheduler runs the loop and leaves
// the FMA pipe idle; one pair in 5 measured fastest on B200 (4, 6 and 8
// within 1-4 %; one in 3 or 2 adds more instructions than it saves SFU
// time).
constexpr int kFmaExp2Every = 5;


// Whether exponential pair i (of 64) is computed on the FMA pipe: one pair
// in kFmaExp2Every, spread through the loop when P is bf16 and the same
// number as the loop's last pairs when P is f16 (the fastest placement of
// each P type measured on B200: bf16 P, config 3, 671 vs 624 TFLOP/s with
// the last pairs; f16 P, config 2, 474 vs 424 spread out, and config 3 with
// bf16 inputs, 666 vs 571).
template <int P_DT>
WATTN_DEVINL constexpr bool fma_exp2_slot(int i) {
  constexpr int every = kFmaExp2Every > 0 ? kFmaExp2Every : 1;
  constexpr int n_fma = kFmaExp2Every > 0 ? 64 / every : 0;
  if constexpr (P_DT == WATTN_F16) return i >= 64 - n_fma;
  return kFmaExp2Every > 0 && i % every == every - 1;
}

struct Smem {
  uint8_t q[2][kTiles][kTileBytes];  // two chunks' query tiles: the next loads during this one
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  // Every unit runs both query tiles (rows past t_q are computed on the zero
  // rows TMA fills in and not stored), so both tiles pass the same sequence
  // of key tiles and share the K/V ring; each tile's products are issued by
  // its own MMA warp against its own barriers.
  // q_empty[i]: Q buffer i may be refilled — the chunk's last S of both
  // tiles is done and both epilogues are done with the buffer (a unit's
  // output tiles are staged there for the TMA store).
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kStages];   // the stage's K and V tiles loaded (TMA)
  uint64_t kv_empty[kStages];  // both warpgroups saw the stage's PV complete (one arrival each)
  uint64_t s_full[kTiles];  // S(t, j) in TMEM (MMA commit)
  uint64_t s_free[kTiles];  // S(t, j) read into registers: S(t, j+1) may overwrite it
  uint64_t p_full[kTiles];  // P(t, j) in TMEM and O(t) rescaled (softmax arrivals)
  uint64_t o_done[kTiles];  // PV(t, j) complete: P(t, j+1) may be written (MMA commit)
  uint64_t o_free[kTiles];  // the epilogue has read O(t): the next unit may overwrite it
  // ep_full[i][t]: every row of output tile t is staged in Q buffer i for
  // the TMA store (per buffer: a buffer is staged again only after the
  // store lane has handed it back, so no waiter falls two phases behind).
  uint64_t ep_full[2][kTiles];
  // sfu_turn[t][w]: warp w of the other warpgroup (on the same scheduler,
  // so the same SFU) has finished an exponential loop, so warp w of
  // warpgroup t may run its next one (the turns alternate, tile 0 first).
  // Per scheduler, a warp need not wait for the slowest of the other four.
  uint64_t sfu_turn[kTiles][4];
  // Split chunks (at most two per CTA, its first two): the warpgroup's
  // partial rows of chunk i are written (all its threads; completes once).
  uint64_t part_bar[kTiles][2];
  uint64_t merge_bar[kTiles];  // merge_flag[t] is set (once, for the CTA's last chunk)
  uint64_t drain;
  uint32_t tmem_base;
  int merge_flag[kTiles];      // 1: this part arrived last and merges; 0: done; -1: timed out
  int abort;
};

// Division by a run-time invariant divisor d in [1, 2^31] through a
// multiply-high (Granlund and Montgomery, "Division by invariant integers
// using multiplication", PLDI 1994): with l = ceil(log2 d) and
// mul = floor(2^32 (2^l - d) / d) + 1, x / d = (mulhi(x, mul) + x) >> l for
// every dividend x < 2^31. The persistent CTAs map unit and key-tile indices
// with it at every unit boundary.
struct FastDiv {
  uint32_t d, mul, shift;
  static FastDiv make(uint32_t d) {
    FastDiv f;
    f.d = d;
    f.shift = 0;
    while ((1ull << f.shift) < d) ++f.shift;
    f.mul = (uint32_t)((((1ull << 32) * ((1ull << f.shift) - d)) / d) + 1);
    return f;
  }
  WATTN_DEVINL uint32_t div(uint32_t x) const { return (__umulhi(x, mul) + x) >> shift; }
};

// Wait sites (kernel 1): role << 16 | barrier << 8 | iteration.
#define TC_SITE(role, bar, j) ((1 << 24) | ((role) << 16) | ((bar) << 8) | ((j) & 0xff))

struct Params {
  void *o;
  int64_t o_rs, o_bs;
  int t_q, t_kv;
  int n_qblk, n_heads, n_units;  // work units: (query block, head, utterance)
  FastDiv by_qblk, by_heads;     // divisions by n_qblk and n_heads
  float scale_log2;  // scale * log2(e)
  int causal, q_pos_offset;
  // Key-tile split schedule (0: whole units dealt round-robin). Each CTA
  // takes the next sk_tiles key tiles of the unit-major sequence of all
  // units' tiles (nkv_unit per unit); a unit cut by a CTA boundary is
  // finished by the last of its parts to arrive, which merges the others'
  // partials (part, kAttnPartFloats per slot) counted in cnt.
  int sk_tiles, nkv_unit;
  FastDiv by_tiles, by_nkv;  // divisions by sk_tiles and nkv_unit (the split schedule)
  float *part;
  int *cnt;
  int *status;
  int tma_out;   // whole units' output tiles leave through map_o (16-bit output)
  // The two softmax warpgroups take turns on the exponential loop: each
  // one's score loads, row max, P stores and epilogue then run while the
  // other's exponentials use the SFU (the two loops at once share it and
  // leave it idle in between).
  int pingpong;
  // bf16 inputs: the largest |v| of each block of the V pre-pass
  // (vmax[0..vmax_n), f32 bits) and the launch's gate: 0 none; 1 run only
  // when V fits f16 faithfully; 2 run only when it does not.
  const uint32_t *vmax;
  int vmax_n, gate;
};

// Normalises 64 accumulated dims by inv and stores them (16-byte stores).
template <typename OutT>
WATTN_DEVINL void store_row(OutT *dst, const uint32_t (&o)[2][32], float inv) {
  auto at = [&](int i) { return __uint_as_float(o[i >> 5][i & 31]) * inv; };
  if constexpr (sizeof(OutT) == 4) {
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int c = 0; c < 16; ++c) d4[c] = make_float4(at(4 * c), at(4 * c + 1), at(4 * c + 2), at(4 * c + 3));
  } else {
    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 w;
      w.x = pack2<OutT>(at(8 * c + 0), at(8 * c + 1));
      w.y = pack2<OutT>(at(8 * c + 2), at(8 * c + 3));
      w.z = pack2<OutT>(at(8 * c + 4), at(8 * c + 5));
      w.w = pack2<OutT>(at(8 * c + 6), at(8 * c + 7));
      d4[c] = w;
    }
  }
}

// Work unit u of the persistent grid: query block fastest, then head, then
// utterance, so the units running at once share their K/V rows in L2. A
// chunk is the part of a unit one CTA computes: key tiles [kv_lo, kv_lo+nkv)
// of it, part `part` of n_parts (n_parts == 1: the whole unit).
struct Unit {
  int q0, head, b, n_tiles, kv_lo, nkv;
  int parts;  // n_parts | part << 16 (n_parts == 1: the whole unit)
  int c0x;    // first CTA holding the unit << 1 | whether the unit starts inside its range
  WATTN_DEVINL int n_parts() const { return parts & 0xffff; }
  WATTN_DEVINL int part() const { return parts >> 16; }
  // Partial slot of part j: the CTA c0 + j holding it keeps two slots, its
  // first chunk's (2c) and its last chunk's (2c + 1). Part 0 is its CTA's
  // last chunk unless the unit starts exactly at that CTA's range.
  WATTN_DEVINL int slot(int j) const { return 2 * ((c0x >> 1) + j) + (j == 0 ? (c0x & 1) : 0); }
};

WATTN_DEVINL Unit unit_of(const Params &p, int u) {
  Unit w;
  const int rest = (int)p.by_qblk.div((uint32_t)u), qb = u - rest * p.n_qblk;
  w.b = (int)p.by_heads.div((uint32_t)rest);
  w.head = rest - w.b * p.n_heads;
  w.q0 = qb * (kBM * kTiles);
  w.n_tiles = kTiles;  // always both tiles (the barriers are shared by them)
  int kv_end = p.t_kv;
  if (p.causal) kv_end = min(kv_end, min(w.q0 + kBM * kTiles, p.t_q) + p.q_pos_offset);
  w.kv_lo = 0;
  w.nkv = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
  w.parts = 1;
  w.c0x = 0;
  return w;
}

// The k-th chunk of this CTA, or false past its last. Under the split
// schedule a CTA's key range [lo, hi) covers whole units and at most two cut
// ones, its first and its last; those two come first, so that their parts
// are merged while the CTA works on whole units.
WATTN_DEVINL bool chunk_at(const Params &p, int k, Unit &w) {
  if (p.sk_tiles == 0) {
    const long long u = (long long)blockIdx.x + (long long)k * gridDim.x;
    if (u >= p.n_units) return false;
    w = unit_of(p, (int)u);
    return true;
  }
  // Key-tile positions are below 2^31 (the host takes the split schedule
  // only then).
  const uint32_t T = (uint32_t)p.sk_tiles, n = (uint32_t)p.nkv_unit;
  const uint32_t lo = blockIdx.x * T;
  const uint32_t hi = min(lo + T, (uint32_t)p.n_units * n);
  if (lo >= hi) return false;
  const uint32_t u0 = p.by_nkv.div(lo), u1 = p.by_nkv.div(hi - 1);
  const int n_ch = (int)(u1 - u0 + 1);
  if (k >= n_ch) return false;
  const int cut0 = (lo != u0 * n || hi < (u0 + 1) * n) ? 1 : 0;  // first chunk is cut
  const int cut1 = (n_ch > 1 && hi != (u1 + 1) * n) ? 1 : 0;     // last chunk is cut
  int idx;  // position in key order
  if (k < cut0 + cut1)
    idx = (k == 0 && cut0) ? 0 : n_ch - 1;
  else
    idx = cut0 + (k - cut0 - cut1);
  const uint32_t u = u0 + idx, ub = u * n;
  w = unit_of(p, (int)u);
  const uint32_t a = max(lo, ub), e = min(hi, ub + n);
  w.kv_lo = (int)(a - ub);
  w.nkv = (int)(e - a);
  const uint32_t c0 = p.by_tiles.div(ub);
  w.c0x = (int)(c0 << 1) | (ub != c0 * T ? 1 : 0);
  w.parts = ((int)(p.by_tiles.div(ub + n - 1) - c0) + 1) | (((int)blockIdx.x - (int)c0) << 16);
  return true;
}

// Partial of part j, query tile t: O [64][128], then m [128] and l [128].
WATTN_DEVINL float *part_of(const Params &p, const Unit &w, int j, int t) {
  return p.part + (size_t)(w.slot(j) * kTiles + t) * kAttnPartFloats;
}

// Counts a finished part of a split unit's tile t (one thread, after the
// part's rows are written): true when it was the last of the unit's parts.
WATTN_DEVINL int count_part(const Params &p, const Unit &w, int t) {
  __threadfence();  // the part's rows, then the count (release)
  int *cnt = p.cnt + (w.c0x >> 1) * kTiles + t;
  const int last = atomicAdd(cnt, 1) == w.n_parts() - 1 ? 1 : 0;
  if (last) {
    __threadfence();     // the other parts' rows (acquire)
    atomicExch(cnt, 0);  // every launch leaves its counters at zero
  }
  return last;
}

// One output row of a split unit from all its parts' partials
// (attention.rs:228-240 over the union of the parts' keys): the offsets m of
// the parts that saw keys are rescaled to the largest.
template <typename OutT>
WATTN_DEVINL void merge_row(const Params &p, const Unit &w, int t, int row, OutT *dst) {
  constexpr int kNear = 4;  // parts whose weights stay in registers (most units have 2 to 4)
  const int np = w.n_parts();
  float mj[kNear], lj[kNear];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kNear; ++j) {
    const float *pj = part_of(p, w, j < np ? j : 0, t);
    mj[j] = __ldcg(pj + 64 * kBM + row);
    lj[j] = j < np ? __ldcg(pj + 65 * kBM + row) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < kNear; ++j)
    if (lj[j] > 0.f) mx = fmaxf(mx, mj[j]);
  for (int j = kNear; j < np; ++j) {
    const float *pj = part_of(p, w, j, t);
    if (__ldcg(pj + 65 * kBM + row) > 0.f) mx = fmaxf(mx, __ldcg(pj + 64 * kBM + row));
  }
  // part weights 2^(m_j - mx) and the merged normaliser
  float aj[kNear];
  float lsum = 0.f;
#pragma unroll
  for (int j = 0; j < kNear; ++j) {
    aj[j] = lj[j] > 0.f ? ex2(mj[j] - mx) : 0.f;
    lsum += lj[j] * aj[j];
  }
  for (int j = kNear; j < np; ++j) {
    const float *pj = part_of(p, w, j, t);
    const float l_j = __ldcg(pj + 65 * kBM + row);
    if (l_j > 0.f) lsum += l_j * ex2(__ldcg(pj + 64 * kBM + row) - mx);
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  // 32 dims at a time (the merge warp runs with few registers)
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kNear; ++j) {
      if (!(aj[j] > 0.f)) continue;
      const float *pj = part_of(p, w, j, t) + h * 32 * kBM;
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = fmaf(aj[j], __ldcg(pj + i * kBM + row), acc[i]);
    }
    for (int j = kNear; j < np; ++j) {
      const float *pj = part_of(p, w, j, t);
      const float l_j = __ldcg(pj + 65 * kBM + row);
      if (!(l_j > 0.f)) continue;
      const float a = ex2(__ldcg(pj + 64 * kBM + row) - mx);
      pj += h * 32 * kBM;
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = fmaf(a, __ldcg(pj + i * kBM + row), acc[i]);
    }
    if constexpr (sizeof(OutT) == 4) {
      float4 *d4 = reinterpret_cast<float4 *>(dst + h * 32);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        d4[c] = make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv,
                            acc[4 * c + 3] * inv);
    } else {
      uint4 *d4 = reinterpret_cast<uint4 *>(dst + h * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack2<OutT>(acc[8 * c + 0] * inv, acc[8 * c + 1] * inv);
        v.y = pack2<OutT>(acc[8 * c + 2] * inv, acc[8 * c + 3] * inv);
        v.z = pack2<OutT>(acc[8 * c + 4] * inv, acc[8 * c + 5] * inv);
        v.w = pack2<OutT>(acc[8 * c + 6] * inv, acc[8 * c + 7] * inv);
        d4[c] = v;
      }
    }
  }
}

// The roles of one CTA (TMA producer and store lane, MMA warps, merge warp,
// softmax warpgroups) over its work units, with P rounded to PV_DT and
// map_v viewing V in that type.
template <int IN_DT, int PV_DT, int OUT_DT>
WATTN_DEVINL void attn_roles(const CUtensorMap &map_q, const CUtensorMap &map_k,
                             const CUtensorMap &map_v, const CUtensorMap &map_o, const Params &p,
                             Smem &s, uint32_t tmem, volatile int *abort, int warp, int lane) {
  using PT = typename Elem<PV_DT>::T;  // the type P is rounded to (that of V)
  using OutT = typename Elem<OUT_DT>::T;
  if (warp == kTmaWarp) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      uint32_t c = 0;  // K/V ring position over all units of this CTA
      int n_units = 0;
      int last_kv = -1;  // ring position of the last stage loaded, for the wind-down
      bool ok = true;
      Unit w;
      for (int kc = 0; ok && chunk_at(p, kc, w); ++kc) {
        if (w.nkv == 0) continue;  // (every role skips such a unit alike)
        // Q buffer n_units % 2 is free once the last S of the chunk before
        // the previous one has run.
        const int qs = n_units & 1;
        if (n_units >= 2 && !mbar_wait(&s.q_empty[qs], ((n_units >> 1) - 1) & 1, abort, p.status,
                                       TC_SITE(1, 0, n_units)))
          break;
        mbar_arrive_expect_tx(&s.q_full[qs], w.n_tiles * kTileBytes);
        for (int t = 0; t < w.n_tiles; ++t)
          tma_load_4d(s.q[qs][t], &map_q, &s.q_full[qs], 0, w.head, w.q0 + t * kBM, w.b);
        for (int j = 0; j < w.nkv; ++j, ++c) {
          const int st = c % kStages;
          const uint32_t ph = (c / kStages) & 1;
          if (!mbar_wait(&s.kv_empty[st], ph ^ 1, abort, p.status, TC_SITE(1, 1, j))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.kv_full[st], 2 * kTileBytes);
          tma_load_4d(s.k[st], &map_k, &s.kv_full[st], 0, w.head, (w.kv_lo + j) * kBN, w.b);
          tma_load_4d(s.v[st], &map_v, &s.kv_full[st], 0, w.head, (w.kv_lo + j) * kBN, w.b);
          last_kv = (int)c;
        }
        ++n_units;
      }
      if (*abort) {
        // Wind-down after a timeout: let the loads still in flight land
        // before the CTA's shared memory is released (bounded waits).
        volatile int no_abort = 0;
        if (last_kv >= 0)
          mbar_wait(&s.kv_full[last_kv % kStages], (last_kv / kStages) & 1, &no_abort, p.status,
                    TC_SITE(1, 3, last_kv));
      }
    } else if (lane == 1 && p.tma_out) {
      // ---------------------------------------------------------- output stores
      // A whole unit's output tiles, staged by the softmax warpgroups in the
      // unit's Q buffer, leave with one TMA tensor store each; the buffer
      // goes back to the producer (lane 0) once the stores have read it.
      // Split parts keep the buffer untouched and hand it back themselves.
      uint32_t n_units = 0, n_st[2] = {0, 0};  // chunks; tiles stored from each buffer
      bool ok = true;
      Unit w;
      for (int kc = 0; ok && chunk_at(p, kc, w); ++kc) {
        if (w.nkv == 0) continue;
        const int qs = n_units & 1;
        ++n_units;
        if (w.n_parts() != 1) continue;
        for (int t = 0; t < kTiles; ++t) {
          if (!mbar_wait(&s.ep_full[qs][t], n_st[qs] & 1, abort, p.status, TC_SITE(1, 7 + t, kc))) {
            ok = false;
            break;
          }
          tma_store_4d(&map_o, s.q[qs][t], 0, w.head, w.q0 + t * kBM, w.b);
          bulk_commit_group();
        }
        bulk_wait_read_all();
        if (!ok) break;
        for (int t = 0; t < kTiles; ++t) mbar_arrive(&s.q_empty[qs]);
        ++n_st[qs];
      }
      bulk_wait_read_all();  // the stores have read the CTA's shared memory
    }
  } else if (warp == kMmaWarp || warp == kMma1Warp) {
    // ---------------------------------------------------------- MMA issuers
    // One warp per query tile issues that tile's tcgen05.mma: S = Q K^T into
    // its S columns, then O += P V. The tiles' products use disjoint tensor
    // memory and their own barriers, so each tile's chain (scores, softmax,
    // PV) runs at its own pace and the two softmax warpgroups need not do
    // their exponentials at the same time. (A commit tracks the products of
    // the thread that issues it.) Per key tile j the warp issues S(t, j+1)
    // as soon as the softmax has read S(t, j), then PV(t, j).
    if (lane == 0) {
      constexpr uint32_t ab = IN_DT == WATTN_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_s = idesc_f16(ab, kBM, kBN, 0, 0);  // Q, K both K-major
      constexpr uint32_t idesc_o =  // P from TMEM, V MN-major, both of V's type
          idesc_f16(PV_DT == WATTN_BF16 ? 1u : 0u, kBM, 64, 0, 1);
      // Shared-memory descriptors of the first Q, K and V tiles; a tile at
      // byte offset off has descriptor base + off / 16 (the start-address
      // field holds address / 16 in 14 bits, and shared addresses stay
      // below 2^18, so the add never carries out of the field).
      const uint64_t dq0 = smem_desc_sw128(smem_u32(s.q[0][0]), 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t dv0 = smem_desc_sw128(smem_u32(s.v[0]), 16384, 1024);
      constexpr uint32_t kTileDesc = kTileBytes >> 4;
      const int t = warp == kMmaWarp ? 0 : 1;
      const int role = 2 + 4 * t;
      const uint32_t d_s = tmem + t * 256, d_p = d_s + 128, d_o = d_s + 192;

      // Running counts (barrier phases continue across units).
      uint32_t n_s = 0, n_pv = 0, n_ep = 0;
      uint32_t c = 0;  // K/V ring position
      int n_units = 0;
      bool ok = true;
      int qs = 0;
      // S(t) for the key tile at ring position cs.
      auto s_step = [&](uint32_t cs, int j) -> bool {
        const int st = cs % kStages;
        if (!mbar_wait(&s.kv_full[st], (cs / kStages) & 1, abort, p.status, TC_SITE(role, 5, j)))
          return false;
        // S(t, j) overwrites S(t, j-1): the softmax must have read it.
        if (n_s > 0 &&
            !mbar_wait(&s.s_free[t], (n_s - 1) & 1, abort, p.status, TC_SITE(role, 7, j)))
          return false;
        tc_fence_after();
        const uint64_t dq = dq0 + (uint32_t)(qs * kTiles + t) * kTileDesc;
        const uint64_t dk = dk0 + (uint32_t)st * kTileDesc;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 4 x K=16 along the head dim (32 bytes each)
          umma_ss(d_s, dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0);
        umma_commit(&s.s_full[t]);
        ++n_s;
        return true;
      };
      Unit w;
      for (int kc = 0; ok && chunk_at(p, kc, w); ++kc) {
        if (w.nkv == 0) continue;
        qs = n_units & 1;  // Q buffer of this chunk
        if (!mbar_wait(&s.q_full[qs], (n_units >> 1) & 1, abort, p.status,
                       TC_SITE(role, 0, n_units)))
          break;
        if (!s_step(c, 0)) break;
        for (int j = 0; j < w.nkv; ++j) {
          const uint32_t cj = c + j;
          const int st = cj % kStages;
          if (j + 1 < w.nkv) {
            if (!s_step(cj + 1, j + 1)) {
              ok = false;
              break;
            }
          } else {
            umma_commit(&s.q_empty[qs]);  // the chunk's last S: its Q may be replaced
          }
          // The unit's first PV overwrites O(t): the previous unit's
          // epilogue must have read it.
          if (j == 0 && n_ep > 0 &&
              !mbar_wait(&s.o_free[t], (n_ep - 1) & 1, abort, p.status, TC_SITE(role, 9, j))) {
            ok = false;
            break;
          }
          if (!mbar_wait(&s.p_full[t], n_pv & 1, abort, p.status, TC_SITE(role, 3, j))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t dv = dv0 + (uint32_t)st * kTileDesc;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 8 x K=16 along the keys (2048 bytes each)
            umma_ts(d_o, d_p + kk * 8, dv + 128 * kk, idesc_o, j > 0 || kk > 0);
          umma_commit(&s.o_done[t]);
          ++n_pv;
        }
        ++n_ep;
        c += w.nkv;
        ++n_units;
      }
      // Drain: every MMA issued above completes before TMEM is freed (the
      // barrier completes once both warps' products are done). This wait
      // ignores `abort` (it must outlive a wind-down) but stays bounded.
      volatile int no_abort = 0;
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0, &no_abort, p.status, TC_SITE(role, 6, 0));
    }
  } else if (warp == kMergeWarp) {
    // ---------------------------------------------------------- split merges
    // The CTA's split chunks other than its last: each tile's part is
    // counted in once the softmax warpgroup has written it and, when it
    // arrived last, merged with the unit's other parts, while the softmax
    // warps go on with the next chunk.
    Unit w, nx;
    bool ok = true;
    for (int kc = 0; ok && kc < 2 && chunk_at(p, kc, w); ++kc) {
      if (w.n_parts() == 1 || !chunk_at(p, kc + 1, nx)) break;
      for (int t = 0; t < w.n_tiles; ++t) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s.part_bar[t][kc], 0, abort, p.status,
                                               TC_SITE(5, t, kc)))) {
          ok = false;
          break;
        }
        int flag = lane == 0 ? count_part(p, w, t) : 0;
        if (!__shfl_sync(0xffffffffu, flag, 0)) continue;
        OutT *out = reinterpret_cast<OutT *>(p.o) + (int64_t)w.b * p.o_bs + w.head * kHeadDim;
        for (int row = lane; row < kBM; row += 32) {
          const int qrow = w.q0 + t * kBM + row;
          if (qrow < p.t_q) merge_row<OutT>(p, w, t, row, out + (int64_t)qrow * p.o_rs);
        }
      }
    }
  } else {
    // ---------------------------------------------------------- softmax + epilogue
    const int t = warp >> 2;   // query tile of this warpgroup
    const int wq = warp & 3;   // TMEM lane quarter of this warp
    const int row = wq * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(wq * 32) << 16);
    const uint32_t t_s = lane_base + t * 256;
    const uint32_t t_p = t_s + 128, t_o = t_s + 192;
    const float c = p.scale_log2;
    uint32_t n_s = 0, n_p = 0;  // S tiles read and P tiles written by this warpgroup
    uint32_t n_ch = 0;  // chunks finished by this warpgroup
    // Key tiles whose K/V stage this warpgroup has handed back (its first
    // thread arrives once the tile's PV is seen complete).
    uint32_t n_rel = 0;
    auto release_kv = [&]() {
      if (n_p > n_rel) {
        if (wq == 0 && lane == 0) mbar_arrive(&s.kv_empty[(n_p - 1) % kStages]);
        n_rel = n_p;
      }
    };
    bool ok = true;
    Unit w;
    for (int kc = 0; ok && chunk_at(p, kc, w); ++kc) {
      if (w.nkv == 0 || t >= w.n_tiles) continue;
      const int qrow = w.q0 + t * kBM + row;
      // keys of this chunk visible to the row, counted from its first tile
      const int key_lim = (p.causal ? min(p.t_kv, qrow + p.q_pos_offset + 1) : p.t_kv) -
                          w.kv_lo * kBN;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < w.nkv; ++j, ++n_s) {
        const bool got =
            mbar_wait(&s.s_full[t], n_s & 1, abort, p.status, TC_SITE(3 + t, 0, j));
        // The whole warp takes the same branch and is converged before the
        // .sync.aligned TMEM accesses below.
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[4][32];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(t_s + q4 * 32, r[q4]);
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) reg_fence(r[q4]);
        // S(t, j) is in registers: the MMA warp may compute the next S now.
        tc_fence_before();
        mbar_arrive(&s.s_free[t]);
        float sv[128];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[q4 * 32 + i] = __uint_as_float(r[q4][i]);
        const int lim = key_lim - j * kBN;
        if (lim < kBN) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= lim) sv[i] = -INFINITY;
        }
        // Row max: four independent chains of three-input max.
        float mx4[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) mx4[a] = fmax3(sv[a * 32], sv[a * 32 + 1], sv[a * 32 + 2]);
#pragma unroll
        for (int i = 3; i < 31; i += 2)
#pragma unroll
          for (int a = 0; a < 4; ++a) mx4[a] = fmax3(mx4[a], sv[a * 32 + i], sv[a * 32 + i + 1]);
#pragma unroll
        for (int a = 0; a < 4; ++a) mx4[a] = fmaxf(mx4[a], sv[a * 32 + 31]);
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        const float mc = mx * c;
        // Lazy rescale: m only moves when the row max grows by more than
        // 2^8, so p <= 256 and l, O stay exact; O itself is rescaled below,
        // after the scores are dead (fewer live registers).
        const bool need = mc > m + kRescaleThreshold;
        const bool warp_need = __any_sync(0xffffffffu, need);
        const float alpha = need ? ex2(m - mc) : 1.f;  // 0 on the first tile (m = -inf)
        if (need) {
          l *= alpha;
          m = mc;
        }
        const float mu = (m == -INFINITY) ? 0.f : m;
        const float2 c2 = make_float2(c, c), nmu2 = make_float2(-mu, -mu);
        // P = 2^(s*c - mu), packed to 16-bit pairs (kept in registers until
        // the previous PV is done, then stored to TMEM). With bf16 P, l sums
        // the *rounded* weights the tensor core multiplies V with: they then
        // sum to exactly one and the rounding error of a dominant weight
        // cancels in acc / l. With f16 P (2^-12 relative rounding), l sums
        // the f32 weights: widening packed f16 back to f32 costs more than
        // the exponentials on B200, and the normaliser then differs from the
        // rounded weights' sum by at most 2^-12 relative.
        if (p.pingpong) {
          // Tile 0's loop k follows tile 1's loop k-1; tile 1's loop k
          // follows tile 0's loop k.
          if (t == 1 || n_s > 0) {
            const uint32_t k = t == 0 ? n_s - 1 : n_s;
            const bool turn =
                mbar_wait(&s.sfu_turn[t][wq], k & 1, abort, p.status, TC_SITE(3 + t, 8, j));
            if (!__all_sync(0xffffffffu, turn)) {
              ok = false;
              break;
            }
          }
        }
        float2 acc2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};
        uint32_t pk[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 x = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), c2, nmu2);
          float2 pv;
          if (fma_exp2_slot<PV_DT>(i)) {
            pv = exp2_fma2(x);
          } else {
            pv.x = ex2(x.x);
            pv.y = ex2(x.y);
          }
          const uint32_t wd = pack2<PT>(pv.x, pv.y);
          pk[i] = wd;
          if constexpr (PV_DT == WATTN_F16)
            acc2[i & 3] = __fadd2_rn(acc2[i & 3], pv);
          else
            acc2[i & 3] = __fadd2_rn(acc2[i & 3], unpack2<PT>(wd));
        }
        l += (acc2[0].x + acc2[0].y) + (acc2[1].x + acc2[1].y) + (acc2[2].x + acc2[2].y) +
             (acc2[3].x + acc2[3].y);
        if (p.pingpong) mbar_arrive(&s.sfu_turn[t ^ 1][wq]);
        // P may only overwrite the previous P once the PV reading it is
        // done (also across units), and O may only be rescaled once the
        // previous PV of this unit has added to it.
        if (n_p > 0) {
          const bool done =
              mbar_wait(&s.o_done[t], (n_p - 1) & 1, abort, p.status, TC_SITE(3 + t, 2, j));
          if (!__all_sync(0xffffffffu, done)) {
            ok = false;
            break;
          }
          tc_fence_after();
          release_kv();
        }
        // O rescale for the rows whose max moved. The TMEM accesses are
        // .sync.aligned, so the whole warp takes the branch when any lane
        // needs it; other lanes scale by 1.
        if (warp_need && j > 0) {
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
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t chunk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) chunk[i] = pk[q4 * 16 + i];
          tmem_st16(t_p + q4 * 16, chunk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s.p_full[t]);
        ++n_p;
      }
      if (!ok) break;
      // ---- epilogue: O(t) / l; the tile's O columns are then free for the
      // next unit's first PV.
      const bool fin = mbar_wait(&s.o_done[t], (n_p - 1) & 1, abort, p.status,
                                 TC_SITE(3 + t, 1, w.nkv));
      if (!__all_sync(0xffffffffu, fin)) {
        ok = false;
        break;
      }
      tc_fence_after();
      release_kv();
      uint32_t o[2][32];
      tmem_ld32(t_o, o[0]);
      tmem_ld32(t_o + 32, o[1]);
      tmem_wait_ld();
      reg_fence(o[0]);
      reg_fence(o[1]);
      tc_fence_before();
      mbar_arrive(&s.o_free[t]);
      const bool live = qrow < p.t_q;
      OutT *dst = reinterpret_cast<OutT *>(p.o) + (int64_t)w.b * p.o_bs + (int64_t)qrow * p.o_rs +
                  w.head * kHeadDim;
      const int qs = n_ch & 1;  // this chunk's Q buffer
      ++n_ch;
      const bool staged = w.n_parts() == 1 && p.tma_out;
      // Paths that leave the Q buffer alone hand it back at once.
      if (!staged && wq == 0 && lane == 0) mbar_arrive(&s.q_empty[qs]);
      if (staged) {
        // The normalised row goes into the unit's Q tile (its last S is
        // done), 128-byte swizzled as the output map expects (16-byte chunk
        // c of row r at chunk c ^ (r & 7)); the store lane of the TMA warp
        // then stores the whole tile (rows past t_q fall outside the map and
        // are not written) and hands the buffer back once the store has read
        // it, while this warpgroup goes on with the next unit.
        if constexpr (sizeof(OutT) == 2) {
          uint8_t *rowp = s.q[qs][t] + row * 128;
          const float inv = l > 0.f ? 1.f / l : 0.f;
          auto at = [&](int i) { return __uint_as_float(o[i >> 5][i & 31]) * inv; };
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            uint4 v4;
            v4.x = pack2<OutT>(at(8 * c8 + 0), at(8 * c8 + 1));
            v4.y = pack2<OutT>(at(8 * c8 + 2), at(8 * c8 + 3));
            v4.z = pack2<OutT>(at(8 * c8 + 4), at(8 * c8 + 5));
            v4.w = pack2<OutT>(at(8 * c8 + 6), at(8 * c8 + 7));
            *reinterpret_cast<uint4 *>(rowp + ((c8 ^ (row & 7)) << 4)) = v4;
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&s.ep_full[qs][t]);
        continue;
      }
      if (w.n_parts() == 1) {
        if (live) store_row<OutT>(dst, o, l > 0.f ? 1.f / l : 0.f);
        continue;
      }
      // ---- one part of a split unit: its partial (O, m, l of every row,
      // [value][row] so a warp's stores are contiguous) goes to its slot;
      // the part that is counted in last merges all of them.
      float *mine = part_of(p, w, w.part(), t);
      if (live) {
#pragma unroll
        for (int i = 0; i < 64; ++i) mine[i * kBM + row] = __uint_as_float(o[i >> 5][i & 31]);
        mine[64 * kBM + row] = m;
        mine[65 * kBM + row] = l;
      }
      // (split chunks are a CTA's first two, so kc is 0 or 1 here)
      mbar_arrive(&s.part_bar[t][kc]);
      {
        Unit nx;
        if (chunk_at(p, kc + 1, nx)) continue;  // the merge warp counts this part in
      }
      // The CTA's last chunk: count it in here (nothing else is left to do).
      // The warpgroup's first warp counts; the others wait for its verdict.
      // Whole warps wait (a lane spinning on a barrier would hold back a lane
      // of its warp that runs another path).
      int flag = -1;
      if (wq == 0) {
        const bool got = __all_sync(
            0xffffffffu, mbar_wait(&s.part_bar[t][kc], 0, abort, p.status, TC_SITE(3 + t, 4, kc)));
        if (got && lane == 0) flag = count_part(p, w, t);
        flag = __shfl_sync(0xffffffffu, flag, 0);
        if (lane == 0) {
          s.merge_flag[t] = flag;
          mbar_arrive(&s.merge_bar[t]);
        }
      } else if (mbar_wait(&s.merge_bar[t], 0, abort, p.status, TC_SITE(3 + t, 5, kc))) {
        flag = *reinterpret_cast<volatile int *>(&s.merge_flag[t]);
      }
      if (!__all_sync(0xffffffffu, flag >= 0)) {
        ok = false;
        break;
      }
      if (flag == 1 && live) merge_row<OutT>(p, w, t, row, dst);
    }
  }

}

// map_v views V in PV_DT: the caller's V, or (bf16 inputs, PV_DT f16) its
// f16 copy.
template <int IN_DT, int PV_DT, int OUT_DT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v,
                       const __grid_constant__ CUtensorMap map_o, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      // a commit from each tile's MMA warp and an arrival from each epilogue
      mbar_init(&s.q_empty[i], 2 * kTiles);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], kTiles);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&s.s_full[t], 1);
      mbar_init(&s.s_free[t], kBM);
      mbar_init(&s.p_full[t], kBM);
      mbar_init(&s.o_done[t], 1);
      mbar_init(&s.o_free[t], kBM);
      mbar_init(&s.ep_full[0][t], kBM);
      mbar_init(&s.ep_full[1][t], kBM);
      for (int q = 0; q < 4; ++q) mbar_init(&s.sfu_turn[t][q], 32);
      mbar_init(&s.part_bar[t][0], kBM);
      mbar_init(&s.part_bar[t][1], kBM);
      mbar_init(&s.merge_bar[t], 1);
    }
    mbar_init(&s.drain, kTiles);  // one commit from each MMA warp
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The set-up above overlaps the end of the previous kernel in the stream
  // (launched with programmatic serialisation); global memory is read and
  // written only after it has completed. The next launch may start its own
  // set-up as this grid's CTAs retire.
  grid_dep_wait();
  grid_dep_launch();
  // bf16 inputs: two launches follow the V pre-pass, one per type of P and
  // V; the gate (a uniform decision on the pre-pass's block maxima) lets the
  // f16 one run when every block's largest |v| lies within f16's faithful
  // range, the bf16 one otherwise. A launch that does not run frees its
  // tensor memory and returns.
  if (p.gate != 0) {
    bool big = false, some = false;  // a block's largest |v| beyond f16 / at least 2^-6
    for (int i = threadIdx.x; i < p.vmax_n; i += kThreads) {
      const float m = __uint_as_float(__ldcg(p.vmax + i));
      big = big || !(m <= 65280.0f);
      some = some || m >= 0.015625f;
    }
    const bool fits = !__syncthreads_or(big) && __syncthreads_or(some);
    if (fits != (p.gate == 1)) {
      tc_fence_before();
      __syncthreads();
      if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(s.tmem_base, kTmemCols);
      }
      return;
    }
  }
  const uint32_t tmem = s.tmem_base;
  attn_roles<IN_DT, PV_DT, OUT_DT>(map_q, map_k, map_v, map_o, p, s, tmem, &s.abort, warp, lane);

  // Teardown: after the last TMEM access of every warp, free the columns.
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- V pre-pass
// bf16 inputs: V is copied to f16, contiguous [batch][t_kv][width], by a
// bandwidth-bound pass (each warp converts one row at a time, 16 bytes per
// lane, so a warp reads and writes 512 contiguous bytes); every block also
// writes its largest |v| (f32 bits) to vmax[blockIdx.x], the attention
// launches' gate. A NaN is passed over (it stays NaN in f16 as in bf16).
constexpr int kVConvThreads = 256;
constexpr int kVConvMaxBlocks = 1024;

__global__ void __launch_bounds__(kVConvThreads)
    v_to_f16_kernel(const uint4 *__restrict__ v, int64_t rs16, int64_t bs16, int t_kv, int rows,
                    int cpr, uint4 *__restrict__ out, uint32_t *__restrict__ vmax) {
  grid_dep_wait();
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kVConvThreads / 32;
  float mx = 0.f;
  for (int r = blockIdx.x * kWarps + warp; r < rows; r += gridDim.x * kWarps) {
    const int b = r / t_kv, t = r - b * t_kv;
    const uint4 *src = v + b * bs16 + t * rs16;
    uint4 *dst = out + (int64_t)r * cpr;
#pragma unroll 4
    for (int c = lane; c < cpr; c += 32) {
      uint4 x = __ldcs(src + c);
      uint32_t *wd = reinterpret_cast<uint32_t *>(&x);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = __uint_as_float(wd[e] << 16), hi = __uint_as_float(wd[e] & 0xffff0000u);
        mx = fmax3(mx, fabsf(lo), fabsf(hi));
        wd[e] = pack2<__half>(lo, hi);
      }
      dst[c] = x;
    }
  }
  __shared__ uint32_t wmax[kWarps];
  const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
  if (lane == 0) wmax[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bm = 0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) bm = max(bm, wmax[i]);
    vmax[blockIdx.x] = bm;
  }
}

template <int IN_DT, int PV_DT, int OUT_DT>
int launch_typed(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                 const CUtensorMap &mo, const Params &p, cudaStream_t stream) {
  auto kern = attn_fwd_tc_kernel<IN_DT, PV_DT, OUT_DT>;
  const int smem = (int)sizeof(Smem) + 1024;
  // Per device and idempotent; cheap enough to repeat on every launch.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(attn_fwd_tc)");
  // Persistent grid: one CTA per SM (the shared memory allows no second),
  // each walking units blockIdx.x, blockIdx.x + gridDim.x, ...
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return check_launch("attn_fwd_tc: device query");
  int n_ctas = std::min(p.n_units, n_sm);
  if (p.sk_tiles > 0)
    n_ctas = (int)(((long long)p.n_units * p.nkv_unit + p.sk_tiles - 1) / p.sk_tiles);
  if (launch_pdl(kern, dim3(n_ctas), dim3(kThreads), smem, stream, mq, mk, mv, mo, p) !=
      cudaSuccess)
    return check_launch("attn_fwd_tc (launch)");
  return check_launch("attn_fwd_tc");
}

int make_qkv_map(CUtensorMap *map, const void *base, int dt, int n_heads, int t, int batch,
                 int64_t rs, int64_t bs) {
  const uint64_t es = elem_size(dt);
  const uint64_t dims[4] = {64, (uint64_t)n_heads, (uint64_t)t, (uint64_t)batch};
  const uint64_t strides[3] = {64 * es, (uint64_t)rs * es,
                               (uint64_t)(batch > 1 ? bs : (int64_t)t * rs) * es};
  const uint32_t box[4] = {64, 1, kBM, 1};
  return encode_tmap(map, tmap_dtype(dt), 4, base, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

// Cost model in key-tile times, fitted to B200 timings of both schedules:
// every chunk (a unit, or a part of one) costs about 1.2 tiles more than its
// key tiles (Q, the first scores, the epilogue). Parts are merged by one
// warp, about five tiles after the part arrives, unseen while the CTA has
// whole units left to compute: with fewer than 2.5 units of key tiles per
// CTA the merges (or the softmax warps' own merge of the CTA's last chunk)
// add about four tiles to the end. The split schedule is taken when it is
// predicted to save 7 %.
int plan_attn_split(long long n_units, int nkv, int n_sm, int causal) {
  if (causal || n_units <= 0 || nkv <= 0 || n_sm <= 0) return 0;
  const long long tiles = n_units * nkv;
  if (tiles > INT_MAX || n_units % n_sm == 0) return 0;
  const double c = 1.2;
  const long long waves = (n_units + n_sm - 1) / n_sm;
  const double whole = (double)waves * (nkv + c);
  const long long T = (tiles + n_sm - 1) / n_sm;
  const long long chunks = (T + nkv - 1) / nkv + 1;  // at most, per CTA
  const double tail = T < 2.5 * nkv ? 4.0 : 1.0;
  const double split = (double)T + (double)chunks * c + tail;
  return split < 0.93 * whole ? (int)T : 0;
}

size_t attn_split_workspace_bytes(int n_sm) {
  return kCounterBytes + (size_t)2 * n_sm * kTiles * kAttnPartFloats * sizeof(float);
}

// [split counters and partials][bf16 inputs: V's f16 copy][its block maxima]
static size_t v_copy_offset(int n_sm) { return round_up_256(attn_split_workspace_bytes(n_sm)); }

size_t attn_workspace_bytes(int in_dtype, int batch, int t_kv, int n_heads, int n_sm) {
  size_t n = v_copy_offset(n_sm);
  if (in_dtype == WATTN_BF16)
    n += round_up_256((size_t)batch * t_kv * n_heads * kHeadDim * 2) +
         kVConvMaxBlocks * sizeof(uint32_t);
  return n;
}

int launch_attn_tc(const void *q, const void *k, const void *v, void *o, int in_dtype,
                   int out_dtype, int batch, int t_q, int t_kv, int n_heads, int64_t q_rs,
                   int64_t kv_rs, int64_t o_rs, int64_t q_bs, int64_t kv_bs, int64_t o_bs,
                   float scale, int causal, int q_pos_offset, cudaStream_t stream,
                   void *split_ws, size_t split_ws_bytes) {
  CUtensorMap mq, mk, mv, mo, mv16;
  int rc;
  if ((rc = make_qkv_map(&mq, q, in_dtype, n_heads, t_q, batch, q_rs, q_bs)) != WATTN_OK) return rc;
  if ((rc = make_qkv_map(&mk, k, in_dtype, n_heads, t_kv, batch, kv_rs, kv_bs)) != WATTN_OK) return rc;
  if ((rc = make_qkv_map(&mv, v, in_dtype, n_heads, t_kv, batch, kv_rs, kv_bs)) != WATTN_OK) return rc;
  // 16-bit output tiles leave through a TMA store (same view as Q); f32
  // output, or an output the map cannot describe, is stored row by row.
  int tma_out = 0;
  mo = mq;
  if (out_dtype != WATTN_F32) {
    if (make_qkv_map(&mo, o, out_dtype, n_heads, t_q, batch, o_rs, o_bs) == WATTN_OK) {
      tma_out = 1;
    } else {
      clear_error();
      mo = mq;
    }
  }
  Params p;
  p.o = o;
  p.o_rs = o_rs;
  p.o_bs = o_bs;
  p.t_q = t_q;
  p.t_kv = t_kv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.q_pos_offset = q_pos_offset;
  p.n_qblk = (t_q + kBM * kTiles - 1) / (kBM * kTiles);
  p.n_heads = n_heads;
  p.by_qblk = FastDiv::make((uint32_t)p.n_qblk);
  p.by_heads = FastDiv::make((uint32_t)n_heads);
  const long long n_units = (long long)p.n_qblk * n_heads * batch;
  if (n_units > INT_MAX)
    return set_error(WATTN_ERR_INVALID, "attention: %lld work units exceed 2^31", n_units);
  p.n_units = (int)n_units;
  p.status = device_status_ptr();
  if (p.status == nullptr) return WATTN_ERR_CUDA;
  p.tma_out = tma_out;
  p.pingpong = 1;
  // Key-tile split schedule when whole units would leave SMs idle at the end
  // (few utterances or heads per GPU).
  p.sk_tiles = 0;
  p.nkv_unit = (t_kv + kBN - 1) / kBN;
  p.by_tiles = FastDiv::make(1);
  p.by_nkv = FastDiv::make((uint32_t)p.nkv_unit);
  p.part = nullptr;
  p.cnt = nullptr;
  p.vmax = nullptr;
  p.vmax_n = 0;
  p.gate = 0;
  int dev = 0, n_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return check_launch("attn_fwd_tc: device query");
  // bf16 inputs need the workspace for V's f16 copy: the caller's, which
  // must then hold it, or the calling thread's.
  const bool conv_v = in_dtype == WATTN_BF16;
  const size_t ws_need = attn_workspace_bytes(in_dtype, batch, t_kv, n_heads, n_sm);
  uint8_t *wsb = reinterpret_cast<uint8_t *>(split_ws);
  if (conv_v) {
    if (wsb != nullptr && split_ws_bytes < ws_need)
      return set_error(WATTN_ERR_INVALID,
                       "attention: a workspace of %zu bytes is needed for bf16 inputs (%zu given)",
                       ws_need, split_ws_bytes);
    if (wsb == nullptr) {
      wsb = reinterpret_cast<uint8_t *>(thread_workspace(ws_need, stream));
      if (wsb == nullptr) return set_error(WATTN_ERR_NOMEM, "attention workspace allocation failed");
    }
  }
  const int T = plan_attn_split(n_units, p.nkv_unit, n_sm, causal);
  if (T > 0) {
    const long long n_ctas = ((long long)n_units * p.nkv_unit + T - 1) / T;
    const size_t need = attn_split_workspace_bytes((int)n_ctas);
    void *ws = wsb;
    if (ws != nullptr && split_ws != nullptr && split_ws_bytes < need)
      ws = nullptr;  // too small: whole units
    if (ws != nullptr && split_ws != nullptr) {
      // a caller's buffer: the counters this launch uses start at zero
      if (cudaMemsetAsync(ws, 0, (size_t)n_ctas * kTiles * sizeof(int), stream) != cudaSuccess)
        return check_launch("attn_fwd_tc: counter reset");
    } else if (ws == nullptr && split_ws == nullptr) {
      ws = thread_workspace(need, stream);
    }
    if (ws != nullptr) {
      p.sk_tiles = T;
      p.by_tiles = FastDiv::make((uint32_t)T);
      p.cnt = reinterpret_cast<int *>(ws);
      p.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ws) + kCounterBytes);
    }
  }
  if (in_dtype == WATTN_F16) {
    if (out_dtype == WATTN_F32)
      return launch_typed<WATTN_F16, WATTN_F16, WATTN_F32>(mq, mk, mv, mo, p, stream);
    return launch_typed<WATTN_F16, WATTN_F16, WATTN_F16>(mq, mk, mv, mo, p, stream);
  }
  // bf16: V's f16 copy and its block maxima, then the two gated launches:
  // the bf16 one first (it finds nothing to do in the usual case, and its
  // set-up overlaps the pre-pass's end), then the f16 one.
  const long long rows = (long long)batch * t_kv;
  if (rows > INT_MAX) return set_error(WATTN_ERR_INVALID, "attention: batch * t_kv exceeds 2^31");
  const int width = n_heads * kHeadDim;
  uint8_t *v16 = wsb + v_copy_offset(n_sm);
  uint32_t *vmax = reinterpret_cast<uint32_t *>(v16 + round_up_256((size_t)rows * width * 2));
  const int n_blk = (int)std::min<long long>(
      std::min<long long>(kVConvMaxBlocks, (long long)n_sm * (2048 / kVConvThreads)),
      (rows + kVConvThreads / 32 - 1) / (kVConvThreads / 32));
  if (launch_pdl(v_to_f16_kernel, dim3(n_blk), dim3(kVConvThreads), 0, stream,
                 reinterpret_cast<const uint4 *>(v), (int64_t)(kv_rs / 8),
                 (int64_t)(batch > 1 ? kv_bs / 8 : 0), t_kv, (int)rows, width / 8,
                 reinterpret_cast<uint4 *>(v16), vmax) != cudaSuccess)
    return check_launch("v_to_f16 (launch)");
  if ((rc = make_qkv_map(&mv16, v16, WATTN_F16, n_heads, t_kv, batch, width,
                         (int64_t)t_kv * width)) != WATTN_OK)
    return rc;
  p.vmax = vmax;
  p.vmax_n = n_blk;
  Params pb = p;
  pb.gate = 2;
  p.gate = 1;
  if (out_dtype == WATTN_F32) {
    rc = launch_typed<WATTN_BF16, WATTN_BF16, WATTN_F32>(mq, mk, mv, mo, pb, stream);
    if (rc == WATTN_OK) rc = launch_typed<WATTN_BF16, WATTN_F16, WATTN_F32>(mq, mk, mv16, mo, p, stream);
    return rc;
  }
  rc = launch_typed<WATTN_BF16, WATTN_BF16, WATTN_BF16>(mq, mk, mv, mo, pb, stream);
  if (rc == WATTN_OK) rc = launch_typed<WATTN_BF16, WATTN_F16, WATTN_BF16>(mq, mk, mv16, mo, p, stream);
  return rc;
}

}  // namespace wattn
