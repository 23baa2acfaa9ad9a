// Past-only beam descent over the segment tree (reference: seg.py:44-70 tree_pass, fastseg.py:254-271
// tree_pass_fast), one warp per query.
//
// Reference rule, per level l from Lm down to the leaf level L0: the candidates are the children of the
// nodes kept at level l+1 plus the newly available past-only subtree (t>>l)-1 when bit l of t is set;
// each is scored q . S_l[c] / 2^l and the best `wmax` are kept; at the leaf level the kept leaves are
// returned best first. (With leaf blocks of 2^L0 tokens this is the reference's tree_pass on the level-
// shifted tree S'[l'] = S[l'+L0-1]: all candidates of a level share one scale, so the order is unchanged.)
//
// Two facts let the kernel skip work without changing the result:
//  * While a level's reachable set R(l) has at most wmax nodes, every node of it is kept, whatever the
//    scores. R(l) is then the contiguous range [a_l, t>>l) with a_l = ((t>>Lm) - bit_Lm(t)) << (Lm-l), so
//    the first level that needs a real top-k, l*, has R(l*) = a contiguous range of <= 2*wmax+1 nodes.
//  * Below l* the candidates are the 2 adjacent children of each kept node plus the injected node.
// Ties are broken by the smaller node id (torch.topk leaves the tie order undefined; parity tests exclude
// queries whose reference scores tie at a cut).
#pragma once
#include "levels.cuh"

namespace ta {

constexpr int WMAX_LIMIT = 64;                  // largest supported wmax
constexpr int CAND_LIMIT = 2 * WMAX_LIMIT + 1;  // largest candidate list of one level

// Per-warp shared scratch of one descent (the staged node rows live in a separate, host-sized buffer of
// (2*wmax+1) * DH floats).
struct __align__(16) DescentScratch {
  float qf[128];  // the query in fp32 (first DH entries), written by the caller before a descent
  unsigned long long ckey[CAND_LIMIT];  // order key of each scored candidate (see order_key)
  int cid[CAND_LIMIT];
  float csc[CAND_LIMIT];
  int kid[WMAX_LIMIT];
  float ksc[WMAX_LIMIT];
};

// One unsigned 64-bit key per candidate whose order is the library's total order on (score, id): higher score
// first (scores mapped monotonically to unsigned, NaN as -inf), then the smaller node id.
__device__ __forceinline__ unsigned long long order_key(float s, int id) {
  uint32_t u = __float_as_uint(rank_key(s));
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(0x7fffffff - id);
}

// Staged node rows are padded to DH + 4 floats so that 8 lanes reading 8 different rows at the same column hit
// 8 different bank groups (conflict-free lane-per-candidate scoring).
template <int DH> __host__ __device__ constexpr int stage_row_floats() { return DH + 4; }

__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Exact 2^-l as a float (l < 127).
__device__ __forceinline__ float pow2_neg(int l) { return __int_as_float((127 - l) << 23); }

template <int DH>
struct Descent {
  static constexpr int G = DH / 4;                      // 16-byte chunks per node row
  static constexpr int SROW = stage_row_floats<DH>();  // staged row stride (floats)

  // Async-copy the contiguous node rows [a, a+n) of one level into stage rows [r0, r0+n).
  static __device__ __forceinline__ void stage_range(const float* __restrict__ lvl, int a, int n, float* stage,
                                                     int r0, int lane) {
    const float* src = lvl + (int64_t)a * DH;
    for (int x = lane; x < n * G; x += 32) {
      const int r = x / G, cc = x - (x / G) * G;
      cp_async16(stage + (size_t)(r0 + r) * SROW + cc * 4, src + (size_t)x * 4);
    }
  }

  // Async-copy the rows of candidates sc.cid[0..n) into stage rows [0, n).
  static __device__ __forceinline__ void stage_gather(const float* __restrict__ lvl, int n, const DescentScratch& sc,
                                                      float* stage, int lane) {
    for (int x = lane; x < n * G; x += 32) {
      const int j = x / G, cc = x - (x / G) * G;
      cp_async16(stage + (size_t)j * SROW + cc * 4, lvl + (int64_t)sc.cid[j] * DH + cc * 4);
    }
  }

  // Score candidates 0..n-1 (candidate j's row = stage + row_of(j) * SROW) into sc.csc: one lane per candidate,
  // the query read from sc.qf by broadcast.
  template <typename RowFn>
  static __device__ __forceinline__ void score(int n, float scale, DescentScratch& sc, const float* stage,
                                               RowFn row_of, int lane) {
    for (int base = 0; base < n; base += 32) {
      const int j = base + lane;
      if (j < n) {
        const float* row = stage + (size_t)row_of(j) * SROW;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int cc = 0; cc < G; ++cc) {
          const float4 qv = *reinterpret_cast<const float4*>(sc.qf + cc * 4);
          const float4 v = *reinterpret_cast<const float4*>(row + cc * 4);
          if (cc & 1) {
            a1 = fmaf(qv.x, v.x, a1); a1 = fmaf(qv.y, v.y, a1); a1 = fmaf(qv.z, v.z, a1); a1 = fmaf(qv.w, v.w, a1);
          } else {
            a0 = fmaf(qv.x, v.x, a0); a0 = fmaf(qv.y, v.y, a0); a0 = fmaf(qv.z, v.z, a0); a0 = fmaf(qv.w, v.w, a0);
          }
        }
        const float v = (a0 + a1) * scale;
        sc.csc[j] = v;
        sc.ckey[j] = order_key(v, sc.cid[j]);
      }
    }
    __syncwarp();
  }

  // Keep the best `keep` of the n scored candidates, best first, into sc.kid / sc.ksc. Returns the count.
  // Lane j owns candidates j, j+32, ... (R per lane); a candidate's rank = how many keys beat it, counted over
  // broadcast shared-memory reads of all n keys.
  template <int R>
  static __device__ __forceinline__ void topk_r(int n, int keep, DescentScratch& sc, int lane) {
    unsigned long long mine[R];
    int rank[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int j = r * 32 + lane;
      mine[r] = j < n ? sc.ckey[j] : 0ull;
      rank[r] = 0;
    }
#pragma unroll 8
    for (int i = 0; i < n; ++i) {
      const unsigned long long ki = sc.ckey[i];
#pragma unroll
      for (int r = 0; r < R; ++r) rank[r] += ki > mine[r] ? 1 : 0;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int j = r * 32 + lane;
      if (j < n && rank[r] < keep) {
        sc.kid[rank[r]] = sc.cid[j];
        sc.ksc[rank[r]] = sc.csc[j];
      }
    }
  }

  static __device__ __forceinline__ int topk(int n, int keep, DescentScratch& sc, int lane) {
    switch ((n + 31) >> 5) {
      case 0: break;
      case 1: topk_r<1>(n, keep, sc, lane); break;
      case 2: topk_r<2>(n, keep, sc, lane); break;
      case 3: topk_r<3>(n, keep, sc, lane); break;
      case 4: topk_r<4>(n, keep, sc, lane); break;
      default: topk_r<5>(n, keep, sc, lane); break;
    }
    __syncwarp();
    return n < keep ? n : keep;
  }

  // Where the descent starts (see run()): l* = -1 when every reachable leaf is kept without scoring.
  struct Plan {
    int lstar;  // first level that needs a real top-k, -1 if none
    int astar;  // first reachable node of level l* (or of L0 when lstar < 0)
    int lp;     // lowest level whose whole reachable range is prefetched
  };

  // max_levels: how many levels from l* down may be prefetched (the rest are gathered level by level, only the
  // children the descent keeps)
  static __device__ __forceinline__ Plan plan(const LevelView& lv, int t, int wmax, int stage_rows,
                                              int max_levels = 64) {
    const int Lm = lv.Lm, L0 = lv.L0;
    const int eLm = t >> Lm;
    const int aLm = eLm - (eLm & 1);
    Plan pl{-1, aLm << (Lm - L0), L0};
    for (int l = Lm; l >= L0; --l) {
      const int e = t >> l, a = aLm << (Lm - l);
      if (e - a > wmax) {
        pl.lstar = l;
        pl.astar = a;
        break;
      }
    }
    if (pl.lstar >= 0) {
      int rows = 0;
      pl.lp = pl.lstar;
      for (int l = pl.lstar; l >= L0 && l > pl.lstar - max_levels; --l) {
        const int n_l = (t >> l) - (pl.astar << (pl.lstar - l));
        if (rows + n_l > stage_rows) break;
        rows += n_l;
        pl.lp = l;
      }
    }
    return pl;
  }

  // Issue (do not wait for) the async copies of the prefetched levels: [a_l, t >> l) for l in [lp, l*], packed
  // from stage row 0. With lstar < 0 the leaf level's reachable range is staged when `need_l0` (it is scored).
  static __device__ __forceinline__ void prefetch(const float* __restrict__ nodes_bh, const LevelView& lv, int t,
                                                  const Plan& pl, bool need_l0, float* stage, int lane) {
    if (pl.lstar < 0) {
      const int n = (t >> lv.L0) - pl.astar;
      if (need_l0 && n > 0) stage_range(nodes_bh + (int64_t)lv.off[lv.L0] * DH, pl.astar, n, stage, 0, lane);
      return;
    }
    int rows = 0;
    for (int l = pl.lstar; l >= pl.lp; --l) {
      const int a_l = pl.astar << (pl.lstar - l);
      const int n_l = (t >> l) - a_l;
      stage_range(nodes_bh + (int64_t)lv.off[l] * DH, a_l, n_l, stage, rows, lane);
      rows += n_l;
    }
  }

  // The descent proper, after prefetch() completed (cp_async_wait_all + __syncwarp) and sc.qf holds the query.
  // Returns the number of kept leaves; sc.kid[0..nk) holds the leaf ids. If `sorted_out` or if more leaves are
  // reachable than `keep_last`, the leaf level is scored and the ids are best first with scores in sc.ksc;
  // otherwise (everything reachable is kept) they are in ascending order and sc.ksc is not written.
  static __device__ int select(const float* __restrict__ nodes_bh, const LevelView& lv, int t, const Plan& pl,
                               int wmax, int keep_last, bool sorted_out, DescentScratch& sc, float* stage, int lane) {
    const int L0 = lv.L0;
    if (pl.lstar < 0) {
      const int a = pl.astar, e = t >> L0;
      const int n = e - a;
      for (int j = lane; j < n; j += 32) sc.cid[j] = a + j;
      __syncwarp();
      if (n > 0 && (sorted_out || n > keep_last)) {
        score(n, pow2_neg(L0), sc, stage, [](int j) { return j; }, lane);
        return topk(n, keep_last, sc, lane);
      }
      for (int j = lane; j < n; j += 32) sc.kid[j] = a + j;
      __syncwarp();
      return n;
    }
    const int lstar = pl.lstar, astar = pl.astar;
    int nk;
    int seg = 0;  // stage row of the first node of the current prefetched level
    {
      const int n = (t >> lstar) - astar;
      for (int j = lane; j < n; j += 32) sc.cid[j] = astar + j;
      __syncwarp();
      score(n, pow2_neg(lstar), sc, stage, [](int j) { return j; }, lane);
      nk = topk(n, lstar == L0 ? keep_last : wmax, sc, lane);
      seg = n;
    }
    for (int l = lstar - 1; l >= L0; --l) {
      const int bit = (t >> l) & 1;
      for (int i = lane; i < nk; i += 32) {
        const int m = sc.kid[i];
        sc.cid[2 * i] = 2 * m;
        sc.cid[2 * i + 1] = 2 * m + 1;
      }
      if (bit && lane == 0) sc.cid[2 * nk] = (t >> l) - 1;
      __syncwarp();
      const int n = 2 * nk + bit;
      if (l >= pl.lp) {
        const int base = seg - (astar << (lstar - l));  // row of node m = base + m
        score(n, pow2_neg(l), sc, stage, [&](int j) { return base + sc.cid[j]; }, lane);
        seg += (t >> l) - (astar << (lstar - l));
      } else {
        stage_gather(nodes_bh + (int64_t)lv.off[l] * DH, n, sc, stage, lane);
        cp_async_wait_all();
        __syncwarp();
        score(n, pow2_neg(l), sc, stage, [](int j) { return j; }, lane);
      }
      nk = topk(n, l == L0 ? keep_last : wmax, sc, lane);
    }
    return nk;
  }

  // plan + prefetch + wait + select. The query must be in sc.qf (fp32) before the call.
  static __device__ int run(const float* __restrict__ nodes_bh, const LevelView& lv, int t, int wmax, int keep_last,
                            bool sorted_out, DescentScratch& sc, float* stage, int stage_rows, int lane) {
    const Plan pl = plan(lv, t, wmax, stage_rows);
    prefetch(nodes_bh, lv, t, pl, true, stage, lane);
    cp_async_wait_all();
    __syncwarp();
    return select(nodes_bh, lv, t, pl, wmax, keep_last, sorted_out, sc, stage, lane);
  }
};

// Widen a query row into the descent scratch (sc.qf) with a warp.
template <typename QT, int DH>
__device__ __forceinline__ void load_qf(const QT* __restrict__ q, DescentScratch& sc, int lane) {
  for (int d = lane; d < DH; d += 32) sc.qf[d] = to_f32(q[d]);
  __syncwarp();
}

// ------------------------------------------------------------------------------------------------ select kernel
struct SelectParams {
  const void* q;             // (B, H, Nq, dh), element strides below, unit stride in dh
  int64_t q_sb, q_sh, q_st;
  const int64_t* tq;         // position of query (b, n) = tq[b*tq_sb + n*tq_st]
  int64_t tq_sb, tq_st;
  LevelView lv;
  int B, H, Nq;
  int wmax, wl;              // beam width; output slots per query
  int64_t* ids;              // (B, H, Nq, wl) leaf ids, best first; invalid slots 0
  uint8_t* vld;              // (B, H, Nq, wl)
  float* sct;                // (B, H, Nq, wl) scores q.S/2^L0 (-inf in invalid slots); may be null
};

template <typename QT, int DH>
__global__ void __launch_bounds__(128) select_kernel(SelectParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int stage_floats = (2 * p.wmax + 1) * stage_row_floats<DH>();
  DescentScratch* scr = reinterpret_cast<DescentScratch*>(smem_raw);
  float* stage_base = reinterpret_cast<float*>(smem_raw + sizeof(DescentScratch) * nwarps);
  DescentScratch& sc = scr[warp];
  float* stage = stage_base + (size_t)warp * stage_floats;

  const int64_t qid = (int64_t)blockIdx.x * nwarps + warp;
  const int64_t nq_total = (int64_t)p.B * p.H * p.Nq;
  if (qid >= nq_total) return;
  const int n = (int)(qid % p.Nq);
  const int bh = (int)(qid / p.Nq);
  const int b = bh / p.H, h = bh % p.H;
  const int64_t tt = p.tq[b * p.tq_sb + n * p.tq_st];
  const size_t obase = (size_t)qid * p.wl;
  if (tt < 0 || tt >= p.lv.cap) {
    if (lane == 0) record_error(DEV_POS_RANGE, K_SELECT, (int)tt, p.lv.cap);
    for (int i = lane; i < p.wl; i += 32) {
      p.ids[obase + i] = 0;
      p.vld[obase + i] = 0;
      if (p.sct) p.sct[obase + i] = -INFINITY;
    }
    return;
  }
  const int t = (int)tt;
  load_qf<QT, DH>(reinterpret_cast<const QT*>(p.q) + b * p.q_sb + h * p.q_sh + n * p.q_st, sc, lane);
  const float* nodes_bh = p.lv.nodes + b * p.lv.s_b + h * p.lv.s_h;
  const int nk = Descent<DH>::run(nodes_bh, p.lv, t, p.wmax, p.wmax, true, sc, stage, 2 * p.wmax + 1, lane);
  for (int i = lane; i < p.wl; i += 32) {
    const bool ok = i < nk;
    p.ids[obase + i] = ok ? sc.kid[i] : 0;
    p.vld[obase + i] = ok ? 1 : 0;
    if (p.sct) p.sct[obase + i] = ok ? sc.ksc[i] : -INFINITY;
  }
}

// ------------------------------------------------------------------------------------------------ tile select
// Whole-sequence descent for 128 queries of one (b, h) per CTA (prefill / select_seg on long sequences). The
// warp-per-query kernel above reads every candidate's node row from L2 and spends most of its instructions on
// per-level scoring and ranking; here the CTA scores each level DENSELY once for all its queries - every node of
// the level in the past of the tile's last query, against all 128 queries - as a small fp32 FMA GEMM on
// shared-memory tiles, and then each thread (one query) descends on its candidates' scores read from shared
// memory, keeping its beam in registers.
//  * The dot products accumulate in exactly the order of Descent::score (even 4-element chunks into one sum, odd
//    chunks into another, in element order, then (a0 + a1) * 2^-l), so scores are bit-identical to the warp
//    kernel's, and so is the selection (same (score, smaller id) order through the same 64-bit keys).
//  * A level whose candidates all fit the beam (every query of the warp) keeps them without ranking; otherwise the
//    best w of the 2*nk + 1 candidate keys are found by fully unrolled bitonic networks on register arrays
//    (compare-exchange on 64-bit keys: the order is a total order, so the networks' result is exact).
constexpr int TS_QT = 128;       // queries per CTA = threads
constexpr int TS_THREADS = 128;  // GEMM: thread = 4 node rows x 8 queries of a 32-row block
constexpr int TS_RB = 32;        // node rows per staged block
constexpr int TS_RMAX = 128;     // largest level (nodes: cap >> L0) the score table may hold
constexpr int TS_WMAX = 16;      // largest beam the register list holds

// rmax = nodes of the leaf level (cap >> L0), the largest level
template <int DH>
__host__ __device__ inline size_t select_tile_smem_bytes(int rmax) {
  return (size_t)DH * TS_QT * 4                  // qT[d][q]
         + (size_t)DH * (TS_RB + 4) * 4          // nodeT[d][r] of one block (padded rows)
         + (size_t)rmax * TS_QT * 4;             // S[r][q] of one level
}

__device__ __forceinline__ int key_id(unsigned long long k) { return 0x7fffffff - (int)(uint32_t)k; }
__device__ __forceinline__ float key_score(unsigned long long k) {
  uint32_t u = (uint32_t)(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}

// Compare-exchange networks on register arrays of 64-bit keys (indices are compile-time after unrolling).
__device__ __forceinline__ void cswap(unsigned long long& a, unsigned long long& b, bool desc) {
  const bool sw = desc ? (a < b) : (a > b);
  const unsigned long long x = sw ? b : a, y = sw ? a : b;
  a = x;
  b = y;
}

// Sort a bitonic sequence of N keys (descending if desc).
template <int N>
__device__ __forceinline__ void bitonic_merge(unsigned long long* v, bool desc) {
#pragma unroll
  for (int j = N / 2; j > 0; j >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i)
      if ((i & j) == 0) cswap(v[i], v[i + j], desc);
}

// Sort N keys (N a power of two; descending if desc).
template <int N>
__device__ __forceinline__ void bitonic_sort(unsigned long long* v, bool desc) {
#pragma unroll
  for (int k = 2; k <= N; k <<= 1)
#pragma unroll
    for (int j = k / 2; j > 0; j >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i)
        if ((i & j) == 0) cswap(v[i], v[i + j], (((i & k) == 0) == desc));
}

template <typename QT, int DH, int W>
__global__ void __launch_bounds__(TS_THREADS) select_tile_kernel(SelectParams p) {
  extern __shared__ __align__(16) unsigned char ts_smem_raw[];
  float* qT = reinterpret_cast<float*>(ts_smem_raw);
  constexpr int NP = TS_RB + 4;  // nodeT row pitch (floats)
  float* nodeT = qT + DH * TS_QT;
  float* S = nodeT + DH * NP;
  __shared__ int s_tmax;

  const int tid = threadIdx.x, lane = tid & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int n0 = blockIdx.x * TS_QT;
  const LevelView& lv = p.lv;
  const float* nodes_bh = lv.nodes + b * lv.s_b + h * lv.s_h;

  // ---------------------------------------------------------------- the tile's queries (fp32, transposed)
  const int q = tid;
  int t = -1;
  if (tid == 0) s_tmax = -1;
  __syncthreads();
  if (n0 + q < p.Nq) {
    const int64_t tt = p.tq[b * p.tq_sb + (int64_t)(n0 + q) * p.tq_st];
    if (tt < 0 || tt >= lv.cap) {
      record_error(DEV_POS_RANGE, K_SELECT, (int)tt, lv.cap);
    } else {
      t = (int)tt;
      atomicMax(&s_tmax, t);
    }
  }
  constexpr int QV = TypeInfo<QT>::VEC;  // elements per 16-byte load (rows 16-byte aligned: checked by the host)
  for (int x = tid; x < TS_QT * (DH / QV); x += TS_THREADS) {
    const int qq = x % TS_QT, c = x / TS_QT;  // consecutive threads: consecutive queries (conflict-free writes)
    float v[QV];
    if (n0 + qq < p.Nq) {
      load_vec_f32<QT>(reinterpret_cast<const QT*>(p.q) + b * p.q_sb + h * p.q_sh + (int64_t)(n0 + qq) * p.q_st +
                           c * QV, v);
    } else {
#pragma unroll
      for (int e = 0; e < QV; ++e) v[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < QV; ++e) qT[(c * QV + e) * TS_QT + qq] = v[e];
  }
  __syncthreads();
  const int tmax = s_tmax;
  const int w = p.wmax;  // <= W
  unsigned long long kept[W];  // this query's beam, best first (0 = empty slot: below every real key)
#pragma unroll
  for (int i = 0; i < W; ++i) kept[i] = 0ull;
  int nk = 0;

  // GEMM: rows tr*4..+3 of the block, queries tq4..tq4+3 and 64+tq4..64+tq4+3 (16 threads read 256 contiguous
  // bytes of a query row: conflict-free)
  const int tr = tid >> 4, tq4 = (tid & 15) * 4;
  for (int l = lv.Lm; l >= lv.L0; --l) {
    const int rows = tmax < 0 ? 0 : min(tmax >> l, lv.cap >> l);  // nodes fully in the past of the last query
    const float scale = pow2_neg(l);
    const float* lvl = nodes_bh + (int64_t)lv.off[l] * DH;
    // ---------------------------------------------------------------- dense scores of this level
    for (int r0 = 0; r0 < rows; r0 += TS_RB) {
      const int nr = min(TS_RB, rows - r0);
      __syncthreads();  // previous block's readers of nodeT are done
      for (int x = tid; x < TS_RB * (DH / 4); x += TS_THREADS) {
        const int r = x % TS_RB, c4 = x / TS_RB;  // consecutive threads: consecutive rows (conflict-free writes)
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nr) v = __ldg(reinterpret_cast<const float4*>(lvl + (int64_t)(r0 + r) * DH + c4 * 4));
        nodeT[(c4 * 4 + 0) * NP + r] = v.x;
        nodeT[(c4 * 4 + 1) * NP + r] = v.y;
        nodeT[(c4 * 4 + 2) * NP + r] = v.z;
        nodeT[(c4 * 4 + 3) * NP + r] = v.w;
      }
      __syncthreads();
      float a0[4][8], a1[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) a0[i][j] = a1[i][j] = 0.f;
#pragma unroll 2
      for (int cc = 0; cc < DH / 4; ++cc) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = cc * 4 + e;
          const float4 nv = *reinterpret_cast<const float4*>(nodeT + d * NP + tr * 4);
          const float4 q0 = *reinterpret_cast<const float4*>(qT + d * TS_QT + tq4);
          const float4 q1 = *reinterpret_cast<const float4*>(qT + d * TS_QT + 64 + tq4);
          const float nr4[4] = {nv.x, nv.y, nv.z, nv.w};
          const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (cc & 1) a1[i][j] = fmaf(qv[j], nr4[i], a1[i][j]);
              else a0[i][j] = fmaf(qv[j], nr4[i], a0[i][j]);
            }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = r0 + tr * 4 + i;
        if (tr * 4 + i < nr) {
          float4 o0, o1;
          o0.x = (a0[i][0] + a1[i][0]) * scale; o0.y = (a0[i][1] + a1[i][1]) * scale;
          o0.z = (a0[i][2] + a1[i][2]) * scale; o0.w = (a0[i][3] + a1[i][3]) * scale;
          o1.x = (a0[i][4] + a1[i][4]) * scale; o1.y = (a0[i][5] + a1[i][5]) * scale;
          o1.z = (a0[i][6] + a1[i][6]) * scale; o1.w = (a0[i][7] + a1[i][7]) * scale;
          *reinterpret_cast<float4*>(S + r * TS_QT + tq4) = o0;
          *reinterpret_cast<float4*>(S + r * TS_QT + 64 + tq4) = o1;
        }
      }
    }
    __syncthreads();
    // ---------------------------------------------------------------- one level of this thread's descent
    // candidates: the children of the kept nodes (all in the past), then the newly available past-only subtree
    const int bit = (t >= 0) ? (t >> l) & 1 : 0;
    unsigned long long c[2 * W + 1];
#pragma unroll
    for (int i = 0; i < W; ++i) {
      if (i < nk) {
        const int m = key_id(kept[i]);
        c[2 * i] = order_key(S[(2 * m) * TS_QT + q], 2 * m);
        c[2 * i + 1] = order_key(S[(2 * m + 1) * TS_QT + q], 2 * m + 1);
      } else {
        c[2 * i] = c[2 * i + 1] = 0ull;
      }
    }
    {
      const int inj = (t >> l) - 1;
      c[2 * W] = bit ? order_key(S[inj * TS_QT + q], inj) : 0ull;
    }
    const int n = 2 * nk + bit;
    const bool rank = (l == lv.L0) || n > w;  // the order matters (the leaf level) or some candidate is dropped
    if (__any_sync(0xffffffffu, rank)) {
      // the best w keys, best first (empty slots hold 0, below every real key): sort the first W children
      // descending and the other W ascending, keep the elementwise larger halves (the W best of the 2W, a
      // bitonic sequence), sort it, then let the injected candidate bubble in
      bitonic_sort<W>(c, true);
      bitonic_sort<W>(c + W, false);
#pragma unroll
      for (int i = 0; i < W; ++i) kept[i] = c[i] > c[W + i] ? c[i] : c[W + i];
      bitonic_merge<W>(kept, true);
      {
        unsigned long long key = c[2 * W];
#pragma unroll
        for (int i = 0; i < W; ++i) {
          const unsigned long long hi = kept[i] > key ? kept[i] : key;
          key = kept[i] > key ? key : kept[i];
          kept[i] = hi;
        }
      }
#pragma unroll
      for (int i = 0; i < W; ++i)
        if (i >= w) kept[i] = 0ull;
    } else {
      // every candidate is kept (order irrelevant above the leaf level): children in place, the injected one after
#pragma unroll
      for (int i = 0; i < W; ++i) kept[i] = i < 2 * nk ? c[i] : (i == 2 * nk ? c[2 * W] : 0ull);
    }
    nk = min(n, w);
    __syncthreads();  // S is rewritten by the next level
  }
  (void)lane;
  // ---------------------------------------------------------------- outputs (best first)
  if (n0 + q < p.Nq) {
    const size_t obase = ((size_t)bh * p.Nq + n0 + q) * p.wl;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      if (i < p.wl) {
        const bool ok = t >= 0 && i < nk;
        p.ids[obase + i] = ok ? key_id(kept[i]) : 0;
        p.vld[obase + i] = ok ? 1 : 0;
        if (p.sct) p.sct[obase + i] = ok ? key_score(kept[i]) : -INFINITY;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ neighbours
// seg.py:73-103 neighbor_pass: query n at position t looks at the NS best leaves stored by each of the Wn previous
// positions (st_* (B, H, T_st, NS), indexed by position), scores each itself (q . S_L0[leaf] * 2^-L0) and matches
// those it scores at least base - rho |base| (base = the stored score); the scan depth is capped by the match rate
// over the first nb_probe positions: cap = cap_min + round_half_even((Wn - cap_min) * rate). One warp per query,
// one lane per stored leaf (Wn * NS <= 32). The threshold, rate and cap are formed with the same fp32 roundings
// as the reference (no fused multiply-add).
struct NeighborParams {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const int64_t* tq;
  int64_t tq_sb, tq_st;
  const float* leaf_nodes;  // level-L0 node rows of (b=0, h=0); row m of (b, h) at + b*n_sb + h*n_sh + m*dh
  int64_t n_sb, n_sh;
  int n_leaf;
  float scale;              // 2^-L0
  const int64_t* st_leaf;   // (B, H, T_st, NS) contiguous
  const float* st_score;
  const uint8_t* st_ok;
  int T_st;
  int B, H, Nq, Wn, NS, probe, cap_min, neighbors;
  float rho;
  int64_t* nid;             // (B, H, Nq, Wn*NS)
  uint8_t* match;           // (B, H, Nq, Wn*NS)
  int64_t* nL;              // (B, H, Nq)
};

template <typename QT, int DH>
__global__ void __launch_bounds__(128) neighbor_pass_kernel(NeighborParams p) {
  __shared__ __align__(16) float qs[4][DH];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.B * p.H * p.Nq) return;
  const int n = (int)(qid % p.Nq);
  const int64_t bh = qid / p.Nq;
  const int b = (int)(bh / p.H), h = (int)(bh % p.H);
  const int64_t t = p.tq[b * p.tq_sb + (int64_t)n * p.tq_st];
  const QT* qrow = reinterpret_cast<const QT*>(p.q) + b * p.q_sb + h * p.q_sh + (int64_t)n * p.q_st;
  for (int d = lane; d < DH; d += 32) qs[warp][d] = to_f32(qrow[d]);
  __syncwarp();
  const int W = p.Wn * p.NS;
  const int j = lane;
  const int dist = j / p.NS + 1, slot = j - (j / p.NS) * p.NS;
  const int64_t jpos = t - dist;
  const bool jval = j < W && jpos >= 0 && jpos < p.T_st;
  const int64_t jc = jpos < 0 ? 0 : (jpos >= p.T_st ? p.T_st - 1 : jpos);
  const int64_t sidx = (bh * p.T_st + jc) * p.NS + slot;
  int64_t id = 0;
  float base = 0.f;
  bool ok0 = false;
  if (j < W) {
    id = p.st_leaf[sidx];
    base = p.st_score[sidx];
    ok0 = jval && p.st_ok[sidx] != 0;
  }
  // this query's own score of the stored leaf
  float sc = 0.f;
  if (ok0) {
    const int64_t m = id < 0 ? 0 : (id >= p.n_leaf ? p.n_leaf - 1 : id);
    const float* row = p.leaf_nodes + b * p.n_sb + h * p.n_sh + m * DH;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int cc = 0; cc < DH / 4; ++cc) {
      const float4 qv = *reinterpret_cast<const float4*>(&qs[warp][cc * 4]);
      const float4 v = __ldg(reinterpret_cast<const float4*>(row + cc * 4));
      if (cc & 1) {
        a1 = fmaf(qv.x, v.x, a1); a1 = fmaf(qv.y, v.y, a1); a1 = fmaf(qv.z, v.z, a1); a1 = fmaf(qv.w, v.w, a1);
      } else {
        a0 = fmaf(qv.x, v.x, a0); a0 = fmaf(qv.y, v.y, a0); a0 = fmaf(qv.z, v.z, a0); a0 = fmaf(qv.w, v.w, a0);
      }
    }
    sc = __fmul_rn(__fadd_rn(a0, a1), p.scale);
  }
  const float thr = __fsub_rn(base, __fmul_rn(p.rho, fabsf(base)));
  bool m = ok0 && sc >= thr;
  const unsigned pm = p.probe >= 32 ? 0xffffffffu : ((1u << p.probe) - 1u);
  const unsigned bm = __ballot_sync(0xffffffffu, m), bo = __ballot_sync(0xffffffffu, ok0);
  const int nm = __popc(bm & pm), no = __popc(bo & pm);
  const float rate = __fdiv_rn((float)nm, (float)(no > 1 ? no : 1));
  const int cap = p.cap_min + (int)rintf(__fmul_rn((float)(p.Wn - p.cap_min), rate));
  m = m && dist <= cap && p.neighbors != 0;
  // distinct matched leaves: a matched lane counts when no lower matched lane holds the same id
  const unsigned long long key = m ? (unsigned long long)id : (0xffffffff00000000ull | (unsigned)lane);
  const unsigned same = __match_any_sync(0xffffffffu, key);
  const bool first = m && (__ffs(same) - 1) == lane;
  const int nl = __popc(__ballot_sync(0xffffffffu, first));
  if (j < W) {
    p.nid[qid * W + j] = id;
    p.match[qid * W + j] = m ? 1 : 0;
  }
  if (lane == 0) p.nL[qid] = nl;
}

// ------------------------------------------------------------------------------------------------ lane tree
// Beam descent over the dynamic content tree (dyntree.py:108-127 LaneTree.search): one query per lane (tree),
// nodes holding key SUMS and counts, packed level by level (level l at rows 2^l - 1 .. 2^(l+1) - 2, l = 0..D).
// From the root, at every level the children of the kept nodes are candidates; a child is valid when its count is
// positive (its parent being valid), scored by q . sum / count; the best min(wmax, 2 * previous width) valid
// ones are kept, best first, ties by the smaller node id. One warp per query: lane-per-candidate scoring from L2,
// rank-counting top-k on the (score, id) order keys (Descent::topk).
struct LaneSearchParams {
  const float* q;      // (P, dh) fp32
  const float* sums;   // (P, NN, dh) fp32, NN = 2^(D+1) - 1
  const int32_t* cnt;  // (P, NN)
  int P, D, wmax, wl;
  int64_t* ids;        // (P, wl) node ids of level D, best first (0 in invalid slots)
  uint8_t* vld;        // (P, wl)
  float* sct;          // (P, wl) scores (-inf invalid), may be null
};

// A lane's packed tree (row r = node r in level order): rows [0, ns) in shared memory (a cached copy of the upper
// levels), the others in global memory. Rows and counts are reached through generic pointers.
template <int DH>
struct LaneTreeRef {
  float* g;
  int32_t* gc;
  float* s;
  int32_t* sc;
  int ns;
  __device__ __forceinline__ float* row(int r) const { return r < ns ? s + (size_t)r * DH : g + (int64_t)r * DH; }
  __device__ __forceinline__ int32_t* cntp(int r) const { return r < ns ? sc + r : gc + r; }
  __device__ __forceinline__ int cnt(int r) const { return *cntp(r); }
};

// The descent of one query (in sc.qf) over one lane's packed tree; the kept level-D nodes end in sc.kid / sc.ksc,
// best first. Returns how many are valid. NC: node rows through the read-only (non-coherent) path - only for a tree
// that no thread writes while the kernel runs (the select loop updates its trees, so it reads them coherently).
template <int DH, bool NC = true>
__device__ __forceinline__ int lane_descend(const float* sums, const int32_t* cnt, int D, int wmax,
                                            DescentScratch& sc, int lane);

template <int DH, bool NC>
__device__ __forceinline__ int lane_descend_t(const LaneTreeRef<DH>& tr, int D, int wmax, DescentScratch& sc,
                                              int lane) {
  if (lane == 0) sc.kid[0] = 0;
  __syncwarp();
  int nk = tr.cnt(0) > 0 ? 1 : 0;
  int w = 1;
  for (int l = 1; l <= D; ++l) {
    const int off = (1 << l) - 1;
    // valid children of the kept nodes, compacted (kept node i -> children 2m, 2m+1)
    int n = 0;
    for (int base = 0; base < 2 * nk; base += 32) {
      const int j = base + lane;
      int c = -1;
      if (j < 2 * nk) {
        const int m = sc.kid[j >> 1];
        c = 2 * m + (j & 1);
        if (tr.cnt(off + c) <= 0) c = -1;
      }
      const unsigned mask = __ballot_sync(0xffffffffu, c >= 0);
      if (c >= 0) sc.cid[n + __popc(mask & ((1u << lane) - 1u))] = c;
      n += __popc(mask);
    }
    __syncwarp();
    // lane-per-candidate scores: (q . sum) / count in fp32
    for (int base = 0; base < n; base += 32) {
      const int j = base + lane;
      if (j < n) {
        const int c = sc.cid[j];
        const float* row = tr.row(off + c);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int cc = 0; cc < DH / 4; ++cc) {
          const float4 qv = *reinterpret_cast<const float4*>(sc.qf + cc * 4);
          const float4 v = NC ? __ldg(reinterpret_cast<const float4*>(row + cc * 4))
                              : *reinterpret_cast<const float4*>(row + cc * 4);
          if (cc & 1) {
            a1 = fmaf(qv.x, v.x, a1); a1 = fmaf(qv.y, v.y, a1); a1 = fmaf(qv.z, v.z, a1); a1 = fmaf(qv.w, v.w, a1);
          } else {
            a0 = fmaf(qv.x, v.x, a0); a0 = fmaf(qv.y, v.y, a0); a0 = fmaf(qv.z, v.z, a0); a0 = fmaf(qv.w, v.w, a0);
          }
        }
        const float s = (a0 + a1) / (float)tr.cnt(off + c);
        sc.csc[j] = s;
        sc.ckey[j] = order_key(s, c);
      }
    }
    __syncwarp();
    w = min(wmax, 2 * w);
    nk = Descent<DH>::topk(n, w, sc, lane);
  }
  __syncwarp();
  return nk;
}

template <int DH, bool NC>
__device__ __forceinline__ int lane_descend(const float* sums, const int32_t* cnt, int D, int wmax,
                                            DescentScratch& sc, int lane) {
  const LaneTreeRef<DH> tr{const_cast<float*>(sums), const_cast<int32_t*>(cnt), nullptr, nullptr, 0};
  return lane_descend_t<DH, NC>(tr, D, wmax, sc, lane);
}

template <int DH>
__global__ void __launch_bounds__(128) lane_search_kernel(LaneSearchParams p) {
  __shared__ DescentScratch scr[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qi = (int64_t)blockIdx.x * 4 + warp;
  if (qi >= p.P) return;
  DescentScratch& sc = scr[warp];
  const int NN = (2 << p.D) - 1;
  for (int d = lane; d < DH; d += 32) sc.qf[d] = p.q[qi * DH + d];
  const int nk = lane_descend<DH>(p.sums + qi * (int64_t)NN * DH, p.cnt + qi * (int64_t)NN, p.D, p.wmax, sc, lane);
  for (int i = lane; i < p.wl; i += 32) {
    const bool ok = i < nk;
    p.ids[qi * p.wl + i] = ok ? sc.kid[i] : 0;
    p.vld[qi * p.wl + i] = ok ? 1 : 0;
    if (p.sct) p.sct[qi * p.wl + i] = ok ? sc.ksc[i] : -INFINITY;
  }
}

// ------------------------------------------------------------------------------------------------ finish
// seg.py:106-119 (leaves_to_pos, finish), one thread per query. Leaf m expands to positions
// [m*leaf, (m+1)*leaf) stored as tree_pos[j*wl + i] = ids[i]*leaf + j (the reference's cat([2*ids, 2*ids+1])
// at leaf 2); invalid -> -1.
struct FinishParams {
  const int64_t* ids;        // (Q, wl)
  const uint8_t* vld;        // (Q, wl)
  const int64_t* nid;        // (Q, nbw) neighbour leaf ids, may be null
  const uint8_t* match;      // (Q, nbw), may be null (no neighbour matches)
  const int64_t* nL;         // (Q), may be null (0)
  const int64_t* lhat;       // (Q)
  int64_t Q;
  int wl, nbw, leaf, wmax;
  int64_t* tree_pos;         // (Q, leaf*wl)
  int64_t* nb_pos;           // (Q, leaf*nbw)
  int64_t* n_tree;           // (Q)
  int64_t* nb_leaves;        // (Q)
};

__device__ __forceinline__ int64_t floor_div2(int64_t x) { return x >= 0 ? x / 2 : -((-x + 1) / 2); }

__global__ void finish_kernel(FinishParams p) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= p.Q) return;
  const int64_t L = p.lhat[q];
  const int64_t nL = p.nL ? p.nL[q] : 0;
  const int64_t lo = floor_div2(L + 1);
  int64_t need = L - nL;
  if (need < 0) need = 0;
  const int64_t floor_b = nL < lo ? 2 : 1;
  int64_t bt = nL >= L ? 0 : (need > floor_b ? need : floor_b);
  if (bt > p.wmax) bt = p.wmax;
  p.n_tree[q] = bt;
  p.nb_leaves[q] = nL;
  if (p.tree_pos == nullptr) return;
  for (int i = 0; i < p.wl; ++i) {
    const bool ok = p.vld[q * p.wl + i] != 0;
    const int64_t m = p.ids[q * p.wl + i];
    for (int j = 0; j < p.leaf; ++j)
      p.tree_pos[q * (int64_t)p.leaf * p.wl + (int64_t)j * p.wl + i] = ok ? m * p.leaf + j : -1;
  }
  if (p.nb_pos == nullptr) return;
  for (int i = 0; i < p.nbw; ++i) {
    const bool ok = p.match ? p.match[q * p.nbw + i] != 0 : false;
    const int64_t m = p.nid ? p.nid[q * p.nbw + i] : 0;
    for (int j = 0; j < p.leaf; ++j)
      p.nb_pos[q * (int64_t)p.leaf * p.nbw + (int64_t)j * p.nbw + i] = ok ? m * p.leaf + j : -1;
  }
}

}  // namespace ta
