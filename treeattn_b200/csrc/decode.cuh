// Fused segment-tree decode step for one layer (reference: engine.py:84-120 seg_attend with the incremental
// tree update of engine.py:41-55 SegState.add), batched over (b, h) and split across a thread-block cluster.
//
// One cluster of S CTAs per (b, h). Every CTA of the cluster runs the tree descent for the new query (warp 0;
// the node rows come from L2 after the first CTA), while a producer warp already streams the local-window
// rows. The key set - used leaf blocks cut at the window, the sink, the window, and the new token - is cut
// into stages of <= CH rows; stage c belongs to CTA c % S. A producer warp fills a ring of NST shared-memory
// stages with 1-D bulk copies (cp.async.bulk, one destination CTA each) and mbarriers; NCW consumer warps run the online
// softmax from shared memory. Partial (max, sum, acc) states are merged across the cluster through
// distributed shared memory, rank 0 writes the output, appends the new K/V rows and, when the new token
// completes a leaf block, forms that leaf node and its right-spine ancestors (fp32, adjacent-pair order).
//
// Position t itself is not read from the cache: rank 0 takes the new token's key/value straight from the
// qkv rows of this step, so no CTA reads a cache row that is written in the same launch. The tree nodes
// written here (node t>>l at each level where (t+1) % 2^l == 0) are not complete before t, so no descent of
// this launch reads them either.
#pragma once
#include "attn.cuh"

namespace ta {

struct DecodeParams {
  const void* qkv;        // (B, 3*H*DH) rows of this step: q | k | v
  int64_t qkv_sb;         // row stride (elements)
  int64_t k_ofs, v_ofs;   // element offsets of the k and v parts inside a row
  void* kc;               // key cache (B, H, cap, DH) with strides below
  void* vc;               // value cache
  int64_t c_sb, c_sh, c_st;
  float* nodes;           // tree levels (mutable), layout of LevelView
  LevelView lv;
  const int32_t* pos;     // (B) position t of this step
  int B, H, wmax, n_tree, Lw;
  float scale;
  void* out;              // (B, H*DH) attention output rows
  int64_t o_sb;
  float* lse;             // (B, H) natural-log LSE, may be null
  int32_t* nkeys;         // (B, H) keys attended, may be null
  int32_t* sel;           // (B, H, wmax + 1): [count, leaf ids...] of the descent, may be null
  int splits;             // cluster size S (grid.x)
  // persistent kernel, split items: the items [0, n_whole) run whole; every later item is cut into psplit parts
  // (its window rows and its leaf rows each in psplit near-equal shares). A part's partial softmax state goes to
  // part[((bh - n_whole) * psplit + j) * (DH + 4)] (m, l, keys, -, acc[DH]) and the part that finishes last
  // (part_cnt[bh], reset to 0 by it) merges them, writes the output and appends the step's rows.
  int psplit, n_whole;
  float* part;
  int32_t* part_cnt;
};

template <typename T, int DH, int CH, int NST, int NCW>
struct DecodeCfg {
  static constexpr int NTHREADS = (NCW + 1) * 32;
  static constexpr int STAGE_ELEMS = 2 * CH * DH;  // K rows then V rows
  static constexpr size_t RING_BYTES = (size_t)NST * STAGE_ELEMS * sizeof(T);
};

struct DecodeShared {
  uint64_t full[8];
  uint64_t empty[8];
  int nrows[8];
  int consumed;
  int rows_cta;
  int nsel;
  int abort_flag;
  RangeList rl;
  DescentScratch ds;
  float part_m[8], part_l[8];
  float cta_m, cta_l;
  int cta_rows;
};

// Dynamic shared memory: [DecodeShared][pad to 128][ring][descent stage rows][part_acc NCW*DH][cta_acc DH]
template <typename T, int DH, int CH, int NST, int NCW>
__host__ __device__ inline size_t decode_smem_bytes(int wmax) {
  size_t off = (sizeof(DecodeShared) + 127) & ~(size_t)127;
  off += DecodeCfg<T, DH, CH, NST, NCW>::RING_BYTES;
  off += (size_t)(2 * wmax + 1) * stage_row_floats<DH>() * sizeof(float);
  off += (size_t)NCW * DH * sizeof(float);
  off += (size_t)DH * sizeof(float);
  return off;
}

// Form the leaf node of the block that position t completes ((t+1) % 2^L0 == 0) and its right-spine
// ancestors. Leaf node = adjacent-pair fp32 sums of rows [n*2^L0, t] (the sink as 0; row t = knew, not yet
// readable from the cache), reduced in shared memory `xs` (xs_floats >= 2^L0) in dim slices. The `nthreads`
// threads (tid 0..nthreads-1) synchronizing on named barrier `bar` (0 = the whole CTA) must all call this.
template <typename T, int DH>
__device__ void tree_update_block(const T* __restrict__ kbase, int64_t c_st, const T* __restrict__ knew, int t,
                                  float* __restrict__ nodes_bh, const LevelView& lv, float* xs, int xs_floats,
                                  int tid, int nthreads, int bar) {
  const int L0 = lv.L0, leaf = 1 << L0;
  const int DS = min(DH, xs_floats / leaf);
  const int n_blk = t >> L0;
  const int p0 = n_blk * leaf;
  float my_node = 0.f;  // this thread's dim of the new leaf node (tid < DH)
  for (int d0 = 0; d0 < DH; d0 += DS) {
    const int dn = min(DS, DH - d0);
    for (int x = tid; x < leaf * dn; x += nthreads) {
      const int i = x / dn, d = d0 + (x - (x / dn) * dn);
      const int pp = p0 + i;
      float v;
      if (pp == 0) v = 0.f;
      else if (pp == t) v = to_f32(knew[d]);
      else v = to_f32(kbase[(int64_t)pp * c_st + d]);
      xs[i * dn + (d - d0)] = v;
    }
    named_bar_sync(bar, nthreads);
    for (int st = 1; st < leaf; st <<= 1) {
      const int pairs = leaf / (2 * st);
      for (int x = tid; x < pairs * dn; x += nthreads) {
        const int pi = x / dn, d = x - (x / dn) * dn;
        const int i = pi * 2 * st;
        xs[i * dn + d] = xs[i * dn + d] + xs[(i + st) * dn + d];
      }
      named_bar_sync(bar, nthreads);
    }
    if (tid >= d0 && tid < d0 + dn) my_node = xs[tid - d0];
    named_bar_sync(bar, nthreads);
  }
  if (tid < DH) {
    nodes_bh[(int64_t)(lv.off[L0] + n_blk) * DH + tid] = my_node;
    // node m = t >> l at level l is complete when (t+1) % 2^l == 0; the node just formed at level l-1 is its
    // right child, so parent = S[l-1][2m] (stored earlier) + S[l-1][2m+1] (just formed)
    float cur = my_node;
    for (int l = L0 + 1; l <= lv.Lm; ++l) {
      if (((t + 1) & ((1 << l) - 1)) != 0) break;
      const int m = t >> l;
      if (m >= (lv.cap >> l)) break;
      const float left = nodes_bh[(int64_t)(lv.off[l - 1] + 2 * m) * DH + tid];
      cur = left + cur;
      nodes_bh[(int64_t)(lv.off[l] + m) * DH + tid] = cur;
    }
  }
}

template <typename T, int DH, int CH, int NST, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32) decode_kernel(DecodeParams p) {
  using Cfg = DecodeCfg<T, DH, CH, NST, NCW>;
  using WA = typename StageAttn<T, DH>::type;
  constexpr int VEC = WA::VEC;
  constexpr int ROWB = DH * (int)sizeof(T);
  static_assert(NST <= 8 && NCW <= 8, "ring too deep");

  extern __shared__ __align__(128) unsigned char smem_raw[];
  DecodeShared& sh = *reinterpret_cast<DecodeShared*>(smem_raw);
  size_t off = (sizeof(DecodeShared) + 127) & ~(size_t)127;
  T* ring = reinterpret_cast<T*>(smem_raw + off);
  off += Cfg::RING_BYTES;
  float* dstage = reinterpret_cast<float*>(smem_raw + off);
  off += (size_t)(2 * p.wmax + 1) * stage_row_floats<DH>() * sizeof(float);
  float* part_acc = reinterpret_cast<float*>(smem_raw + off);
  off += (size_t)NCW * DH * sizeof(float);
  float* cta_acc = reinterpret_cast<float*>(smem_raw + off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.splits;
  const int rank = (S > 1) ? (int)cluster_ctarank() : 0;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int leaf = 1 << p.lv.L0;
  pdl_wait();  // every input (positions, q/k/v rows, caches, tree) may come from the grid this one follows
  pdl_launch_dependents();

  int t = p.pos[b];
  bool active = true;
  if (t < 0 || t >= p.lv.cap) {
    if (tid == 0 && rank == 0) record_error(DEV_POS_RANGE, K_DECODE, t, p.lv.cap);
    active = false;
    t = 0;
  }
  const int w0 = max(t - p.Lw + 1, 0);
  const int nwin = active ? t - w0 : 0;   // window rows read from the cache: [w0, t)
  const int nA = ceil_div(nwin, CH);      // window stages

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], NCW);
    }
    sh.consumed = 0;
    sh.rows_cta = 0;
    sh.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const T* kbase = reinterpret_cast<const T*>(p.kc) + b * p.c_sb + h * p.c_sh;
  const T* vbase = reinterpret_cast<const T*>(p.vc) + b * p.c_sb + h * p.c_sh;
  const T* qkv_row = reinterpret_cast<const T*>(p.qkv) + b * p.qkv_sb;

  if (warp == NCW) {
    // ------------------------------------------------------------------ producer warp (lane 0 issues)
    const uint64_t pol = l2_policy_evict_first();
    int it = 0;  // stages issued by this CTA (lane 0)
    bool ok = true;
    auto acquire = [&](int& s) -> bool {
      s = it % NST;
      if (it >= NST) return mbar_wait_bounded(&sh.empty[s], ((it / NST) - 1) & 1, K_DECODE, 1);
      return true;
    };
    if (lane == 0) {
      // phase A: the window rows [w0, t), CH rows per stage
      for (int c = 0; c < nA && ok; ++c) {
        if (c % S != rank) continue;
        int s;
        if (!(ok = acquire(s))) break;
        const int r0 = w0 + c * CH;
        const int n = min(CH, t - r0);
        sh.nrows[s] = n;
        T* kd = ring + (size_t)s * Cfg::STAGE_ELEMS;
        mbar_arrive_expect_tx(&sh.full[s], (uint32_t)(2 * n * ROWB));
        bulk_g2s_hint(kd, kbase + (int64_t)r0 * p.c_st, (uint32_t)(n * ROWB), &sh.full[s], pol);
        bulk_g2s_hint(kd + CH * DH, vbase + (int64_t)r0 * p.c_st, (uint32_t)(n * ROWB), &sh.full[s], pol);
        ++it;
      }
    }
    __syncwarp();
    // wait for the descent's range list (warp 0 arrives on named barrier 1)
    named_bar_sync(1, 64);
    if (lane == 0) {
      // phase B: leaf ranges + sink, packed CH rows per stage; every CTA walks the same packing
      if (ok && active) {
        const RangeList& rl = sh.rl;
        int ri = 0, roff = 0;
        for (int c = nA; ri < rl.n && ok; ++c) {
          const bool mine = (c % S) == rank;
          int s = 0;
          if (mine && !(ok = acquire(s))) break;
          T* kd = ring + (size_t)s * Cfg::STAGE_ELEMS;
          int n = 0;
          {  // rows of this stage
            int ri2 = ri, roff2 = roff;
            while (n < CH && ri2 < rl.n) {
              const int len = rl.pref[ri2 + 1] - rl.pref[ri2];
              const int take = min(CH - n, len - roff2);
              n += take;
              roff2 += take;
              if (roff2 == len) { ++ri2; roff2 = 0; }
            }
          }
          if (mine) {
            sh.nrows[s] = n;
            mbar_arrive_expect_tx(&sh.full[s], (uint32_t)(2 * n * ROWB));
          }
          int put = 0;
          while (put < n) {
            const int len = rl.pref[ri + 1] - rl.pref[ri];
            const int take = min(n - put, len - roff);
            if (mine) {
              const int64_t r0 = rl.start[ri] + roff;
              bulk_g2s_hint(kd + (size_t)put * DH, kbase + r0 * p.c_st, (uint32_t)(take * ROWB), &sh.full[s], pol);
              bulk_g2s_hint(kd + (size_t)(CH + put) * DH, vbase + r0 * p.c_st, (uint32_t)(take * ROWB),
                            &sh.full[s], pol);
            }
            put += take;
            roff += take;
            if (roff == len) { ++ri; roff = 0; }
          }
          if (mine) ++it;
        }
      }
      // sentinel stage: no copy, only an arrival
      if (ok) {
        int s;
        if ((ok = acquire(s))) {
          sh.nrows[s] = -1;
          mbar_arrive(&sh.full[s]);
        }
      }
      if (!ok) atomicExch(&sh.abort_flag, 1);
    }
    __syncwarp();
    // wait until the consumers stopped, then make sure no copy of this CTA is still in flight
    named_bar_sync(2, Cfg::NTHREADS);
    if (lane == 0) {
      for (int i = sh.consumed; i < it; ++i) mbar_wait_bounded(&sh.full[i % NST], (i / NST) & 1, K_DECODE, 2);
    }
  } else {
    // ------------------------------------------------------------------ consumer warps
    WA wa;
    wa.init(qkv_row + h * DH, p.scale * LOG2E, lane);
    if (warp == 0) {
      int nk = 0;
      if (active) {
        load_qf<T, DH>(qkv_row + h * DH, sh.ds, lane);
        const float* nodes_bh = p.lv.nodes + b * p.lv.s_b + h * p.lv.s_h;
        const int keep = min(p.n_tree, p.wmax);
        nk = Descent<DH>::run(nodes_bh, p.lv, t, p.wmax, keep, false, sh.ds, dstage, 2 * p.wmax + 1, lane);
        build_ranges(
            sh.rl, nk, [&](int i) -> int64_t { return sh.ds.kid[i]; }, leaf, t, p.Lw, w0, lane);
      } else if (lane == 0) {
        sh.rl.n = 0;
        sh.rl.pref[0] = 0;
      }
      if (lane == 0) sh.nsel = nk;
      __syncwarp();
      named_bar_arrive(1, 64);
      if (rank == 0 && active) {
        // the new token (position t) from this step's k/v rows
        wa.one_row(qkv_row + p.k_ofs + h * DH, qkv_row + p.v_ofs + h * DH);
      }
    }
    // stream the ring
    int it = 0, rows_mine = 0;
    bool ok = true;
    while (true) {
      const int s = it % NST;
      if (!mbar_wait_bounded(&sh.full[s], (it / NST) & 1, K_DECODE, 3)) {
        ok = false;
        break;
      }
      const int n = sh.nrows[s];
      if (n < 0) break;
      const T* kst = ring + (size_t)s * Cfg::STAGE_ELEMS;
      wa.stage(kst, kst + CH * DH, n, warp, NCW);
      if (warp == 0) rows_mine += n;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.empty[s]);
      ++it;
    }
    if (!ok) atomicExch(&sh.abort_flag, 1);
    if (warp == 0 && lane == 0) {
      sh.consumed = it;
      sh.rows_cta = rows_mine + ((rank == 0 && active) ? 1 : 0);
    }
    // warp partials
    wa.reduce_rows();
    if (lane == 0) {
      sh.part_m[warp] = wa.m;
      sh.part_l[warp] = wa.l;
    }
    if (wa.sub == 0) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) part_acc[warp * DH + wa.c * VEC + i] = wa.acc[i];
    }
    named_bar_sync(2, Cfg::NTHREADS);
  }

  // ------------------------------------------------------------------ CTA partial (threads < DH)
  __syncthreads();
  if (tid < DH) {
    float m = -INFINITY, l = 0.f, a = 0.f;
    for (int w = 0; w < NCW; ++w) {
      const float mw = sh.part_m[w];
      const float mn = fmaxf(m, mw);
      if (mn == -INFINITY) continue;
      const float fa = exp2f(m - mn), fb = exp2f(mw - mn);
      l = l * fa + sh.part_l[w] * fb;
      a = a * fa + part_acc[w * DH + tid] * fb;
      m = mn;
    }
    cta_acc[tid] = a;
    if (tid == 0) {
      sh.cta_m = m;
      sh.cta_l = l;
      sh.cta_rows = sh.rows_cta;
    }
  }
  // ------------------------------------------------------------------ cluster merge
  if (S > 1) cluster_sync_all();
  else __syncthreads();
  if (rank == 0) {
    if (tid < DH) {
      float m = sh.cta_m, l = sh.cta_l, a = cta_acc[tid];
      for (int r = 1; r < S; ++r) {
        const DecodeShared* rs = cluster_map(&sh, (uint32_t)r);
        const float* racc = cluster_map(cta_acc, (uint32_t)r);
        const float mr = rs->cta_m;
        const float mn = fmaxf(m, mr);
        if (mn == -INFINITY) continue;
        const float fa = exp2f(m - mn), fb = exp2f(mr - mn);
        l = l * fa + rs->cta_l * fb;
        a = a * fa + racc[tid] * fb;
        m = mn;
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      cta_acc[tid] = a * inv;  // reuse as the normalised output
      if (tid == 0) {
        int rows = sh.cta_rows;
        for (int r = 1; r < S; ++r) rows += cluster_map(&sh, (uint32_t)r)->cta_rows;
        if (p.lse) p.lse[bh] = l > 0.f ? (m + log2f(l)) * LN2 : -INFINITY;
        if (p.nkeys) p.nkeys[bh] = rows;
        if (p.sel) {
          int32_t* so = p.sel + (int64_t)bh * (p.wmax + 1);
          so[0] = sh.nsel;
          for (int i = 0; i < p.wmax; ++i) so[1 + i] = i < sh.nsel ? sh.ds.kid[i] : -1;
        }
      }
    }
  }
  if (S > 1) cluster_sync_all();  // remote shared memory stays alive until rank 0 has read it
  if (rank != 0 || !active) return;
  __syncthreads();
  // ------------------------------------------------------------------ output + append (rank 0)
  T* orow = reinterpret_cast<T*>(p.out) + b * p.o_sb + h * DH;
  T* kdst = reinterpret_cast<T*>(p.kc) + b * p.c_sb + h * p.c_sh + (int64_t)t * p.c_st;
  T* vdst = reinterpret_cast<T*>(p.vc) + b * p.c_sb + h * p.c_sh + (int64_t)t * p.c_st;
  if (tid < DH / VEC) {
    store_vec_from_f32<T>(orow + tid * VEC, cta_acc + tid * VEC);
    *reinterpret_cast<uint4*>(kdst + tid * VEC) = *reinterpret_cast<const uint4*>(qkv_row + p.k_ofs + h * DH + tid * VEC);
    *reinterpret_cast<uint4*>(vdst + tid * VEC) = *reinterpret_cast<const uint4*>(qkv_row + p.v_ofs + h * DH + tid * VEC);
  }
  // ------------------------------------------------------------------ incremental tree update
  if (((t + 1) & (leaf - 1)) != 0) return;
  constexpr int RING_FLOATS = (int)(Cfg::RING_BYTES / sizeof(float));
  tree_update_block<T, DH>(kbase, p.c_st, qkv_row + p.k_ofs + h * DH, t,
                           p.nodes + b * p.lv.s_b + h * p.lv.s_h, p.lv, reinterpret_cast<float*>(ring), RING_FLOATS,
                           tid, Cfg::NTHREADS, 0);
}

// ------------------------------------------------------------------------------------------------ append
// SegState.add (engine.py:41-55) for a batch: write k, v of position pos[b] into the caches and, when that
// position completes a leaf block, form the leaf node and its right-spine ancestors. One CTA per (b, h).
struct AppendParams {
  const void* k;          // (B, H, DH) new key rows, strides k_sb, k_sh
  const void* v;
  int64_t k_sb, k_sh, v_sb, v_sh;
  void* kc;
  void* vc;
  int64_t c_sb, c_sh, c_st;
  float* nodes;
  LevelView lv;
  const int32_t* pos;
  int B, H;
};

constexpr int APPEND_THREADS = 128;
constexpr int APPEND_SMEM_FLOATS = 8192;

template <typename T, int DH>
__global__ void __launch_bounds__(APPEND_THREADS) append_kernel(AppendParams p) {
  extern __shared__ __align__(16) float xs[];
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int tid = threadIdx.x;
  const int t = p.pos[b];
  if (t < 0 || t >= p.lv.cap) {
    if (tid == 0) record_error(DEV_POS_RANGE, K_APPEND, t, p.lv.cap);
    return;
  }
  constexpr int VEC = TypeInfo<T>::VEC;
  const T* kr = reinterpret_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
  const T* vr = reinterpret_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
  T* kbase = reinterpret_cast<T*>(p.kc) + b * p.c_sb + h * p.c_sh;
  T* vbase = reinterpret_cast<T*>(p.vc) + b * p.c_sb + h * p.c_sh;
  if (tid < DH / VEC) {
    *reinterpret_cast<uint4*>(kbase + (int64_t)t * p.c_st + tid * VEC) = *reinterpret_cast<const uint4*>(kr + tid * VEC);
    *reinterpret_cast<uint4*>(vbase + (int64_t)t * p.c_st + tid * VEC) = *reinterpret_cast<const uint4*>(vr + tid * VEC);
  }
  const int leaf = 1 << p.lv.L0;
  if (((t + 1) & (leaf - 1)) != 0) return;
  tree_update_block<T, DH>(kbase, p.c_st, kr, t, p.nodes + b * p.lv.s_b + h * p.lv.s_h, p.lv, xs,
                           APPEND_SMEM_FLOATS, tid, APPEND_THREADS, 0);
}

// ================================================================================================ persistent
// Persistent, warp-specialized decode for large batches (B*H >= #SMs). CTA c owns the (b, h) items
// c, c + G, c + 2G, ... (G = gridDim.x) and pipelines them:
//   selector warp    : copies item k+1's q/k/v rows into a descriptor slot and runs its tree descent while item k
//                      streams (descriptor ready -> mbarrier ifull[slot])
//   producer warp    : 1-D bulk copies (one destination CTA) of item k's K/V rows into a ring of NST shared-memory
//                      stages - the window rows first (they need no descent), then the used leaf blocks and the
//                      sink - and one end-of-item marker stage per consumer group
//   consumer groups  : NCG groups of WPG warps take the stages in turn (stage i -> group i % NCG), so several
//                      groups' math overlaps; a warp moves its rows of a stage into registers, frees the stage,
//                      then runs the online softmax. At the end of an item every warp hands its partial state to
//                      warp 0, which merges, writes the output, appends the new k/v rows and, when the new token
//                      completes a leaf block, forms that leaf node and its right-spine ancestors (fp32,
//                      adjacent-pair order)
// Every wait between warps is a bounded mbarrier wait, so a protocol error ends in a recorded error, not a hang.
constexpr int PSLOTS = 2;
constexpr int STAGE_FIRST = 1, STAGE_LAST = 2;

template <typename T, int DH>
struct __align__(16) PItem {
  T q[DH], k[DH], v[DH];  // this step's rows of the item's (b, h)
  RangeList rl;           // used leaf blocks cut at the window start, and the sink; the window is not listed
  int sel[WMAX_LIMIT];
  int t, bh, nsel, active, part, np;
};

template <typename T, int DH, int NST, int NCW, int NCG>
struct __align__(16) PShared {
  PItem<T, DH> item[PSLOTS];
  DescentScratch ds;
  uint64_t full[NST], empty[NST], ifull[PSLOTS], iempty[PSLOTS], pready[2], pfree[2];
  int nrows[NST], slot[NST], flags[NST];
  float part_m[2][NCW], part_l[2][NCW];
  int part_rows[2][NCW];
  int consumed[NCG];
  int abort_flag;
};

template <typename T, int DH, int CH, int NST, int NCG, int WPG>
struct PCfg {
  static constexpr int NCW = NCG * WPG;
  // two producer warps for 256-byte rows (keys and values issued separately: measured faster there), one for
  // narrower rows (no gain measured)
  static constexpr int NPROD = (DH * (int)sizeof(T) >= 256) ? 2 : 1;
  static constexpr int NTHREADS = (NCW + 2 + NPROD) * 32;  // consumers, producer(s), selector, finalizer
  static constexpr int STAGE_ELEMS = 2 * CH * DH;
  static constexpr size_t RING_BYTES = (size_t)NST * STAGE_ELEMS * sizeof(T);
  static constexpr int TU_FLOATS = 2048;
  using Sh = PShared<T, DH, NST, NCW, NCG>;
  static size_t smem_bytes(int stage_rows) {
    size_t off = (sizeof(Sh) + 127) & ~(size_t)127;
    return off + RING_BYTES + (size_t)stage_rows * stage_row_floats<DH>() * 4 + (size_t)2 * NCW * DH * 4 +
           (size_t)TU_FLOATS * 4;
  }
};

// One warp forms the leaf node completed by position t and its right-spine ancestors (same arithmetic and order
// as tree_update_block), reducing in `xs` (xs_floats >= 2^L0) with warp-level synchronization only.
template <typename T, int DH>
__device__ void tree_update_warp(const T* __restrict__ kbase, int64_t c_st, const T* knew, int t,
                                 float* __restrict__ nodes_bh, const LevelView& lv, float* xs, int xs_floats,
                                 int lane) {
  const int L0 = lv.L0, leaf = 1 << L0;
  const int DS = min(DH, xs_floats / leaf);
  const int n_blk = t >> L0;
  const int p0 = n_blk * leaf;
  for (int d0 = 0; d0 < DH; d0 += DS) {
    const int dn = min(DS, DH - d0);
    for (int x = lane; x < leaf * dn; x += 32) {
      const int i = x / dn, d = d0 + (x - (x / dn) * dn);
      const int pp = p0 + i;
      float v;
      if (pp == 0) v = 0.f;
      else if (pp == t) v = to_f32(knew[d]);
      else v = to_f32(kbase[(int64_t)pp * c_st + d]);
      xs[i * dn + (d - d0)] = v;
    }
    __syncwarp();
    for (int st = 1; st < leaf; st <<= 1) {
      const int pairs = leaf / (2 * st);
      for (int x = lane; x < pairs * dn; x += 32) {
        const int pi = x / dn, d = x - (x / dn) * dn;
        const int i = pi * 2 * st;
        xs[i * dn + d] = xs[i * dn + d] + xs[(i + st) * dn + d];
      }
      __syncwarp();
    }
    for (int d = lane; d < dn; d += 32) {
      float cur = xs[d];
      const int dd = d0 + d;
      nodes_bh[(int64_t)(lv.off[L0] + n_blk) * DH + dd] = cur;
      for (int l = L0 + 1; l <= lv.Lm; ++l) {
        if (((t + 1) & ((1 << l) - 1)) != 0) break;
        const int m = t >> l;
        if (m >= (lv.cap >> l)) break;
        cur = nodes_bh[(int64_t)(lv.off[l - 1] + 2 * m) * DH + dd] + cur;
        nodes_bh[(int64_t)(lv.off[l] + m) * DH + dd] = cur;
      }
    }
    __syncwarp();
  }
}

// SPLIT: items cut into p.psplit parts (a separate instantiation, so that whole items run the unsplit code).
template <typename T, int DH, int CH, int NST, int NCG, int WPG, bool SPLIT>
__global__ void __launch_bounds__(PCfg<T, DH, CH, NST, NCG, WPG>::NTHREADS) decode_persistent_kernel(DecodeParams p,
                                                                                                   int stage_rows) {
  using Cfg = PCfg<T, DH, CH, NST, NCG, WPG>;
  constexpr int NCW = Cfg::NCW;
  using Sh = typename Cfg::Sh;
  using WA = typename StageAttn<T, DH>::type;
  constexpr int VEC = WA::VEC;
  constexpr int ROWB = DH * (int)sizeof(T);
  // a warp's rows of a stage fit one register-staged call when early release is possible
  constexpr bool EARLY = EarlyRelease<WA>::value && (CH <= WPG * RowsPerCall<WA>::value);
  // NST % NCG == 0: every ring slot is always consumed by the same group. If two groups shared a slot, a group
  // could reach a slot whose previous phase (the other group's stage) is still in flight, and a parity wait would
  // take the older completed phase of the same parity for the new one.
  static_assert(NCW >= 2 && NST <= 16 && NST % NCG == 0, "pipeline shape");
  // with two producer warps W_PROD issues every stage's key copies (and writes the stage descriptors), W_PROD_V the
  // value copies: one thread's bulk copies proceed one after another, so two issuers keep more in flight
  constexpr int NPROD = Cfg::NPROD;
  constexpr int W_PROD = NCW, W_SEL = NCW + 1, W_FIN = NCW + 2, W_PROD_V = NPROD == 2 ? NCW + 3 : -1;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);
  size_t off = (sizeof(Sh) + 127) & ~(size_t)127;
  T* ring = reinterpret_cast<T*>(smem_raw + off);
  off += Cfg::RING_BYTES;
  float* dstage = reinterpret_cast<float*>(smem_raw + off);
  off += (size_t)stage_rows * stage_row_floats<DH>() * sizeof(float);
  float* part_acc = reinterpret_cast<float*>(smem_raw + off);  // [2][NCW][DH]
  off += (size_t)2 * NCW * DH * sizeof(float);
  float* tu = reinterpret_cast<float*>(smem_raw + off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int n_all = p.B * p.H;
  // work units: the whole items [0, NW), then PT parts of every later item
  const int PT = SPLIT ? (p.psplit > 1 ? p.psplit : 1) : 1;
  const int NW = SPLIT ? min(max(p.n_whole, 0), n_all) : n_all;
  const int n_units = NW + (n_all - NW) * PT;
  auto unit_item = [&](int u, int& part, int& np) -> int {
    if (u < NW) { part = 0; np = 1; return u; }
    const int v = u - NW;
    part = v % PT;
    np = PT;
    return NW + v / PT;
  };
  const int K = ((int)blockIdx.x < n_units) ? (n_units - (int)blockIdx.x + G - 1) / G : 0;  // units of this CTA
  const int leaf = 1 << p.lv.L0;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&sh.full[s], NPROD);  // one arrival per producer warp
      mbar_init(&sh.empty[s], WPG);
    }
    for (int s = 0; s < PSLOTS; ++s) {
      mbar_init(&sh.ifull[s], 1);
      mbar_init(&sh.iempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.pready[s], NCW);
      mbar_init(&sh.pfree[s], 1);
    }
    for (int g = 0; g < NCG; ++g) sh.consumed[g] = g;
    sh.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // every input (positions, q/k/v rows, caches, tree) may come from the grid this one follows
  pdl_launch_dependents();

  if (warp == W_SEL) {
    // ------------------------------------------------------------------ selector warp
    const int keep = min(p.n_tree, p.wmax);
    for (int k = 0; k < K; ++k) {
      const int slot = k % PSLOTS;
      if (k >= PSLOTS && !mbar_wait_bounded(&sh.iempty[slot], ((k / PSLOTS) - 1) & 1, K_DECODE, 10)) {
        if (lane == 0) atomicExch(&sh.abort_flag, 1);
        break;
      }
      PItem<T, DH>& it = sh.item[slot];
      const int unit = (int)blockIdx.x + k * G;
      int upart, unp;
      const int bh = unit_item(unit, upart, unp);
      const int b = bh / p.H, h = bh % p.H;
      int t = p.pos[b];
      const bool active = t >= 0 && t < p.lv.cap;
      if (!active) {
        if (lane == 0) record_error(DEV_POS_RANGE, K_DECODE, t, p.lv.cap);
        t = 0;
      }
      // this step's q/k/v rows and the node rows of the descent (they depend on t only) in one round of async
      // copies
      const T* row = reinterpret_cast<const T*>(p.qkv) + b * p.qkv_sb;
      constexpr int CPR = DH / VEC;  // 16-byte chunks per row
      for (int x = lane; x < 3 * CPR; x += 32) {
        const int part = x / CPR, c = x - (x / CPR) * CPR;
        const int64_t src = (part == 0 ? 0 : (part == 1 ? p.k_ofs : p.v_ofs)) + h * DH + c * VEC;
        T* dst = (part == 0 ? it.q : (part == 1 ? it.k : it.v)) + c * VEC;
        cp_async16(dst, row + src);
      }
      const float* nodes_bh = p.lv.nodes + b * p.lv.s_b + h * p.lv.s_h;
      // when CTAs hold several units, only level l* is prefetched and the levels below are gathered child by child:
      // this selector runs a unit ahead of the streaming, so the extra round trips hide (configuration 4:
      // 46.1 -> 45.1 us per launch, the ~6 MB of never-scored leaf-level rows no longer read). With one unit per
      // CTA (small batches) nothing would hide them: the whole reachable range is prefetched in one round trip
      // (8 / 16 sequences: 0.565 / 0.562 ms per step against 0.571 / 0.571 with one level)
      const typename Descent<DH>::Plan pl =
          Descent<DH>::plan(p.lv, t, p.wmax, stage_rows, n_units > G ? 1 : 64);
      if (active) Descent<DH>::prefetch(nodes_bh, p.lv, t, pl, keep < (t >> p.lv.L0), dstage, lane);
      cp_async_wait_all();
      __syncwarp();
      int nk = 0;
      if (active) {
        load_qf<T, DH>(it.q, sh.ds, lane);
        nk = Descent<DH>::select(nodes_bh, p.lv, t, pl, p.wmax, keep, false, sh.ds, dstage, lane);
        build_ranges(
            it.rl, nk, [&](int i) -> int64_t { return sh.ds.kid[i]; }, leaf, t, p.Lw, max(t - p.Lw + 1, 0), lane);
        for (int i = lane; i < nk; i += 32) it.sel[i] = sh.ds.kid[i];
      } else if (lane == 0) {
        it.rl.n = 0;
        it.rl.pref[0] = 0;
      }
      if (lane == 0) {
        it.t = t;
        it.bh = bh;
        it.part = upart;
        it.np = unp;
        it.nsel = nk;
        it.active = active ? 1 : 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.ifull[slot]);
    }
  } else if (warp == W_PROD || warp == W_PROD_V) {
    // ------------------------------------------------------------------ producer warps (lane 0 issues)
    // Both run the same stage sequence; the key producer writes each stage's descriptor before its arrival, and
    // a stage is complete (full[s]) once both producers have arrived and all of its bytes have landed.
    const bool vrole = warp == W_PROD_V;
    const bool kcopy = !vrole, vcopy = vrole || NPROD == 1;  // which copies this warp issues
    const uint32_t nsides = (kcopy ? 1u : 0u) + (vcopy ? 1u : 0u);
    int it = 0;
    bool ok = true;
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      auto acquire = [&](int& s) -> bool {
        s = it % NST;
        if (it >= NST) return mbar_wait_bounded(&sh.empty[s], ((it / NST) - 1) & 1, K_DECODE, 1);
        return true;
      };
      for (int k = 0; k < K && ok; ++k) {
        const int slot = k % PSLOTS;
        const int unit = (int)blockIdx.x + k * G;
        int part, PS;
        const int bh = unit_item(unit, part, PS);
        const int b = bh / p.H, h = bh % p.H;
        int t = p.pos[b];
        const bool active = t >= 0 && t < p.lv.cap;
        if (!active) t = 0;
        const int wa0 = max(t - p.Lw + 1, 0);
        // this part's share of the window rows [wa0, t)
        const int w0 = wa0 + (int)((int64_t)(t - wa0) * part / PS);
        const int w1 = wa0 + (int)((int64_t)(t - wa0) * (part + 1) / PS);
        const T* kbase = reinterpret_cast<const T*>(p.kc) + b * p.c_sb + h * p.c_sh;
        const T* vbase = reinterpret_cast<const T*>(p.vc) + b * p.c_sb + h * p.c_sh;
        unsigned started = 0, lasted = 0;  // consumer groups that got a FIRST / LAST stage of item k
        // flags of the stage about to be issued (index it -> group it % NCG)
        auto flags_for = [&](bool last) -> int {
          const int g = it % NCG;
          int f = ((started >> g) & 1) ? 0 : STAGE_FIRST;
          started |= 1u << g;
          if (last && !((lasted >> g) & 1)) {
            f |= STAGE_LAST;
            lasted |= 1u << g;
          }
          return f;
        };
        for (int r0 = w0; active && r0 < w1; r0 += CH) {  // window rows [w0, w1) (their LAST is not known yet)
          int s;
          if (!(ok = acquire(s))) break;
          const int n = min(CH, w1 - r0);
          const int f = flags_for(false);
          if (!vrole) {
            sh.nrows[s] = n;
            sh.flags[s] = f;
            sh.slot[s] = slot;
          }
          T* kd = ring + (size_t)s * Cfg::STAGE_ELEMS;
          mbar_arrive_expect_tx(&sh.full[s], nsides * (uint32_t)(n * ROWB));
          if (kcopy) bulk_g2s_hint(kd, kbase + (int64_t)r0 * p.c_st, (uint32_t)(n * ROWB), &sh.full[s], pol);
          if (vcopy) bulk_g2s_hint(kd + CH * DH, vbase + (int64_t)r0 * p.c_st, (uint32_t)(n * ROWB), &sh.full[s], pol);
          ++it;
        }
        if (!ok) break;
        if (!(ok = mbar_wait_bounded(&sh.ifull[slot], (k / PSLOTS) & 1, K_DECODE, 11))) break;
        const RangeList& rl = sh.item[slot].rl;
        if constexpr (!SPLIT) {
          const int n_leaf_stages = ceil_div(rl.pref[rl.n], CH);
          int ri = 0, roff = 0;
          for (int j = 0; j < n_leaf_stages; ++j) {  // leaf blocks + sink, packed CH rows per stage
            int s;
            if (!(ok = acquire(s))) break;
            int n = 0;
            {
              int ri2 = ri, roff2 = roff;
              while (n < CH && ri2 < rl.n) {
                const int len = rl.pref[ri2 + 1] - rl.pref[ri2];
                const int take = min(CH - n, len - roff2);
                n += take;
                roff2 += take;
                if (roff2 == len) { ++ri2; roff2 = 0; }
              }
            }
            const int f = flags_for(j >= n_leaf_stages - NCG);  // the last stage of each group ends the item
            if (!vrole) {
              sh.nrows[s] = n;
              sh.flags[s] = f;
              sh.slot[s] = slot;
            }
            T* kd = ring + (size_t)s * Cfg::STAGE_ELEMS;
            mbar_arrive_expect_tx(&sh.full[s], nsides * (uint32_t)(n * ROWB));
            int put = 0;
            while (put < n) {
              const int len = rl.pref[ri + 1] - rl.pref[ri];
              const int take = min(n - put, len - roff);
              const int64_t r0 = rl.start[ri] + roff;
              if (kcopy)
                bulk_g2s_hint(kd + (size_t)put * DH, kbase + r0 * p.c_st, (uint32_t)(take * ROWB), &sh.full[s], pol);
              if (vcopy)
                bulk_g2s_hint(kd + (size_t)(CH + put) * DH, vbase + r0 * p.c_st, (uint32_t)(take * ROWB),
                              &sh.full[s], pol);
              put += take;
              roff += take;
              if (roff == len) { ++ri; roff = 0; }
            }
            ++it;
          }
        } else {
          // this part's share [la, lb) of the leaf rows (flattened over the ranges)
          const int R = rl.pref[rl.n];
          const int la = (int)((int64_t)R * part / PS), lb = (int)((int64_t)R * (part + 1) / PS);
          const int n_leaf_stages = ceil_div(lb - la, CH);
          int ri = 0, roff = 0;
          while (ri < rl.n && rl.pref[ri + 1] <= la) ++ri;
          if (ri < rl.n) roff = la - rl.pref[ri];
          int left = lb - la;
          for (int j = 0; j < n_leaf_stages; ++j) {  // leaf blocks + sink, packed CH rows per stage
            int s;
            if (!(ok = acquire(s))) break;
            const int cap_n = min(CH, left);
            int n = 0;
            {
              int ri2 = ri, roff2 = roff;
              while (n < cap_n && ri2 < rl.n) {
                const int len = rl.pref[ri2 + 1] - rl.pref[ri2];
                const int take = min(cap_n - n, len - roff2);
                n += take;
                roff2 += take;
                if (roff2 == len) { ++ri2; roff2 = 0; }
              }
            }
            const int f = flags_for(j >= n_leaf_stages - NCG);  // the last stage of each group ends the item
            if (!vrole) {
              sh.nrows[s] = n;
              sh.flags[s] = f;
              sh.slot[s] = slot;
            }
            T* kd = ring + (size_t)s * Cfg::STAGE_ELEMS;
            mbar_arrive_expect_tx(&sh.full[s], nsides * (uint32_t)(n * ROWB));
            int put = 0;
            while (put < n) {
              const int len = rl.pref[ri + 1] - rl.pref[ri];
              const int take = min(n - put, len - roff);
              const int64_t r0 = rl.start[ri] + roff;
              if (kcopy)
                bulk_g2s_hint(kd + (size_t)put * DH, kbase + r0 * p.c_st, (uint32_t)(take * ROWB), &sh.full[s], pol);
              if (vcopy)
                bulk_g2s_hint(kd + (size_t)(CH + put) * DH, vbase + r0 * p.c_st, (uint32_t)(take * ROWB),
                              &sh.full[s], pol);
              put += take;
              roff += take;
              if (roff == len) { ++ri; roff = 0; }
            }
            left -= n;
            ++it;
          }
        }
        while (ok && lasted != (1u << NCG) - 1u) {  // groups still without a LAST: empty end-of-item stages
          int s;
          if (!(ok = acquire(s))) break;
          const int f = flags_for(true);
          if (!vrole) {
            sh.nrows[s] = 0;
            sh.flags[s] = f;
            sh.slot[s] = slot;
          }
          mbar_arrive(&sh.full[s]);
          ++it;
        }
      }
      for (int g = 0; g < NCG && ok; ++g) {  // one sentinel per consumer group
        int s;
        if ((ok = acquire(s))) {
          if (!vrole) sh.nrows[s] = -1;
          mbar_arrive(&sh.full[s]);
          ++it;
        }
      }
      if (!ok) atomicExch(&sh.abort_flag, 1);
    }
    __syncwarp();
    named_bar_sync(2, (NCW + NPROD) * 32);
    if (lane == 0) {  // no bulk copy of this CTA may still be in flight when it exits
      for (int i = 0; i < it; ++i)
        if (i >= sh.consumed[i % NCG]) mbar_wait_bounded(&sh.full[i % NST], (i / NST) & 1, K_DECODE, 2);
    }
  } else if (warp == W_FIN) {
    // ------------------------------------------------------------------ finalizer warp
    for (int k = 0; k < K; ++k) {
      const int slot = k % PSLOTS, par = k & 1;
      if (!mbar_wait_bounded(&sh.pready[par], (k >> 1) & 1, K_DECODE, 6)) {
        if (lane == 0) atomicExch(&sh.abort_flag, 1);
        break;
      }
      PItem<T, DH>& item = sh.item[slot];
      const float* pacc = part_acc + (size_t)par * NCW * DH;
      bool finish = item.active != 0;
      if (item.active) {
        const int b = item.bh / p.H, h = item.bh % p.H;
        float m = -INFINITY;
        for (int w = 0; w < NCW; ++w) m = fmaxf(m, sh.part_m[par][w]);
        float l = 0.f;
        int keys = 0;
        for (int w = 0; w < NCW; ++w) {
          if (sh.part_m[par][w] != -INFINITY) l += sh.part_l[par][w] * exp2f(sh.part_m[par][w] - m);
          keys += sh.part_rows[par][w];
        }
        T* orow = reinterpret_cast<T*>(p.out) + b * p.o_sb + h * DH;
        if (!SPLIT || item.np == 1) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          for (int d = lane; d < DH; d += 32) {
            float a = 0.f;
            for (int w = 0; w < NCW; ++w)
              if (sh.part_m[par][w] != -INFINITY) a += pacc[w * DH + d] * exp2f(sh.part_m[par][w] - m);
            orow[d] = from_f32<T>(a * inv);
          }
        } else {
          // this part's state to the scratch; the part that arrives last merges all of them (no waiting)
          float* prow = p.part + ((int64_t)(item.bh - NW) * PT + item.part) * (DH + 4);
          for (int d = lane; d < DH; d += 32) {
            float a = 0.f;
            for (int w = 0; w < NCW; ++w)
              if (sh.part_m[par][w] != -INFINITY) a += pacc[w * DH + d] * exp2f(sh.part_m[par][w] - m);
            prow[4 + d] = a;
          }
          if (lane == 0) {
            prow[0] = m;
            prow[1] = l;
            prow[2] = __int_as_float(keys);
          }
          __threadfence();
          __syncwarp();
          int last = 0;
          if (lane == 0) last = atomicAdd(&p.part_cnt[item.bh], 1) == PT - 1 ? 1 : 0;
          last = __shfl_sync(0xffffffffu, last, 0);
          finish = last != 0;
          if (finish) {
            __threadfence();
            const float* pb = p.part + (int64_t)(item.bh - NW) * PT * (DH + 4);
            m = -INFINITY;
            for (int j = 0; j < PT; ++j) m = fmaxf(m, __ldcg(pb + j * (DH + 4)));
            l = 0.f;
            keys = 0;
            for (int j = 0; j < PT; ++j) {
              const float mj = __ldcg(pb + j * (DH + 4));
              if (mj != -INFINITY) l += __ldcg(pb + j * (DH + 4) + 1) * exp2f(mj - m);
              keys += __float_as_int(__ldcg(pb + j * (DH + 4) + 2));
            }
            const float inv = l > 0.f ? 1.f / l : 0.f;
            for (int d = lane; d < DH; d += 32) {
              float a = 0.f;
              for (int j = 0; j < PT; ++j) {
                const float mj = __ldcg(pb + j * (DH + 4));
                if (mj != -INFINITY) a += __ldcg(pb + j * (DH + 4) + 4 + d) * exp2f(mj - m);
              }
              orow[d] = from_f32<T>(a * inv);
            }
            if (lane == 0) p.part_cnt[item.bh] = 0;
          }
        }
        if (finish && lane == 0) {
          if (p.lse) p.lse[item.bh] = l > 0.f ? (m + log2f(l)) * LN2 : -INFINITY;
          if (p.nkeys) p.nkeys[item.bh] = keys;
          if (p.sel) {
            int32_t* so = p.sel + (int64_t)item.bh * (p.wmax + 1);
            so[0] = item.nsel;
            for (int i = 0; i < p.wmax; ++i) so[1 + i] = i < item.nsel ? item.sel[i] : -1;
          }
        }
        if (finish) {
          // append this step's k / v rows at position t
          const int t = item.t;
          T* kc = reinterpret_cast<T*>(p.kc) + b * p.c_sb + h * p.c_sh;
          T* vc = reinterpret_cast<T*>(p.vc) + b * p.c_sb + h * p.c_sh;
          for (int c = lane; c < DH / VEC; c += 32) {
            *reinterpret_cast<uint4*>(kc + (int64_t)t * p.c_st + c * VEC) =
                *reinterpret_cast<const uint4*>(item.k + c * VEC);
            *reinterpret_cast<uint4*>(vc + (int64_t)t * p.c_st + c * VEC) =
                *reinterpret_cast<const uint4*>(item.v + c * VEC);
          }
          if (((t + 1) & (leaf - 1)) == 0)
            tree_update_warp<T, DH>(kc, p.c_st, item.k, t, p.nodes + b * p.lv.s_b + h * p.lv.s_h, p.lv, tu,
                                    Cfg::TU_FLOATS, lane);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sh.pfree[par]);
        mbar_arrive(&sh.iempty[slot]);
      }
    }
  } else {
    // ------------------------------------------------------------------ consumer warps
    const int cg = warp / WPG, wig = warp - cg * WPG;
    WA wa;
    int it = cg, k = 0, rows = 0;
    bool ok = true;
    while (true) {
      const int s = it % NST;
      if (!mbar_wait_bounded(&sh.full[s], (it / NST) & 1, K_DECODE, 3)) {
        ok = false;
        break;
      }
      const int n = sh.nrows[s];
      if (n < 0) {
        it += NCG;  // the sentinel counts as consumed
        break;
      }
      const int fl = sh.flags[s], slot = sh.slot[s];
      if (fl & STAGE_FIRST) {
        if (!mbar_wait_bounded(&sh.ifull[slot], (k / PSLOTS) & 1, K_DECODE, 4)) {
          ok = false;
          break;
        }
        PItem<T, DH>& item = sh.item[slot];
        wa.init(item.q, p.scale * LOG2E, lane);
        rows = 0;
        if (warp == 0 && item.active && (!SPLIT || item.part == 0)) {  // the new token (part 0 of a split item)
          wa.one_row(item.k, item.v);
          rows = 1;
        }
      }
      const T* kst = ring + (size_t)s * Cfg::STAGE_ELEMS;
      if constexpr (EARLY) {
        if (n > 0) wa.load(kst, kst + CH * DH, wig * WA::G, n);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.empty[s]);
        if (n > 0) wa.compute();
      } else {
        if (n > 0) wa.stage(kst, kst + CH * DH, n, wig, WPG);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.empty[s]);
      }
      if (wig == 0) rows += n;
      it += NCG;
      if (!(fl & STAGE_LAST)) continue;
      // ---------------------------------------------------------------- end of item k: hand the partial over
      const int par = k & 1;
      wa.reduce_rows();
      float* pacc = part_acc + (size_t)par * NCW * DH;
      if (k >= 2 && !mbar_wait_bounded(&sh.pfree[par], ((k >> 1) - 1) & 1, K_DECODE, 5)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        sh.part_m[par][warp] = wa.m;
        sh.part_l[par][warp] = wa.l;
        sh.part_rows[par][warp] = wig == 0 ? rows : 0;
      }
      if (wa.sub == 0) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) pacc[warp * DH + wa.c * VEC + i] = wa.acc[i];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.pready[par]);
      ++k;
    }
    if (!ok) atomicExch(&sh.abort_flag, 1);
    if (wig == 0 && lane == 0) sh.consumed[cg] = it;
    named_bar_sync(2, (NCW + NPROD) * 32);
  }
}

}  // namespace ta
