// Block forest (reference forest.py, attention.py; attn='block'): one content-sorted binary tree per block of B
// keys. The content sort is the dynamic tree's 2-means split with every slot valid (ta_lane_order); this file has
// the per-block node sums (with the optional soft mean-log gate) and the per-query descent over the trees of the
// earlier blocks.
#pragma once
#include "dyn.cuh"

namespace ta {

constexpr int FOREST_MAX_LEVELS = 9;  // blocks of up to 512 keys

// ------------------------------------------------------------------------------------------------ node sums
// forest.py:68-75: level l of block p has 2^l nodes; node m sums the keys of ranks [m B / 2^l, (m + 1) B / 2^l)
// (rank r = the key at local position perm[p][r]). One CTA per block: the keys are staged in rank order in fp32,
// the sums (and, with the gate, the sums of log|x| + 1e-6) are formed bottom-up in adjacent pairs, each level is
// written in the keys' dtype. With the gate (forest.py:36-44), one warp per node: ml = log-sum / size,
// thr = torch.quantile(ml, gate_q), g = sigmoid((ml - thr) / gate_temp), out = (sm * g) * (dh / max(sum g, 1)) with
// sm the node sum rounded to the keys' dtype.
struct ForestLevelsParams {
  const void* k;            // (P * B, dh): block p's keys at rows p B .. p B + B - 1
  const int32_t* perm;      // (P, B)
  int P, B, depth, nb, zero_sink, gate;
  float gate_q, gate_temp;
  void* out[FOREST_MAX_LEVELS];  // level l: (P 2^l, dh)
};

template <typename T, int DH>
__global__ void __launch_bounds__(256) forest_levels_kernel(ForestLevelsParams p) {
  extern __shared__ __align__(16) float fl_smem[];
  constexpr int NPL = (DH + 31) / 32;
  const int64_t blk = blockIdx.x;
  const int B = p.B;
  float* cur = fl_smem;                 // B/2 x DH: the sums of the current level
  float* nxt = cur + (B / 2) * DH;      // B/4 x DH
  float* lcur = nxt + (B / 4) * DH;     // log sums, same shapes
  float* lnxt = lcur + (B / 2) * DH;
  const T* kb = reinterpret_cast<const T*>(p.k) + blk * (int64_t)B * DH;
  const int32_t* perm = p.perm + blk * (int64_t)B;
  const bool sink_block = p.zero_sink && (blk % p.nb) == 0;
  // level depth (groups of 2 keys in rank order)
  for (int e = threadIdx.x; e < (B / 2) * DH; e += blockDim.x) {
    const int m = e / DH, d = e - m * DH;
    const int i0 = perm[2 * m], i1 = perm[2 * m + 1];
    const float x0 = (sink_block && i0 == 0) ? 0.f : to_f32(kb[(int64_t)i0 * DH + d]);
    const float x1 = (sink_block && i1 == 0) ? 0.f : to_f32(kb[(int64_t)i1 * DH + d]);
    cur[e] = x0 + x1;
    if (p.gate) lcur[e] = log_mag(x0) + log_mag(x1);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int l = p.depth; l >= 0; --l) {
    const int n = 1 << l;
    T* out = reinterpret_cast<T*>(p.out[l]) + (blk << l) * (int64_t)DH;
    if (!p.gate) {
      for (int e = threadIdx.x; e < n * DH; e += blockDim.x) out[e] = from_f32<T>(cur[e]);
    } else {
      const float inv_size = __int_as_float((127 - (p.depth + 1 - l)) << 23);  // 1 / (B >> l), exact
      for (int m = warp; m < n; m += nw) {
        float sm[NPL], ml[NPL];
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          const int d = i * 32 + lane;
          const bool on = d < DH;
          sm[i] = on ? to_f32(from_f32<T>(cur[m * DH + d])) : 0.f;
          ml[i] = on ? lcur[m * DH + d] * inv_size : INFINITY;
        }
        const float thr = warp_quantile<DH>(ml, p.gate_q, lane);
        float g[NPL], gs = 0.f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          const bool on = i * 32 + lane < DH;
          const float z = __fdiv_rn(__fsub_rn(ml[i], thr), p.gate_temp);
          g[i] = on ? 1.0f / (1.0f + expf(-z)) : 0.f;
          gs += g[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
        const float scale = __fdiv_rn((float)DH, gs > 1.f ? gs : 1.f);
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          const int d = i * 32 + lane;
          if (d < DH) out[m * DH + d] = from_f32<T>(__fmul_rn(__fmul_rn(sm[i], g[i]), scale));
        }
      }
    }
    if (l == 0) break;
    for (int e = threadIdx.x; e < (n / 2) * DH; e += blockDim.x) {
      const int m = e / DH, d = e - m * DH;
      nxt[e] = cur[(2 * m) * DH + d] + cur[(2 * m + 1) * DH + d];
      if (p.gate) lnxt[e] = lcur[(2 * m) * DH + d] + lcur[(2 * m + 1) * DH + d];
    }
    __syncthreads();
    float* t = cur; cur = nxt; nxt = t;
    t = lcur; lcur = lnxt; lnxt = t;
  }
}

// forest.py:36-44 soft_gate on explicit nodes: sm (N, dh) node sums, grp (N, S, dh) their member keys; one warp per
// node as in forest_levels_kernel (the log-magnitude mean summed over the members in order).
template <typename T, int DH>
__global__ void __launch_bounds__(128) soft_gate_kernel(const T* __restrict__ sm, const T* __restrict__ grp,
                                                       T* __restrict__ out, int64_t N, int S, float gate_q,
                                                       float gate_temp) {
  constexpr int NPL = (DH + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int64_t node = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (node >= N) return;
  float v[NPL], ml[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int d = i * 32 + lane;
    const bool on = d < DH;
    v[i] = on ? to_f32(sm[node * DH + d]) : 0.f;
    float a = 0.f;
    if (on)
      for (int s = 0; s < S; ++s) a += log_mag(to_f32(grp[(node * S + s) * DH + d]));
    ml[i] = on ? __fdiv_rn(a, (float)S) : INFINITY;
  }
  const float thr = warp_quantile<DH>(ml, gate_q, lane);
  float g[NPL], gs = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const float z = __fdiv_rn(__fsub_rn(ml[i], thr), gate_temp);
    g[i] = i * 32 + lane < DH ? 1.0f / (1.0f + expf(-z)) : 0.f;
    gs += g[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
  const float scale = __fdiv_rn((float)DH, gs > 1.f ? gs : 1.f);
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int d = i * 32 + lane;
    if (d < DH) out[node * DH + d] = from_f32<T>(__fmul_rn(__fmul_rn(v[i], g[i]), scale));
  }
}

// ------------------------------------------------------------------------------------------------ descent
// attention.py:73-90 and 112-118, one warp per query t of (b, h) in block blk = t / B: level 0 scores the roots of
// the blocks 0..blk-1 (q . sum, rounded to the keys' dtype as a torch einsum of that dtype would), keeps the best
// min(wmax, width) (ties by the smaller node id), of which the first bq stay valid; each level's candidates are the
// two children of the valid kept nodes, down to level depth (groups of two keys). Output per query: the leaf ids
// and validity (wl), the key positions tkey[j wl + i] = block B + perm[block][2 m + j] of leaf i = block 2^depth + m,
// and tok = valid and not one of the static keys (the sink and the two previous tokens when in earlier blocks).
// Optionally the kept lists of every level (the routing loss's candidates).
struct ForestSelectParams {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const void* lv[FOREST_MAX_LEVELS];  // level sums (Bn H nb 2^l, dh)
  const int32_t* perm;                // (Bn H nb, B)
  const int64_t* bq;                  // (Bn, H, T) valid budget per query, or null (bq_const)
  int bq_const;
  int Bn, H, T, B, nb, depth, wmax, wl;
  int64_t* leaf;                      // (Bn, H, T, wl)
  uint8_t* leafv;                     // (Bn, H, T, wl)
  int64_t* tkey;                      // (Bn, H, T, 2 wl)
  uint8_t* tok;                       // (Bn, H, T, 2 wl)
  int32_t* lsel[FOREST_MAX_LEVELS];   // optional: (Bn, H, T, w_l) kept node ids of level l (0 = invalid slot)
  uint8_t* lselv[FOREST_MAX_LEVELS];
};

// q . row for one node row (16-byte loads through the read-only path), rounded to T as a T-typed einsum.
template <typename T, int DH>
__device__ __forceinline__ float forest_score(const float* qf, const T* row) {
  constexpr int V = 16 / sizeof(T);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int c = 0; c < DH; c += V) {
    float x[V];
    ldg_vec_f32<T>(row + c, x);
#pragma unroll
    for (int i = 0; i < V; i += 2) {
      a0 = fmaf(qf[c + i], x[i], a0);
      a1 = fmaf(qf[c + i + 1], x[i + 1], a1);
    }
  }
  return to_f32(from_f32<T>(a0 + a1));
}

template <typename T, int DH>
__global__ void __launch_bounds__(128) forest_select_kernel(ForestSelectParams p) {
  __shared__ DescentScratch scr[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.Bn * p.H * p.T) return;
  DescentScratch& sc = scr[warp];
  const int t = (int)(qid % p.T);
  const int64_t bh = qid / p.T;
  const int b = (int)(bh / p.H), h = (int)(bh % p.H);
  const int blk = t / p.B;
  const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + (int64_t)t * p.q_st;
  for (int d = lane; d < DH; d += 32) sc.qf[d] = to_f32(qrow[d]);
  __syncwarp();
  const int bq = p.bq ? (int)p.bq[qid] : p.bq_const;
  // level 0: running top-w over the earlier blocks' roots in chunks
  const T* lv0 = reinterpret_cast<const T*>(p.lv[0]) + bh * (int64_t)p.nb * DH;
  int w = p.wmax < p.nb ? p.wmax : p.nb;
  int nk = 0;
  for (int c0 = 0; c0 < blk;) {
    // candidates: the kept ones so far, then as many new roots as fit
    for (int i = lane; i < nk; i += 32) {
      sc.cid[i] = sc.kid[i];
      sc.csc[i] = sc.ksc[i];
      sc.ckey[i] = order_key(sc.ksc[i], sc.kid[i]);
    }
    const int take = min(blk - c0, CAND_LIMIT - nk);
    for (int j = lane; j < take; j += 32) {
      const int id = c0 + j;
      const float s = forest_score<T, DH>(sc.qf, lv0 + (int64_t)id * DH);
      sc.cid[nk + j] = id;
      sc.csc[nk + j] = s;
      sc.ckey[nk + j] = order_key(s, id);
    }
    __syncwarp();
    const int n = nk + take;
    nk = Descent<DH>::topk(n, min(w, n), sc, lane);
    __syncwarp();
    c0 += take;
  }
  int nvk = nk < bq ? nk : bq;  // valid kept nodes
  if (p.lsel[0]) {
    for (int i = lane; i < w; i += 32) {
      p.lsel[0][qid * w + i] = i < nk ? sc.kid[i] : 0;
      p.lselv[0][qid * w + i] = i < nvk ? 1 : 0;
    }
  }
  int wc = w;
  for (int l = 1; l <= p.depth; ++l) {
    const T* lvl = reinterpret_cast<const T*>(p.lv[l]) + bh * ((int64_t)p.nb << l) * DH;
    wc = 2 * w;                     // candidates of this level (valid or not)
    const int n = 2 * nvk;          // the valid ones: both children of every valid kept node
    for (int j = lane; j < n; j += 32) {
      const int par = sc.kid[j < nvk ? j : j - nvk];
      const int id = 2 * par + (j < nvk ? 0 : 1);
      sc.cid[j] = id;
    }
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
      const int id = sc.cid[j];
      const float s = forest_score<T, DH>(sc.qf, lvl + (int64_t)id * DH);
      sc.csc[j] = s;
      sc.ckey[j] = order_key(s, id);
    }
    __syncwarp();
    w = p.wmax < wc ? p.wmax : wc;
    nk = Descent<DH>::topk(n, min(w, n), sc, lane);
    __syncwarp();
    nvk = nk < bq ? nk : bq;
    if (p.lsel[l]) {
      for (int i = lane; i < w; i += 32) {
        p.lsel[l][qid * w + i] = i < nk ? sc.kid[i] : 0;
        p.lselv[l][qid * w + i] = i < nvk ? 1 : 0;
      }
    }
  }
  // leaves -> key positions; static keys of this query: 0, t-1, t-2 when before its block
  const int lim = blk * p.B;
  const int32_t* perm = p.perm;
  for (int i = lane; i < p.wl; i += 32) {
    const bool ok = i < nvk;
    const int id = ok ? sc.kid[i] : 0;
    p.leaf[qid * p.wl + i] = id;
    p.leafv[qid * p.wl + i] = ok ? 1 : 0;
    const int bl = id >> p.depth, m = id & ((1 << p.depth) - 1);
    for (int j = 0; j < 2; ++j) {
      int64_t key = -1;
      bool keep = false;
      if (ok) {
        key = (int64_t)bl * p.B + perm[(bh * p.nb + bl) * (int64_t)p.B + 2 * m + j];
        const bool dup = (key == 0 && 0 < lim) || (key == t - 1 && t - 1 >= 0 && t - 1 < lim) ||
                         (key == t - 2 && t - 2 >= 0 && t - 2 < lim);
        keep = !dup;
      }
      p.tkey[qid * 2 * p.wl + j * p.wl + i] = key;
      p.tok[qid * 2 * p.wl + j * p.wl + i] = keep ? 1 : 0;
    }
  }
}

}  // namespace ta
