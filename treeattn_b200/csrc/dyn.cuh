// Dynamic content tree (reference dyntree.py, attn='dyn'): per-lane balanced binary trees over key prefixes.
//
// A lane's tree has capacity C (a power of two) key slots and levels 0..D, D = log2(C) - 1; level l has 2^l nodes,
// each holding the fp32 SUM of the keys below it and their count, packed level by level (level l at rows
// 2^l - 1 .. 2^(l+1) - 2 of a (2^(D+1) - 1, dh) block per lane); the last level's nodes are groups of two slots
// whose key positions are kept in `slot` (2^D, 2) int32, -1 = empty.
//
// Kernels:
//  * lane_split_kernel: one level of the build (dyntree.py:54-73): inside every group of S = C >> lvl slots the
//    valid keys are ordered by a 2-means projection (dyntree.py:6-31) and dealt to the two halves, ceil(n/2) left.
//    A "team" (a warp, or the 8 warps of a CTA for large groups) owns one group: one warp per key row with the
//    lanes over the head dim (coalesced 128-byte row reads, shuffle-reduced dots), per-warp partial centre sums
//    in registers reduced across the team in shared memory, and a bitonic sort of 64-bit (projection, slot) keys.
//  * lane_sums_kernel: the slots of the built tree and its node sums / counts bottom-up in adjacent pairs.
//  * lane_insert_kernel: dyntree.py:83-106, one warp per lane.
//  * lane_select_kernel: dyntree.py:150-243 select_keys, one warp per lane walking the lane's tokens in order:
//    neighbour rescoring, beam descent (lane_descend, shared with ta_lane_search), insertion; the tree stays in
//    global memory (L2) and is updated in place.
#pragma once
#include "select.cuh"

namespace ta {

// Ascending order key of a float: the unsigned order of the result is the float order (-0 counted as +0).
__device__ __forceinline__ uint32_t asc_bits(float x) {
  uint32_t u = __float_as_uint(x + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ------------------------------------------------------------------------------------------------ build: split
struct LaneSplitParams {
  const float* keys;         // fp32 key rows (dh floats each)
  int64_t key_lane_div;      // lanes sharing one key array: lane p reads keys + (p / key_lane_div) * key_stride
  int64_t key_stride;        // floats between key arrays
  const int32_t* perm_in;    // (P, C) key row of every slot
  const uint8_t* valid_in;   // (P, C)
  int32_t* perm_out;
  uint8_t* valid_out;
  int P, C, lvl, iters;
};

template <int NW>
__device__ __forceinline__ void team_sync() {
  if (NW == 1) __syncwarp(); else __syncthreads();
}

// Shared memory of one team: sort keys (S) | mean, c0, c1, diff (4 DH floats) | per-warp partials (2 NW DH) |
// per-warp scalars.
template <int NW, int DH>
struct SplitSmem {
  static __host__ __device__ size_t bytes(int S) {
    return (size_t)S * 8 + 4 * DH * 4 + (size_t)2 * NW * DH * 4 + NW * 32;
  }
};

template <int NW, int DH>
struct TwoMeans {
  static constexpr int NJ = (DH + 31) / 32;  // head dims per lane
  static constexpr int TEAM = NW * 32;

  // Team-sum of per-warp vectors acc[NJ] (lane owns dims lane + 32 j) into out[DH].
  static __device__ __forceinline__ void reduce_vec(const float (&acc)[NJ], float* red, float* out, int w, int lane,
                                                    int tid) {
    if (NW == 1) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int d = lane + 32 * j;
        if (d < DH) out[d] = acc[j];
      }
      __syncwarp();
      return;
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < DH) red[w * DH + d] = acc[j];
    }
    __syncthreads();
    for (int d = tid; d < DH; d += TEAM) {
      float s = 0.f;
      for (int i = 0; i < NW; ++i) s += red[i * DH + d];
      out[d] = s;
    }
    __syncthreads();
  }

  static __device__ __forceinline__ int reduce_int(int v, int* redi, int w, int lane) {
    if (NW == 1) return v;
    if (lane == 0) redi[w] = v;
    __syncthreads();
    int s = 0;
    for (int i = 0; i < NW; ++i) s += redi[i];
    __syncthreads();
    return s;
  }

  static __device__ __forceinline__ unsigned long long reduce_max(unsigned long long v, unsigned long long* redk,
                                                                  int w, int lane) {
    if (NW == 1) return v;
    if (lane == 0) redk[w] = v;
    __syncthreads();
    unsigned long long m = 0;
    for (int i = 0; i < NW; ++i) m = redk[i] > m ? redk[i] : m;
    __syncthreads();
    return m;
  }

  static __device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  }

  static __device__ __forceinline__ void load_row(const float* row, float (&x)[NJ], int lane) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      x[j] = d < DH ? __ldg(row + d) : 0.f;
    }
  }

  // Order the S slots of one group and write the split (dyntree.py:6-31 and 58-73). tid = thread in team.
  static __device__ void run(const LaneSplitParams& p, int64_t group, unsigned char* smem, int tid) {
    const int w = tid >> 5, lane = tid & 31;
    const int G = 1 << p.lvl;
    const int S = p.C >> p.lvl;
    const int64_t lanep = group / G;
    const int64_t base = lanep * p.C + (group % G) * (int64_t)S;
    const float* keys = p.keys + (lanep / p.key_lane_div) * p.key_stride;
    const int32_t* perm = p.perm_in + base;
    const uint8_t* valid = p.valid_in + base;

    unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem);
    float* mean = reinterpret_cast<float*>(smem + (size_t)S * 8);
    float* c0 = mean + DH;
    float* c1 = c0 + DH;
    float* diff = c1 + DH;
    float* red = diff + DH;                                   // 2 NW DH
    int* redi = reinterpret_cast<int*>(red + 2 * NW * DH);    // NW
    unsigned long long* redk = reinterpret_cast<unsigned long long*>(redi + 2 * NW);  // NW (8-byte aligned)

    // (1) count and mean of the valid keys
    float acc[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j] = 0.f;
    int nv = 0;
    for (int s = w; s < S; s += NW) {
      if (!valid[s]) continue;
      float x[NJ];
      load_row(keys + (int64_t)perm[s] * DH, x, lane);
#pragma unroll
      for (int j = 0; j < NJ; ++j) acc[j] += x[j];
      ++nv;
    }
    const int ng = reduce_int(nv, redi, w, lane);
    reduce_vec(acc, red, mean, w, lane, tid);
    for (int d = tid; d < DH; d += TEAM) mean[d] = mean[d] / (float)(ng > 1 ? ng : 1);
    team_sync<NW>();

    if (ng >= 1) {
      // (2) a = the valid key farthest from the mean, (3) b = the valid key farthest from a (first index on ties)
      for (int pass = 0; pass < 2; ++pass) {
        const float* ref = pass == 0 ? mean : c0;
        unsigned long long best = 0;
        for (int s = w; s < S; s += NW) {
          if (!valid[s]) continue;
          float x[NJ];
          load_row(keys + (int64_t)perm[s] * DH, x, lane);
          float v = 0.f;
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const int d = lane + 32 * j;
            const float e = d < DH ? x[j] - ref[d] : 0.f;
            v = fmaf(e, e, v);
          }
          v = warp_sum(v);
          const unsigned long long key = ((unsigned long long)asc_bits(v) << 32) | (uint32_t)(0xffffffffu - s);
          best = key > best ? key : best;
        }
        best = reduce_max(best, redk, w, lane);
        const int sel = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
        float* dst = pass == 0 ? c0 : c1;
        for (int d = tid; d < DH; d += TEAM) dst[d] = keys[(int64_t)perm[sel] * DH + d];
        team_sync<NW>();
      }
      // (4) 2-means rounds: nearer centre by |x|^2 - 2 x.c + |c|^2 (first centre on ties), centres to the means
      for (int it = 0; it < p.iters; ++it) {
        float q0 = 0.f, q1 = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int d = lane + 32 * j;
          if (d < DH) { q0 = fmaf(c0[d], c0[d], q0); q1 = fmaf(c1[d], c1[d], q1); }
        }
        const float csq0 = warp_sum(q0), csq1 = warp_sum(q1);
        float a0[NJ], a1[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) { a0[j] = 0.f; a1[j] = 0.f; }
        int n1 = 0, n0 = 0;
        for (int s = w; s < S; s += NW) {
          if (!valid[s]) continue;
          float x[NJ];
          load_row(keys + (int64_t)perm[s] * DH, x, lane);
          float xx = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const int d = lane + 32 * j;
            if (d < DH) { xx = fmaf(x[j], x[j], xx); d0 = fmaf(x[j], c0[d], d0); d1 = fmaf(x[j], c1[d], d1); }
          }
          xx = warp_sum(xx); d0 = warp_sum(d0); d1 = warp_sum(d1);
          const float dist0 = (xx - 2.f * d0) + csq0, dist1 = (xx - 2.f * d1) + csq1;
          if (dist1 < dist0) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) a1[j] += x[j];
            ++n1;
          } else {
#pragma unroll
            for (int j = 0; j < NJ; ++j) a0[j] += x[j];
            ++n0;
          }
        }
        const int m0 = reduce_int(n0, redi, w, lane);
        const int m1 = reduce_int(n1, redi, w, lane);
        // the team sums land in diff (centre 0) and mean (centre 1; the mean is no longer needed)
        reduce_vec(a0, red, diff, w, lane, tid);
        reduce_vec(a1, red + NW * DH, mean, w, lane, tid);
        for (int d = tid; d < DH; d += TEAM) {
          if (m0 > 0) c0[d] = diff[d] / (float)m0;
          if (m1 > 0) c1[d] = mean[d] / (float)m1;
        }
        team_sync<NW>();
      }
      for (int d = tid; d < DH; d += TEAM) diff[d] = c0[d] - c1[d];
      team_sync<NW>();
    }
    // (5) projections (valid keys) -> ascending (projection, slot) keys; empty slots last
    for (int s = w; s < S; s += NW) {
      uint32_t hi = 0xffffffffu;
      if (valid[s] && ng >= 1) {
        float x[NJ];
        load_row(keys + (int64_t)perm[s] * DH, x, lane);
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int d = lane + 32 * j;
          if (d < DH) v = fmaf(x[j], diff[d], v);
        }
        hi = asc_bits(warp_sum(v));
        if (hi == 0xffffffffu) hi = 0xfffffffeu;  // a NaN projection still sorts before the empty slots
      }
      if (lane == 0) skey[s] = ((unsigned long long)hi << 32) | (uint32_t)s;
    }
    team_sync<NW>();
    // bitonic sort, ascending
    for (int kk = 2; kk <= S; kk <<= 1) {
      for (int j = kk >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < S; i += TEAM) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const unsigned long long a = skey[i], b = skey[ixj];
            const bool up = (i & kk) == 0;
            if ((a > b) == up) { skey[i] = b; skey[ixj] = a; }
          }
        }
        team_sync<NW>();
      }
    }
    // (6) deal: sorted rank r < nl -> left half position r, nl <= r < ng -> right half position half + r - nl;
    // the free positions are empty and point at the last sorted slot (dyntree.py:66-71)
    const int nl = (ng + 1) / 2, nr = ng - nl, half = S >> 1;
    const int32_t last = perm[(int)(skey[S - 1] & 0xffffffffu)];
    int32_t* po = p.perm_out + base;
    uint8_t* vo = p.valid_out + base;
    for (int r = tid; r < S; r += TEAM) {
      if (r < ng) {
        const int s = (int)(skey[r] & 0xffffffffu);
        const int dst = r < nl ? r : half + (r - nl);
        po[dst] = perm[s];
        vo[dst] = 1;
      }
      const bool empty = r < half ? r >= nl : (r - half) >= nr;
      if (empty) {
        po[r] = last;
        vo[r] = 0;
      }
    }
  }
};

// Groups of > 256 slots: one group per CTA of 8 warps.
template <int DH>
__global__ void __launch_bounds__(256) lane_split_cta_kernel(LaneSplitParams p) {
  extern __shared__ __align__(16) unsigned char split_smem[];
  TwoMeans<8, DH>::run(p, blockIdx.x, split_smem, threadIdx.x);
}

// Groups of <= 256 slots: one group per warp, 8 per CTA.
template <int DH>
__global__ void __launch_bounds__(256) lane_split_warp_kernel(LaneSplitParams p, int64_t n_groups, int S) {
  extern __shared__ __align__(16) unsigned char split_smem[];
  const int w = threadIdx.x >> 5;
  const int64_t g = (int64_t)blockIdx.x * 8 + w;
  if (g >= n_groups) return;
  const size_t per = (SplitSmem<1, DH>::bytes(S) + 15) & ~(size_t)15;
  TwoMeans<1, DH>::run(p, g, split_smem + per * w, threadIdx.x & 31);
}

// ------------------------------------------------------------------------------------------------ build: sums
struct LaneSumsParams {
  const float* keys;
  int64_t key_lane_div, key_stride;
  const int32_t* perm;     // (P, C)
  const uint8_t* valid;    // (P, C)
  int P, C, D, dh;
  float* sums;             // (P, 2^(D+1) - 1, dh)
  int32_t* cnt;            // (P, 2^(D+1) - 1)
  int32_t* slot;           // (P, 2^D, 2)
};

// One CTA per lane: slots and level D from the key pairs, then every upper level from its children.
__global__ void __launch_bounds__(512) lane_sums_kernel(LaneSumsParams p) {
  const int64_t lanep = blockIdx.x;
  const int dh = p.dh, D = p.D;
  const int NN = (2 << D) - 1;
  const float* keys = p.keys + (lanep / p.key_lane_div) * p.key_stride;
  const int32_t* perm = p.perm + lanep * p.C;
  const uint8_t* valid = p.valid + lanep * p.C;
  float* sums = p.sums + lanep * (int64_t)NN * dh;
  int32_t* cnt = p.cnt + lanep * (int64_t)NN;
  int32_t* slot = p.slot + lanep * (int64_t)p.C;
  const int nD = 1 << D, offD = nD - 1;
  for (int i = threadIdx.x; i < p.C; i += blockDim.x) slot[i] = valid[i] ? perm[i] : -1;
  for (int m = threadIdx.x; m < nD; m += blockDim.x) cnt[offD + m] = (int)valid[2 * m] + (int)valid[2 * m + 1];
  for (int64_t e = threadIdx.x; e < (int64_t)nD * dh; e += blockDim.x) {
    const int m = (int)(e / dh), d = (int)(e - (int64_t)m * dh);
    const float x0 = valid[2 * m] ? keys[(int64_t)perm[2 * m] * dh + d] : 0.f;
    const float x1 = valid[2 * m + 1] ? keys[(int64_t)perm[2 * m + 1] * dh + d] : 0.f;
    sums[(int64_t)(offD + m) * dh + d] = x0 + x1;
  }
  __syncthreads();
  for (int l = D - 1; l >= 0; --l) {
    const int o = (1 << l) - 1, oc = (2 << l) - 1, n = 1 << l;
    for (int m = threadIdx.x; m < n; m += blockDim.x) cnt[o + m] = cnt[oc + 2 * m] + cnt[oc + 2 * m + 1];
    for (int64_t e = threadIdx.x; e < (int64_t)n * dh; e += blockDim.x) {
      const int m = (int)(e / dh), d = (int)(e - (int64_t)m * dh);
      sums[(int64_t)(o + m) * dh + d] =
          sums[(int64_t)(oc + 2 * m) * dh + d] + sums[(int64_t)(oc + 2 * m + 1) * dh + d];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ insert
// dyntree.py:83-106 for one lane, by one warp: the key joins the root, then at every level the child whose mean
// scores higher against it (kv . sum / count; -1e9 when empty, -inf when full; ties left), and the first free slot
// of the last group. kv in shared memory (DH floats). The warp's writes are ordered before its later reads.
template <int DH>
__device__ __forceinline__ void lane_insert_warp(float* sums, int32_t* cnt, int32_t* slot, const float* kv, int D,
                                                 int C, int32_t kpos, int lane) {
  constexpr int NJ = (DH + 31) / 32;
  float k[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int d = lane + 32 * j;
    k[j] = d < DH ? kv[d] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int d = lane + 32 * j;
    if (d < DH) sums[d] += k[j];
  }
  if (lane == 0) cnt[0] += 1;
  __syncwarp();
  int node = 0;
  for (int lvl = 0; lvl < D; ++lvl) {
    const int o = (2 << lvl) - 1;
    const int left = 2 * node, right = left + 1;
    const int cap = C >> (lvl + 1);
    const int cL = cnt[o + left], cR = cnt[o + right];
    const float* SL = sums + (int64_t)(o + left) * DH;
    const float* SR = sums + (int64_t)(o + right) * DH;
    float pl = 0.f, pr = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < DH) { pl = fmaf(k[j], SL[d], pl); pr = fmaf(k[j], SR[d], pr); }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      pl += __shfl_xor_sync(0xffffffffu, pl, off);
      pr += __shfl_xor_sync(0xffffffffu, pr, off);
    }
    float sL = pl / (float)(cL > 1 ? cL : 1), sR = pr / (float)(cR > 1 ? cR : 1);
    if (cL == 0) sL = -1e9f;
    if (cL >= cap) sL = -INFINITY;
    if (cR == 0) sR = -1e9f;
    if (cR >= cap) sR = -INFINITY;
    node = sR > sL ? right : left;
    float* dst = sums + (int64_t)(o + node) * DH;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < DH) dst[d] += k[j];
    }
    if (lane == 0) cnt[o + node] += 1;
    __syncwarp();
  }
  if (lane == 0) {
    const int s = slot[2 * node] >= 0 ? 1 : 0;
    slot[2 * node + s] = kpos;
  }
  __syncwarp();
}

struct LaneInsertParams {
  const float* kv;        // (P, dh)
  const int64_t* kpos;    // (P)
  const uint8_t* active;  // (P)
  int P, D, C;
  float* sums;
  int32_t* cnt;
  int32_t* slot;
};

template <int DH>
__global__ void __launch_bounds__(128) lane_insert_kernel(LaneInsertParams p) {
  __shared__ __align__(16) float kb[4][DH];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pl = (int64_t)blockIdx.x * 4 + warp;
  if (pl >= p.P || !p.active[pl]) return;
  const int NN = (2 << p.D) - 1;
  for (int d = lane; d < DH; d += 32) kb[warp][d] = p.kv[pl * DH + d];
  __syncwarp();
  lane_insert_warp<DH>(p.sums + pl * (int64_t)NN * DH, p.cnt + pl * (int64_t)NN, p.slot + pl * (int64_t)p.C,
                       kb[warp], p.D, p.C, (int32_t)p.kpos[pl], lane);
}

// ------------------------------------------------------------------------------------------------ select
struct LaneSelectParams {
  const float* q;          // (B, H, T, dh) fp32
  const float* k;          // (B, H, T, dh) fp32
  const int64_t* lhat;     // (B, H, T)
  float* sums;             // (P, NN, dh), P = B*H*nl lanes (lane = (b*H + h)*nl + l)
  int32_t* cnt;            // (P, NN)
  int32_t* slot;           // (P, 2^D, 2)
  int B, H, T, Y, nl, D, wmax, wl, Wn, NS, probe, cap_min, neighbors;
  float rho;
  int64_t* tree_pos;       // (B, H, T, 2 wl)
  uint8_t* leaf_ok;        // (B, H, T, wl)
  int64_t* nb_pos;         // (B, H, T, 2 Wn NS)
  int64_t* n_tree;         // (B, H, T)
  int64_t* nb_leaves;      // (B, H, T)
};

template <int DH>
__global__ void __launch_bounds__(128) lane_select_kernel(LaneSelectParams p) {
  __shared__ DescentScratch scr[4];
  __shared__ __align__(16) float kb[4][DH];
  __shared__ int32_t ring_id[4][32];
  __shared__ float ring_sc[4][32];
  __shared__ uint8_t ring_ok[4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pl = (int64_t)blockIdx.x * 4 + warp;
  const int64_t P = (int64_t)p.B * p.H * p.nl;
  if (pl >= P) return;
  DescentScratch& sc = scr[warp];
  const int64_t bh = pl / p.nl;
  const int start = (int)(pl % p.nl) * p.Y;
  const int NN = (2 << p.D) - 1, C = p.T;
  const int offD = (1 << p.D) - 1;
  float* sums = p.sums + pl * (int64_t)NN * DH;
  int32_t* cnt = p.cnt + pl * (int64_t)NN;
  int32_t* slot = p.slot + pl * (int64_t)C;
  const int W = p.Wn * p.NS, wl = p.wl;
  ring_ok[warp][lane] = 0;
  ring_id[warp][lane] = 0;
  ring_sc[warp][lane] = 0.f;
  __syncwarp();
  for (int i = 0; i < p.Y; ++i) {
    const int t = start + i;
    const int64_t row = bh * p.T + t;
    for (int d = lane; d < DH; d += 32) {
      sc.qf[d] = p.q[row * DH + d];
      kb[warp][d] = p.k[row * DH + d];
    }
    __syncwarp();
    // (1) neighbour search over the groups stored by the previous Wn queries of this lane (dyntree.py:197-214)
    const int j = lane;
    const int dist = j / p.NS + 1, sl = j - (j / p.NS) * p.NS;
    const bool jval = j < W && dist <= i;
    int id = 0;
    float base = 0.f;
    bool ok0 = false;
    if (jval) {
      const int r = ((i - dist) % p.Wn) * p.NS + sl;
      id = ring_id[warp][r];
      base = ring_sc[warp][r];
      ok0 = ring_ok[warp][r] != 0;
    }
    bool m = false;
    if (ok0) {
      const int cn = cnt[offD + id];
      const float* nrow = sums + (int64_t)(offD + id) * DH;
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int cc = 0; cc < DH / 4; ++cc) {
        const float4 qv = *reinterpret_cast<const float4*>(sc.qf + cc * 4);
        const float4 v = *reinterpret_cast<const float4*>(nrow + cc * 4);
        if (cc & 1) {
          a1 = fmaf(qv.x, v.x, a1); a1 = fmaf(qv.y, v.y, a1); a1 = fmaf(qv.z, v.z, a1); a1 = fmaf(qv.w, v.w, a1);
        } else {
          a0 = fmaf(qv.x, v.x, a0); a0 = fmaf(qv.y, v.y, a0); a0 = fmaf(qv.z, v.z, a0); a0 = fmaf(qv.w, v.w, a0);
        }
      }
      const float st = __fdiv_rn(__fadd_rn(a0, a1), (float)(cn > 1 ? cn : 1));
      const float thr = __fsub_rn(base, __fmul_rn(p.rho, fabsf(base)));
      m = cn > 0 && st >= thr;
    }
    const unsigned pm = p.probe >= 32 ? 0xffffffffu : ((1u << p.probe) - 1u);
    const unsigned bm = __ballot_sync(0xffffffffu, m), bo = __ballot_sync(0xffffffffu, ok0);
    const int nmt = __popc(bm & pm), no = __popc(bo & pm);
    const float rate = __fdiv_rn((float)nmt, (float)(no > 1 ? no : 1));
    const int cap = p.cap_min + (int)rintf(__fmul_rn((float)(p.Wn - p.cap_min), rate));
    m = m && dist <= cap && p.neighbors != 0;
    const unsigned long long key = m ? (unsigned long long)id : (0xffffffff00000000ull | (unsigned)lane);
    const unsigned same = __match_any_sync(0xffffffffu, key);
    const bool first = m && (__ffs(same) - 1) == lane;
    const int nL = __popc(__ballot_sync(0xffffffffu, first));
    if (j < W) {
      int32_t n0 = -1, n1 = -1;
      if (m) { n0 = slot[2 * id]; n1 = slot[2 * id + 1]; }
      p.nb_pos[row * 2 * W + j] = n0 < 0 ? -1 : n0;
      p.nb_pos[row * 2 * W + W + j] = n1 < 0 ? -1 : n1;
    }
    // (2) the tree's budget and the beam descent (dyntree.py:216-227)
    const int64_t L = p.lhat[row];
    const int64_t lo = (L + 1) / 2;
    const int64_t need = L - nL > 0 ? L - nL : 0;
    const int64_t floor_b = nL < lo ? 2 : 1;
    int64_t b_tree = nL >= L ? 0 : (need > floor_b ? need : floor_b);
    b_tree = b_tree < p.wmax ? b_tree : p.wmax;
    const int nk = lane_descend<DH>(sums, cnt, p.D, p.wmax, sc, lane);
    for (int x = lane; x < wl; x += 32) {
      const bool ok = x < nk;
      int32_t s0 = -1, s1 = -1;
      if (ok) { s0 = slot[2 * sc.kid[x]]; s1 = slot[2 * sc.kid[x] + 1]; }
      p.tree_pos[row * 2 * wl + x] = s0 < 0 ? -1 : s0;
      p.tree_pos[row * 2 * wl + wl + x] = s1 < 0 ? -1 : s1;
      p.leaf_ok[row * wl + x] = ok ? 1 : 0;
    }
    if (lane == 0) {
      p.n_tree[row] = b_tree;
      p.nb_leaves[row] = nL;
    }
    __syncwarp();
    if (lane < p.NS) {
      const int r = (i % p.Wn) * p.NS + lane;
      const bool ok = lane < nk;
      ring_id[warp][r] = ok ? sc.kid[lane] : 0;
      ring_sc[warp][r] = ok ? sc.ksc[lane] : -INFINITY;
      ring_ok[warp][r] = ok ? 1 : 0;
    }
    __syncwarp();
    // (3) the token's key joins the tree (the sink, position 0, never does)
    if (t >= 1) lane_insert_warp<DH>(sums, cnt, slot, kb[warp], p.D, C, t, lane);
    __syncwarp();
  }
}

}  // namespace ta
