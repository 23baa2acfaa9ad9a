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
//    A "team" (a warp, or the 8 warps of a CTA for large groups) owns one group: dh/8 lanes per key row, 8 head
//    dims each (two 16-byte loads), so a warp holds 32 / (dh/8) rows at once, two such steps in flight; per-row
//    dots reduce over the row's lanes, partial centre sums stay in registers until the end of a pass and are
//    reduced across the team in shared memory; then a bitonic sort of 64-bit (projection, slot) keys.
//  * lane_sums_kernel: the slots of the built tree and its node sums / counts bottom-up in adjacent pairs.
//  * lane_insert_kernel: dyntree.py:83-106, one warp per lane.
//  * lane_select_kernel: dyntree.py:150-243 select_keys, one warp per lane walking the lane's tokens in order:
//    neighbour rescoring, beam descent (lane_descend_t, shared with ta_lane_search), insertion; the tree's upper
//    levels are copied to shared memory for the loop and written back after it, the rest is updated in place in
//    global memory (L2).
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

// Barrier of a team of NW warps: the warp itself, the whole CTA (bid 0), or named barrier bid of NW warps.
template <int NW>
__device__ __forceinline__ void team_sync(int bid) {
  if (NW == 1) {
    __syncwarp();
  } else if (bid == 0) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(bid), "r"(NW * 32) : "memory");
  }
}

// Shared memory of one team: sort keys (S) | mean, c0, c1, diff (4 DH floats) | per-warp partials (2 NW DH) |
// per-warp scalars.
template <int NW, int DH>
struct SplitSmem {
  static __host__ __device__ size_t bytes(int S) {
    return (size_t)S * 8 + 4 * DH * 4 + (size_t)2 * NW * DH * 4 + NW * 32;
  }
};

// Place of the 16-byte chunk c (head dims 4c .. 4c + 3) inside a staged key row: the even chunks first, then the
// odd ones. Lane `sub` of a row reads chunks 2 sub and 2 sub + 1 (dims 8 sub .. 8 sub + 7), i.e. places sub and
// DH / 8 + sub: consecutive 16-byte places across the lanes, on distinct banks (in natural order the lanes'
// chunks are 32 bytes apart and two lanes of every eight meet on the same banks).
template <int DH>
__host__ __device__ constexpr int stage_chunk(int c) { return (c >> 1) + (DH / 8) * (c & 1); }

// SWZ: the key rows are a shared-memory stage whose 16-byte chunks are placed by stage_chunk (below), so that the
// two loads of the LPR lanes of a row each fall on distinct banks; otherwise rows are plain (global memory).
template <int NW, int DH, bool SWZ = false>
struct TwoMeans {
  // Each key row is read by LPR lanes holding 8 consecutive head dims each (two 16-byte loads), so a warp holds
  // RPW rows at once and U such steps are in flight per iteration; per-row dots reduce over the LPR lanes only.
  static constexpr int LPR = DH / 8;
  static constexpr int RPW = 32 / LPR;
  static constexpr int U = 2;
  static constexpr int STEP = NW * RPW * U;  // rows per team iteration
  static constexpr int TEAM = NW * 32;

  static __device__ __forceinline__ float row_sum(float v) {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  }

  // Sum a per-lane 8-dim vector over the RPW row slots of the warp (lanes with the same dim chunk).
  static __device__ __forceinline__ void slots_sum(float (&a)[8]) {
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int d = 0; d < 8; ++d) a[d] += __shfl_xor_sync(0xffffffffu, a[d], o);
  }

  static __device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  }

  static __device__ __forceinline__ unsigned long long warp_kmax(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
      v = u > v ? u : v;
    }
    return v;
  }

  // Team sum of the warps' 8-dim chunks (already summed over the warp's row slots) into out[DH].
  static __device__ __forceinline__ void team_vec(const float (&a)[8], float* red, float* out, int w, int lane,
                                                  int tid, int bid) {
    const int sub = lane % LPR;
    if (lane < LPR) {
#pragma unroll
      for (int d = 0; d < 8; ++d) red[w * DH + sub * 8 + d] = a[d];
    }
    team_sync<NW>(bid);
    for (int d = tid; d < DH; d += TEAM) {
      float s = 0.f;
      for (int i = 0; i < NW; ++i) s += red[i * DH + d];
      out[d] = s;
    }
    team_sync<NW>(bid);
  }

  static __device__ __forceinline__ int team_int(int v, int* redi, int w, int lane, int bid) {
    if (NW == 1) return v;
    if (lane == 0) redi[w] = v;
    team_sync<NW>(bid);
    int s = 0;
    for (int i = 0; i < NW; ++i) s += redi[i];
    team_sync<NW>(bid);
    return s;
  }

  static __device__ __forceinline__ unsigned long long team_kmax(unsigned long long v, unsigned long long* redk,
                                                                 int w, int lane, int bid) {
    if (NW == 1) return v;
    if (lane == 0) redk[w] = v;
    team_sync<NW>(bid);
    unsigned long long m = 0;
    for (int i = 0; i < NW; ++i) m = redk[i] > m ? redk[i] : m;
    team_sync<NW>(bid);
    return m;
  }

  // Load this lane's 8 dims of rows base + u*RPW + slot (u < U); rows past S or empty load as absent.
  static __device__ __forceinline__ void load_rows(const float* keys, const int32_t* perm, const uint8_t* valid,
                                                   int S, int base, int slot, int sub, float (&x)[U][8],
                                                   bool (&ok)[U], int (&s_of)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = base + u * RPW + slot;
      s_of[u] = s;
      ok[u] = s < S && valid[s];
      if (ok[u]) {
        const float4* r = reinterpret_cast<const float4*>(keys + (int64_t)perm[s] * DH);
        const float4 a = SWZ ? r[sub] : r[2 * sub], b = SWZ ? r[LPR + sub] : r[2 * sub + 1];
        x[u][0] = a.x; x[u][1] = a.y; x[u][2] = a.z; x[u][3] = a.w;
        x[u][4] = b.x; x[u][5] = b.y; x[u][6] = b.z; x[u][7] = b.w;
      } else {
#pragma unroll
        for (int d = 0; d < 8; ++d) x[u][d] = 0.f;
      }
    }
  }

  static __device__ __forceinline__ void load_vec(const float* v, int sub, float (&r)[8]) {
#pragma unroll
    for (int d = 0; d < 8; ++d) r[d] = v[sub * 8 + d];
  }

  // Order the S slots of one group and write the split (dyntree.py:6-31 and 58-73). Slot s holds key row
  // keys + perm[s] * DH (global or shared memory) when valid[s]; the split is written to po / vo (other arrays
  // than perm / valid). tid = thread in team, bid = the team's barrier (see team_sync).
  static __device__ void run(const float* keys, const int32_t* perm, const uint8_t* valid, int S, int iters,
                             int32_t* po, uint8_t* vo, unsigned char* smem, int tid, int bid) {
    const int w = tid >> 5, lane = tid & 31;
    const int slot = lane / LPR, sub = lane % LPR;

    unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem);
    float* mean = reinterpret_cast<float*>(smem + (size_t)S * 8);
    float* c0 = mean + DH;
    float* c1 = c0 + DH;
    float* diff = c1 + DH;
    float* red = diff + DH;                                   // 2 NW DH
    int* redi = reinterpret_cast<int*>(red + 2 * NW * DH);    // 2 NW
    unsigned long long* redk = reinterpret_cast<unsigned long long*>(redi + 2 * NW);  // NW

    float x[U][8];
    bool ok[U];
    int s_of[U];

    // (0) count the valid keys and find the end of the last one: the passes below stop there (the builds keep each
    // group's valid slots in front, so the slots past Se are empty). With at most two keys there is nothing to
    // cluster: the split is one key per side (in either orientation, both keys being equally far from their mean)
    // and the 2-means passes are skipped.
    int nv = 0, vend = 0;
    for (int r = tid; r < S; r += TEAM)
      if (valid[r]) {
        ++nv;
        vend = r + 1;
      }
    const int ng = team_int(warp_isum(nv), redi, w, lane, bid);
    const int Se = (int)team_kmax(warp_kmax((unsigned long long)vend), redk, w, lane, bid);
    if (ng <= 2) {
      for (int r = tid; r < S; r += TEAM)
        skey[r] = ((unsigned long long)(valid[r] ? 0u : 0xffffffffu) << 32) | (uint32_t)r;
    } else {
    // (1) mean of the valid keys
    float acc[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[d] = 0.f;
    for (int b = w * RPW * U; b < Se; b += STEP) {
      load_rows(keys, perm, valid, S, b, slot, sub, x, ok, s_of);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int d = 0; d < 8; ++d) acc[d] += x[u][d];
    }
    slots_sum(acc);
    team_vec(acc, red, mean, w, lane, tid, bid);
    for (int d = tid; d < DH; d += TEAM) mean[d] = mean[d] / (float)ng;
    team_sync<NW>(bid);

    {
      // (2) a = the valid key farthest from the mean, (3) b = the valid key farthest from a (first index on ties)
      for (int pass = 0; pass < 2; ++pass) {
        float ref[8];
        load_vec(pass == 0 ? mean : c0, sub, ref);
        unsigned long long best = 0;
        for (int b = w * RPW * U; b < Se; b += STEP) {
          load_rows(keys, perm, valid, S, b, slot, sub, x, ok, s_of);
          float v[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            v[u] = 0.f;
#pragma unroll
            for (int d = 0; d < 8; ++d) {
              const float e = x[u][d] - ref[d];
              v[u] = fmaf(e, e, v[u]);
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const float t = row_sum(v[u]);
            if (ok[u]) {
              const unsigned long long key =
                  ((unsigned long long)asc_bits(t) << 32) | (uint32_t)(0xffffffffu - s_of[u]);
              best = key > best ? key : best;
            }
          }
        }
        best = team_kmax(warp_kmax(best), redk, w, lane, bid);
        const int sel = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
        float* dst = pass == 0 ? c0 : c1;
        for (int d = tid; d < DH; d += TEAM)
          dst[d] = keys[(int64_t)perm[sel] * DH + (SWZ ? stage_chunk<DH>(d >> 2) * 4 + (d & 3) : d)];
        team_sync<NW>(bid);
      }
      // (4) 2-means rounds: nearer centre by |x|^2 - 2 x.c + |c|^2 (first centre on ties), centres to the means
      for (int it = 0; it < iters; ++it) {
        float r0[8], r1[8];
        load_vec(c0, sub, r0);
        load_vec(c1, sub, r1);
        float q0 = 0.f, q1 = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) { q0 = fmaf(r0[d], r0[d], q0); q1 = fmaf(r1[d], r1[d], q1); }
        const float csq0 = row_sum(q0), csq1 = row_sum(q1);
        float a0[8], a1[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) { a0[d] = 0.f; a1[d] = 0.f; }
        int n0 = 0, n1 = 0;
        for (int b = w * RPW * U; b < Se; b += STEP) {
          load_rows(keys, perm, valid, S, b, slot, sub, x, ok, s_of);
          float xx[U], d0[U], d1[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            xx[u] = 0.f; d0[u] = 0.f; d1[u] = 0.f;
#pragma unroll
            for (int d = 0; d < 8; ++d) {
              xx[u] = fmaf(x[u][d], x[u][d], xx[u]);
              d0[u] = fmaf(x[u][d], r0[d], d0[u]);
              d1[u] = fmaf(x[u][d], r1[d], d1[u]);
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const float sx = row_sum(xx[u]), s0 = row_sum(d0[u]), s1 = row_sum(d1[u]);
            const float dist0 = (sx - 2.f * s0) + csq0, dist1 = (sx - 2.f * s1) + csq1;
            const bool one = dist1 < dist0;
            if (ok[u]) {
              if (one) {
#pragma unroll
                for (int d = 0; d < 8; ++d) a1[d] += x[u][d];
                n1 += sub == 0 ? 1 : 0;
              } else {
#pragma unroll
                for (int d = 0; d < 8; ++d) a0[d] += x[u][d];
                n0 += sub == 0 ? 1 : 0;
              }
            }
          }
        }
        slots_sum(a0);
        slots_sum(a1);
        const int m0 = team_int(warp_isum(n0), redi, w, lane, bid);
        const int m1 = team_int(warp_isum(n1), redi + NW, w, lane, bid);
        // the team sums land in diff (centre 0) and mean (centre 1; the mean is no longer needed)
        team_vec(a0, red, diff, w, lane, tid, bid);
        team_vec(a1, red + NW * DH, mean, w, lane, tid, bid);
        for (int d = tid; d < DH; d += TEAM) {
          if (m0 > 0) c0[d] = diff[d] / (float)m0;
          if (m1 > 0) c1[d] = mean[d] / (float)m1;
        }
        team_sync<NW>(bid);
      }
      for (int d = tid; d < DH; d += TEAM) diff[d] = c0[d] - c1[d];
      team_sync<NW>(bid);
    }
    // (5) projections (valid keys) -> ascending (projection, slot) keys; empty slots last
    {
      float df[8];
      load_vec(diff, sub, df);
      for (int b = w * RPW * U; b < Se; b += STEP) {
        load_rows(keys, perm, valid, S, b, slot, sub, x, ok, s_of);
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          v[u] = 0.f;
#pragma unroll
          for (int d = 0; d < 8; ++d) v[u] = fmaf(x[u][d], df[d], v[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float t = row_sum(v[u]);
          uint32_t hi = 0xffffffffu;
          if (ok[u]) {
            hi = asc_bits(t);
            if (hi == 0xffffffffu) hi = 0xfffffffeu;  // a NaN projection still sorts before the empty slots
          }
          if (sub == 0 && s_of[u] < Se) skey[s_of[u]] = ((unsigned long long)hi << 32) | (uint32_t)s_of[u];
        }
      }
      for (int r = Se + tid; r < S; r += TEAM) skey[r] = (0xffffffffull << 32) | (uint32_t)r;
    }
    }
    team_sync<NW>(bid);
    // bitonic sort, ascending, of the first Sp keys (the power of two that covers Se): the keys past it are empty
    // slots in slot order, above every key before them, so they are in place already
    int Sp = 2;
    while (Sp < Se) Sp <<= 1;
    for (int kk = 2; kk <= Sp; kk <<= 1) {
      for (int j = kk >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < Sp; i += TEAM) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const unsigned long long a = skey[i], b = skey[ixj];
            const bool up = (i & kk) == 0;
            if ((a > b) == up) { skey[i] = b; skey[ixj] = a; }
          }
        }
        team_sync<NW>(bid);
      }
    }
    // (6) deal: sorted rank r < nl -> left half position r, nl <= r < ng -> right half position half + r - nl;
    // the free positions are empty and point at the last sorted slot (dyntree.py:66-71)
    const int nl = (ng + 1) / 2, nr = ng - nl, half = S >> 1;
    const int32_t last = perm[(int)(skey[S - 1] & 0xffffffffu)];
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

// The group of one (lane, level) in global memory: slot rows of the lane's key array, in / out permutations.
struct GroupRef {
  const float* keys;
  const int32_t* perm;
  const uint8_t* valid;
  int32_t* po;
  uint8_t* vo;
  int S;
};

__device__ __forceinline__ GroupRef group_ref(const LaneSplitParams& p, int64_t group) {
  const int G = 1 << p.lvl;
  const int S = p.C >> p.lvl;
  const int64_t lanep = group / G;
  const int64_t base = lanep * p.C + (group % G) * (int64_t)S;
  return GroupRef{p.keys + (lanep / p.key_lane_div) * p.key_stride, p.perm_in + base, p.valid_in + base,
                  p.perm_out + base, p.valid_out + base, S};
}

// Groups of more than SUBTREE_SLOTS slots: one group per CTA of 8 warps, rows read from global memory (L2).
template <int DH>
__global__ void __launch_bounds__(256) lane_split_cta_kernel(LaneSplitParams p) {
  extern __shared__ __align__(16) unsigned char split_smem[];
  const GroupRef g = group_ref(p, blockIdx.x);
  TwoMeans<8, DH>::run(g.keys, g.perm, g.valid, g.S, p.iters, g.po, g.vo, split_smem, threadIdx.x, 0);
}

// The remaining levels of a subtree of at most SUBTREE_SLOTS slots, in one CTA: its key rows are staged in shared
// memory once, then every level's groups are split there (a level of n groups: min(n, 8) teams of 8 / min(n, 8)
// warps, each team on its own named barrier), and the final slot order is written back.
#ifndef TA_SUBTREE_SLOTS
#define TA_SUBTREE_SLOTS 128
#endif
constexpr int SUBTREE_SLOTS = TA_SUBTREE_SLOTS;

template <int DH>
struct Subtree {
  static __host__ __device__ constexpr size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }
  // per-team scratch at group size s with NW warps per team, for 8 / NW teams
  static __host__ __device__ size_t scratch(int S0) {
    size_t m = 0;
    for (int s = S0; s >= 4; s >>= 1) {
      const int groups = S0 / s, teams = groups < 8 ? groups : 8, nw = 8 / teams;
      const size_t per = align16((size_t)s * 8 + 4 * DH * 4 + (size_t)2 * nw * DH * 4 + nw * 32);
      m = per * teams > m ? per * teams : m;
    }
    return m;
  }
  static __host__ __device__ size_t bytes(int S0) {
    return align16((size_t)S0 * DH * 4) + 2 * align16((size_t)S0 * 4) + 2 * align16((size_t)S0) + scratch(S0);
  }
};

template <int NW, int DH>
__device__ __forceinline__ void subtree_level(const float* stage, const int32_t* lp, const uint8_t* lv, int32_t* lpo,
                                              uint8_t* lvo, int S0, int s, int iters, unsigned char* scratch) {
  constexpr int TEAMS = 8 / NW;
  const int team = threadIdx.x / (NW * 32), tid = threadIdx.x % (NW * 32);
  const size_t per = Subtree<DH>::align16((size_t)s * 8 + 4 * DH * 4 + (size_t)2 * NW * DH * 4 + NW * 32);
  const int bid = NW == 8 ? 0 : 1 + team;
  for (int g = team; g < S0 / s; g += TEAMS) {
    const int o = g * s;
    TwoMeans<NW, DH, true>::run(stage, lp + o, lv + o, s, iters, lpo + o, lvo + o, scratch + per * team, tid, bid);
    team_sync<NW>(bid);
  }
}

// Three CTAs per SM: the register cap that keeps the 2-means passes at 80 registers (uncapped they take 128 and
// only two CTAs fit, which costs more than it gains in this latency-bound kernel).
#ifndef TA_SUBTREE_MINB
#define TA_SUBTREE_MINB 3
#endif
template <int DH>
__global__ void __launch_bounds__(256, TA_SUBTREE_MINB) lane_subtree_kernel(LaneSplitParams p, int levels) {
  extern __shared__ __align__(16) unsigned char split_smem[];
  const int S0 = p.C >> p.lvl;
  const GroupRef g = group_ref(p, blockIdx.x);
  float* stage = reinterpret_cast<float*>(split_smem);
  unsigned char* q = split_smem + Subtree<DH>::align16((size_t)S0 * DH * 4);
  int32_t* lpa = reinterpret_cast<int32_t*>(q);
  int32_t* lpb = reinterpret_cast<int32_t*>(q + Subtree<DH>::align16((size_t)S0 * 4));
  uint8_t* lva = q + 2 * Subtree<DH>::align16((size_t)S0 * 4);
  uint8_t* lvb = lva + Subtree<DH>::align16((size_t)S0);
  unsigned char* scratch = lvb + Subtree<DH>::align16((size_t)S0);
  // stage the valid rows (row i of the stage = slot i of the subtree; chunks placed by stage_chunk)
  for (int e = threadIdx.x; e < S0 * (DH / 4); e += blockDim.x) {
    const int i = e / (DH / 4), c = e - i * (DH / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g.valid[i]) v = *reinterpret_cast<const float4*>(g.keys + (int64_t)g.perm[i] * DH + c * 4);
    *reinterpret_cast<float4*>(stage + (size_t)i * DH + stage_chunk<DH>(c) * 4) = v;
  }
  for (int i = threadIdx.x; i < S0; i += blockDim.x) {
    lpa[i] = i;
    lva[i] = g.valid[i];
  }
  __syncthreads();
  int s = S0;
  for (int l = 0; l < levels; ++l, s >>= 1) {
    const int groups = S0 / s;
    if (groups == 1) subtree_level<8, DH>(stage, lpa, lva, lpb, lvb, S0, s, p.iters, scratch);
    else if (groups == 2) subtree_level<4, DH>(stage, lpa, lva, lpb, lvb, S0, s, p.iters, scratch);
    else if (groups == 4) subtree_level<2, DH>(stage, lpa, lva, lpb, lvb, S0, s, p.iters, scratch);
    else subtree_level<1, DH>(stage, lpa, lva, lpb, lvb, S0, s, p.iters, scratch);
    __syncthreads();
    int32_t* tp = lpa; lpa = lpb; lpb = tp;
    uint8_t* tv = lva; lva = lvb; lvb = tv;
  }
  // slot i of the subtree now holds stage row lpa[i] = subtree slot lpa[i] of the input order
  for (int i = threadIdx.x; i < S0; i += blockDim.x) {
    g.po[i] = g.perm[lpa[i]];
    g.vo[i] = lva[i];
  }
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
__device__ __forceinline__ void lane_insert_warp(const LaneTreeRef<DH>& tr, int32_t* slot, const float* kv, int D,
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
    if (d < DH) tr.row(0)[d] += k[j];
  }
  if (lane == 0) *tr.cntp(0) += 1;
  __syncwarp();
  int node = 0;
  for (int lvl = 0; lvl < D; ++lvl) {
    const int o = (2 << lvl) - 1;
    const int left = 2 * node, right = left + 1;
    const int cap = C >> (lvl + 1);
    const int cL = tr.cnt(o + left), cR = tr.cnt(o + right);
    const float* SL = tr.row(o + left);
    const float* SR = tr.row(o + right);
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
    float* dst = tr.row(o + node);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < DH) dst[d] += k[j];
    }
    if (lane == 0) *tr.cntp(o + node) += 1;
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
  const LaneTreeRef<DH> tr{p.sums + pl * (int64_t)NN * DH, p.cnt + pl * (int64_t)NN, nullptr, nullptr, 0};
  lane_insert_warp<DH>(tr, p.slot + pl * (int64_t)p.C, kb[warp], p.D, p.C, (int32_t)p.kpos[pl], lane);
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

// Rows of a lane's tree that the select loop keeps in shared memory: the upper levels, about 16 KB per warp (every
// token's descent and insertion passes through them, and the insertion rewrites one node per level).
template <int DH>
__host__ __device__ constexpr int lane_cache_rows() {
  return DH <= 16 ? 255 : DH <= 32 ? 127 : DH <= 64 ? 63 : 31;
}
template <int DH>
__host__ __device__ constexpr size_t lane_select_smem_bytes() {
  return (size_t)4 * lane_cache_rows<DH>() * (DH * sizeof(float) + sizeof(int32_t));
}

template <int DH>
__global__ void __launch_bounds__(128) lane_select_kernel(LaneSelectParams p) {
  extern __shared__ __align__(16) unsigned char lane_cache_smem[];
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
  // the upper levels of this lane's tree move to shared memory for the loop and back to global memory after it
  constexpr int NSR = lane_cache_rows<DH>();
  const int ns = NN < NSR ? NN : NSR;
  float* s_sums = reinterpret_cast<float*>(lane_cache_smem) + warp * NSR * DH;
  int32_t* s_cnt = reinterpret_cast<int32_t*>(lane_cache_smem + (size_t)4 * NSR * DH * sizeof(float)) + warp * NSR;
  for (int e = lane; e < ns * (DH / 4); e += 32)
    reinterpret_cast<float4*>(s_sums)[e] = reinterpret_cast<const float4*>(sums)[e];
  for (int r = lane; r < ns; r += 32) s_cnt[r] = cnt[r];
  const LaneTreeRef<DH> tr{sums, cnt, s_sums, s_cnt, ns};
  __syncwarp();
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
      const int cn = tr.cnt(offD + id);
      const float* nrow = tr.row(offD + id);
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
    const int nk = lane_descend_t<DH, false>(tr, p.D, p.wmax, sc, lane);  // the tree changes as the loop runs
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
    if (t >= 1) lane_insert_warp<DH>(tr, slot, kb[warp], p.D, C, t, lane);
    __syncwarp();
  }
  for (int e = lane; e < ns * (DH / 4); e += 32)
    reinterpret_cast<float4*>(sums)[e] = reinterpret_cast<const float4*>(s_sums)[e];
  for (int r = lane; r < ns; r += 32) cnt[r] = s_cnt[r];
}

}  // namespace ta
