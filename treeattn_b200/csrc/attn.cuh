// Exact softmax attention over selected keys, gather-dot and duplicate removal.
//
// Reference: fastseg.py:134-141 sparse_attn_ref / fastseg.py:49-78 _attn_fwd (online softmax over the kept
// keys, scale 1/sqrt(dh), fp32 accumulation, -1 = unused slot); fastseg.py:118-130 gather_dot;
// fastseg.py:227-234 dedupe_fast and attention_dyn.py:12-17 dedupe (keep the first valid copy).
//
// Lane layout shared by all warp-per-query kernels here: one key row of DH elements is read as DH/VEC
// 16-byte chunks by LPR = DH/VEC consecutive lanes, so a warp covers RPW = 32/LPR rows per pass with fully
// coalesced 128-bit loads. Row scores are reduced across the LPR lanes with shuffles.
#pragma once
#include "select.cuh"

namespace ta {

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

template <typename T, int DH>
struct WarpAttn {
  static constexpr int VEC = TypeInfo<T>::VEC;
  static constexpr int LPR = DH / VEC;
  static constexpr int RPW = 32 / LPR;
  static_assert(LPR >= 1 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "unsupported head dim");

  float q[VEC];    // this lane's query chunk, pre-multiplied by scale*log2(e)
  float acc[VEC];  // running sum of p * v for this lane's rows and dims
  float m;         // running max of the (log2-domain) scores, warp-uniform
  float l;         // running sum of p over this lane's rows
  int sub, c;

  __device__ __forceinline__ void init(const T* __restrict__ qrow, float scale_log2, int lane) {
    sub = lane / LPR;
    c = lane - sub * LPR;
    float tmp[VEC];
    load_vec_f32<T>(qrow + c * VEC, tmp);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      q[i] = tmp[i] * scale_log2;
      acc[i] = 0.f;
    }
    m = -INFINITY;
    l = 0.f;
  }

  // Score one K chunk (already widened) -> full-row score on every lane of the row group.
  __device__ __forceinline__ float row_score(const float (&kf)[VEC]) const {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) s = fmaf(q[i], kf[i], s);
    return warp_sum_sub(s, LPR);
  }

  // Online-softmax update with U row groups at once (scores s[u], values vf[u]; invalid rows have s = -inf).
  template <int U>
  __device__ __forceinline__ void update(const float (&s)[U], const float (&vf)[U][VEC]) {
    float mx = s[0];
#pragma unroll
    for (int u = 1; u < U; ++u) mx = fmaxf(mx, s[u]);
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m, mx);
    if (m_new == -INFINITY) return;  // nothing valid yet (warp-uniform)
    const float alpha = exp2f(m - m_new);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] *= alpha;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = (s[u] == -INFINITY) ? 0.f : exp2f(s[u] - m_new);
      l += p;
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = fmaf(p, vf[u][i], acc[i]);
    }
    m = m_new;
  }

  // Process U row groups read from global memory (row pointers for this lane; null = invalid row).
  template <int U>
  __device__ __forceinline__ void rows_global(const T* const (&kr)[U], const T* const (&vr)[U]) {
    float kf[U][VEC], vf[U][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (kr[u]) {
        ldg_vec_f32<T>(kr[u] + c * VEC, kf[u]);
        ldg_vec_f32<T>(vr[u] + c * VEC, vf[u]);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) kf[u][i] = vf[u][i] = 0.f;
      }
    }
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float x = row_score(kf[u]);
      s[u] = kr[u] ? x : -INFINITY;
    }
    update<U>(s, vf);
  }

  // Sum l and acc over the row groups; afterwards every lane holds the warp totals for its dim chunk c.
  __device__ __forceinline__ void reduce_rows() {
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
  }

  // This warp's share (row groups warp, warp + nw, ...) of n staged rows (row stride DH).
  __device__ __forceinline__ void stage(const T* kst, const T* vst, int n, int warp, int nw) {
    const int ngroups = ceil_div(n, RPW);
    for (int g0 = warp; g0 < ngroups; g0 += 2 * nw) {
      float kf[2][VEC], vf[2][VEC], sc[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int g = g0 + u * nw;
        const int r = g * RPW + sub;
        const bool valid = (g < ngroups) && (r < n);
        if (valid) {
          load_vec_f32<T>(kst + (size_t)r * DH + c * VEC, kf[u]);
          load_vec_f32<T>(vst + (size_t)r * DH + c * VEC, vf[u]);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) kf[u][i] = vf[u][i] = 0.f;
        }
        const float x = row_score(kf[u]);
        sc[u] = valid ? x : -INFINITY;
      }
      update<2>(sc, vf);
    }
  }

  // One row (k, v: DH elements each, any 16-byte aligned memory).
  __device__ __forceinline__ void one_row(const T* k, const T* v) {
    float kf[1][VEC], vf[1][VEC], sc[1];
    load_vec_f32<T>(k + c * VEC, kf[0]);
    load_vec_f32<T>(v + c * VEC, vf[0]);
    const float x = row_score(kf[0]);
    sc[0] = sub == 0 ? x : -INFINITY;
    update<1>(sc, vf);
  }
};

// ------------------------------------------------------------------------------------------------ packed math
// bf16 / fp16 rows without widening: fma.rn.f32.{bf16,f16} multiplies two 16-bit values exactly and adds in fp32
// with one rounding, i.e. the same result as widening both and using an fp32 FMA.
template <typename T> struct Mixed;
template <> struct Mixed<__nv_bfloat16> {
  // c += a.lo*b.lo ; c += a.hi*b.hi   (a, b: packed pairs)
  static __device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float c) {
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %0;\n\tfma.rn.f32.bf16 %0, ah, bh, %0;\n\t}"
        : "+f"(c) : "r"(a), "r"(b));
    return c;
  }
  // (c0, c1) += p * (v.lo, v.hi)   (p: one 16-bit value in the low half of pp)
  static __device__ __forceinline__ void axpy2(uint32_t pp, uint32_t v, float& c0, float& c1) {
    asm("{\n\t.reg .b16 pl, ph, vl, vh;\n\tmov.b32 {pl, ph}, %2;\n\tmov.b32 {vl, vh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, pl, vl, %0;\n\tfma.rn.f32.bf16 %1, pl, vh, %1;\n\t}"
        : "+f"(c0), "+f"(c1) : "r"(pp), "r"(v));
  }
  static __device__ __forceinline__ uint32_t pack(float p) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p));
  }
  static __device__ __forceinline__ float unpack(uint32_t pp) {
    return __bfloat162float(__ushort_as_bfloat16((unsigned short)(pp & 0xffffu)));
  }
};
template <> struct Mixed<__half> {
  static __device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float c) {
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\tfma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
        : "+f"(c) : "r"(a), "r"(b));
    return c;
  }
  static __device__ __forceinline__ void axpy2(uint32_t pp, uint32_t v, float& c0, float& c1) {
    asm("{\n\t.reg .b16 pl, ph, vl, vh;\n\tmov.b32 {pl, ph}, %2;\n\tmov.b32 {vl, vh}, %3;\n\t"
        "fma.rn.f32.f16 %0, pl, vl, %0;\n\tfma.rn.f32.f16 %1, pl, vh, %1;\n\t}"
        : "+f"(c0), "+f"(c1) : "r"(pp), "r"(v));
  }
  static __device__ __forceinline__ uint32_t pack(float p) {
    return (uint32_t)__half_as_ushort(__float2half_rn(p));
  }
  static __device__ __forceinline__ float unpack(uint32_t pp) {
    return __half2float(__ushort_as_half((unsigned short)(pp & 0xffffu)));
  }
};

// Online softmax over rows staged in shared memory, 16-bit K/V. Lane layout as WarpAttn (LPR lanes per row, 8
// elements = one 16-byte chunk per lane, RPW rows per warp pass). A call processes G row groups (G*RPW rows):
//  * QK: each lane dots its chunk for the G groups (mixed FMAs, no widening), then ONE reduce-scatter across the
//    LPR lanes of a row leaves lane c holding the full score of group c / (LPR/G) (log2(LPR) shuffle rounds,
//    G-1 + log2(LPR/G) shuffles in total instead of G*log2(LPR));
//  * one max / rescale per call; p = exp2(s - m) is rounded to the K/V type and used both in the numerator
//    (mixed FMA with V) and in the running sum l, so the weights stay a convex combination.
template <typename T, int DH>
struct PackedAttn {
  static constexpr int VEC = 8;
  static constexpr int LPR = DH / VEC;
  static constexpr int RPW = 32 / LPR;
  static constexpr int G = LPR >= 4 ? 4 : LPR;
  static constexpr int SPAN = LPR / G;  // lanes holding the same group after the reduce-scatter

  uint32_t q2[4];  // this lane's query chunk, packed pairs (unscaled)
  float acc[VEC];
  float m, l;
  float qscale;    // softmax scale * log2(e)
  int sub, c;

  __device__ __forceinline__ void init(const T* qrow, float scale_log2, int lane) {
    sub = lane / LPR;
    c = lane - sub * LPR;
    const uint4 v = *reinterpret_cast<const uint4*>(qrow + c * VEC);
    q2[0] = v.x; q2[1] = v.y; q2[2] = v.z; q2[3] = v.w;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
    m = -INFINITY;
    l = 0.f;
    qscale = scale_log2;
  }

  // Staged rows of the current call (registers), so the shared-memory stage can be released before the math.
  uint4 kk[G], vv[G];
  bool ok[G];

  // Load rows r = (g0 + g) * RPW + sub for g < G (valid when r < n); K rows at kst, V rows at vst (stride DH).
  __device__ __forceinline__ void load(const T* kst, const T* vst, int g0, int n) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int r = (g0 + g) * RPW + sub;
      ok[g] = r < n;
      kk[g] = vv[g] = make_uint4(0u, 0u, 0u, 0u);
      if (ok[g]) {
        kk[g] = *reinterpret_cast<const uint4*>(kst + (size_t)r * DH + c * VEC);
        vv[g] = *reinterpret_cast<const uint4*>(vst + (size_t)r * DH + c * VEC);
      }
    }
  }

  // Online-softmax update with the loaded rows.
  __device__ __forceinline__ void compute() {
    float part[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float a = Mixed<T>::dot2(q2[0], kk[g].x, 0.f);
      a = Mixed<T>::dot2(q2[1], kk[g].y, a);
      a = Mixed<T>::dot2(q2[2], kk[g].z, a);
      part[g] = Mixed<T>::dot2(q2[3], kk[g].w, a);
    }
    // reduce-scatter over the LPR lanes of a row: halve the value list while it has more than one entry
    int nv = G;
#pragma unroll
    for (int o = LPR / 2; o >= 1; o >>= 1) {
      if (nv > 1) {
        const int h = nv / 2;
        const bool up = (c & o) != 0;
#pragma unroll
        for (int j = 0; j < G / 2; ++j) {
          if (j < h) {
            const float keep = up ? part[j + h] : part[j];
            const float send = up ? part[j] : part[j + h];
            part[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        nv = h;
      } else {
        part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
      }
    }
    const int myg = c / SPAN;
    bool myok = false;
#pragma unroll
    for (int g = 0; g < G; ++g) myok |= (g == myg) && ok[g];
    const float s = myok ? part[0] * qscale : -INFINITY;
    float mx = s;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m, mx);
    if (m_new == -INFINITY) return;  // nothing valid yet (warp-uniform)
    const float alpha = exp2f(m - m_new);
    const uint32_t pp = myok ? Mixed<T>::pack(exp2f(s - m_new)) : 0u;
    l *= alpha;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] *= alpha;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint32_t pg = __shfl_sync(0xffffffffu, pp, sub * LPR + g * SPAN);
      if (ok[g]) {
        l += Mixed<T>::unpack(pg);
        Mixed<T>::axpy2(pg, vv[g].x, acc[0], acc[1]);
        Mixed<T>::axpy2(pg, vv[g].y, acc[2], acc[3]);
        Mixed<T>::axpy2(pg, vv[g].z, acc[4], acc[5]);
        Mixed<T>::axpy2(pg, vv[g].w, acc[6], acc[7]);
      }
    }
    m = m_new;
  }

  __device__ __forceinline__ void groups(const T* kst, const T* vst, int g0, int n) {
    load(kst, vst, g0, n);
    compute();
  }

  __device__ __forceinline__ void reduce_rows() {
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
  }

  __device__ __forceinline__ void stage(const T* kst, const T* vst, int n, int warp, int nw) {
    const int ngroups = ceil_div(n, RPW);
    for (int gb = warp * G; gb < ngroups; gb += nw * G) groups(kst, vst, gb, n);
  }

  __device__ __forceinline__ void one_row(const T* k, const T* v) { groups(k, v, 0, 1); }
};

// Attention math used on staged rows: widening fp32 math for fp32 caches, packed mixed-precision math for 16-bit.
template <typename T, int DH> struct StageAttn { using type = WarpAttn<T, DH>; };
template <typename WA> struct EarlyRelease { static constexpr bool value = false; };
template <typename T, int DH> struct EarlyRelease<PackedAttn<T, DH>> { static constexpr bool value = true; };
// Rows one register-staged call of a warp covers (PackedAttn only).
template <typename WA> struct RowsPerCall { static constexpr int value = 0; };
template <typename T, int DH> struct RowsPerCall<PackedAttn<T, DH>> {
  static constexpr int value = PackedAttn<T, DH>::G * PackedAttn<T, DH>::RPW;
};
template <int DH> struct StageAttn<__nv_bfloat16, DH> { using type = PackedAttn<__nv_bfloat16, DH>; };
template <int DH> struct StageAttn<__half, DH> { using type = PackedAttn<__half, DH>; };

// Merge partial softmax state b into a (both in the log2 domain).
__device__ __forceinline__ void merge_state(float& ma, float& la, float* acca, float mb, float lb, const float* accb,
                                            int n) {
  const float m = fmaxf(ma, mb);
  if (m == -INFINITY) return;
  const float fa = exp2f(ma - m), fb = exp2f(mb - m);
  la = la * fa + lb * fb;
  for (int i = 0; i < n; ++i) acca[i] = acca[i] * fa + accb[i] * fb;
  ma = m;
}

// ------------------------------------------------------------------------------------------------ key ranges
// The key set of one query of the segment-tree path, as disjoint position ranges (no duplicate positions):
// every used leaf block [m*leaf, (m+1)*leaf) cut at the window start w0, the sink {0} unless a used leaf or the
// window already holds it, and the local window [w0, t] (fastseg.py:372-381 static keys + dedupe_fast).
constexpr int MAX_RANGES = WMAX_LIMIT + 2;

struct RangeList {
  int start[MAX_RANGES];
  int pref[MAX_RANGES + 1];  // prefix sums of the lengths
  int n;
};

// Build the ranges of one query with a warp. `leaf_of(i)` returns the leaf id of slot i or -1 when the slot is
// not used (ids whose block does not end before the window start are ignored). `t_end` = one past the last window position (t+1 when position t is read from the cache, t when
// the caller handles position t itself). Returns the total number of keys in the ranges.
template <typename LeafFn>
__device__ __forceinline__ int build_ranges(RangeList& rl, int nslots, LeafFn leaf_of, int leaf, int t, int Lw,
                                            int t_end, int lane) {
  const int w0 = max(t - Lw + 1, 0);
  int cnt = 0;
  bool leaf0 = false;
  for (int base = 0; base < nslots; base += 32) {
    const int i = base + lane;
    int st = 0, len = 0;
    if (i < nslots) {
      const int64_t m = leaf_of(i);
      // a used leaf lies entirely before the window start; anything else (a bad id) contributes nothing
      if (m >= 0 && m * (int64_t)leaf < (int64_t)w0) {
        st = (int)(m * leaf);
        const int en = min(st + leaf, w0);
        len = max(en - st, 0);
        if (m == 0) leaf0 = true;
      }
    }
    const unsigned mask = __ballot_sync(0xffffffffu, len > 0);
    if (len > 0) {
      const int idx = cnt + __popc(mask & ((1u << lane) - 1u));
      rl.start[idx] = st;
      rl.pref[idx + 1] = len;  // lengths for now
    }
    cnt += __popc(mask);
  }
  leaf0 = __any_sync(0xffffffffu, leaf0);
  __syncwarp();
  if (lane == 0) {
    if (w0 > 0 && !leaf0) {
      rl.start[cnt] = 0;
      rl.pref[cnt + 1] = 1;
      ++cnt;
    }
    if (t_end > w0) {
      rl.start[cnt] = w0;
      rl.pref[cnt + 1] = t_end - w0;
      ++cnt;
    }
    rl.pref[0] = 0;
    for (int r = 0; r < cnt; ++r) rl.pref[r + 1] += rl.pref[r];
    rl.n = cnt;
  }
  __syncwarp();
  return rl.pref[rl.n];
}

// ------------------------------------------------------------------------------------------------ seg attention
// One warp per query: key set from the selected leaves (best first, the first n_tree valid ones are used),
// the sink and the local window; exact online-softmax attention over it, K/V read straight from HBM/L2.
struct SegAttnParams {
  const void *q, *k, *v;
  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  const int64_t* tq;
  int64_t tq_sb, tq_st;
  const int64_t* ids;     // (B,H,Nq,wl)
  const uint8_t* vld;     // (B,H,Nq,wl)
  const int64_t* n_tree;  // (B,H,Nq) or null -> ntree_const
  int ntree_const;
  int B, H, Nq, wl, leaf, Lw, T_kv;
  float scale;
  void* o;                // (B,H,Nq,dh) with strides
  int64_t o_sb, o_sh, o_st;
  float* lse;             // (B,H,Nq) natural-log LSE, may be null
  int32_t* nkeys;         // (B,H,Nq) keys attended, may be null
};

template <typename T, int DH>
__global__ void __launch_bounds__(128) seg_attn_kernel(SegAttnParams p) {
  __shared__ RangeList s_rl[4];
  using WA = WarpAttn<T, DH>;
  constexpr int U = (WA::RPW >= 8) ? 2 : 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.B * p.H * p.Nq) return;
  const int n = (int)(qid % p.Nq);
  const int bh = (int)(qid / p.Nq);
  const int b = bh / p.H, h = bh % p.H;
  const int64_t tt = p.tq[b * p.tq_sb + n * p.tq_st];
  RangeList& rl = s_rl[warp];
  if (tt < 0 || tt >= p.T_kv) {
    if (lane == 0) record_error(DEV_POS_RANGE, K_SEG_ATTN, (int)tt, p.T_kv);
    return;
  }
  const int t = (int)tt;
  const int ntree = p.n_tree ? (int)p.n_tree[qid] : p.ntree_const;
  const int64_t sbase = qid * p.wl;
  const int total = build_ranges(
      rl, p.wl,
      [&](int i) -> int64_t {
        return (p.vld[sbase + i] && i < ntree) ? p.ids[sbase + i] : (int64_t)-1;
      },
      p.leaf, t, p.Lw, t + 1, lane);

  const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + n * p.q_st;
  const T* kb = reinterpret_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
  const T* vb = reinterpret_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
  WA wa;
  wa.init(qrow, p.scale * LOG2E, lane);
  int ri = 0;  // this lane's current range
  for (int base = 0; base < total; base += WA::RPW * U) {
    const T* kr[U];
    const T* vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * WA::RPW + wa.sub;
      kr[u] = vr[u] = nullptr;
      if (g < total) {
        while (g >= rl.pref[ri + 1]) ++ri;
        const int pos = rl.start[ri] + (g - rl.pref[ri]);
        kr[u] = kb + pos * p.k_st;
        vr[u] = vb + pos * p.v_st;
      }
    }
    wa.template rows_global<U>(kr, vr);
  }
  wa.reduce_rows();
  const float inv = wa.l > 0.f ? 1.f / wa.l : 0.f;
  if (wa.sub == 0) {
    float outv[WA::VEC];
#pragma unroll
    for (int i = 0; i < WA::VEC; ++i) outv[i] = wa.acc[i] * inv;
    T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + n * p.o_st;
    store_vec_from_f32<T>(orow + wa.c * WA::VEC, outv);
  }
  if (lane == 0) {
    if (p.lse) p.lse[qid] = wa.l > 0.f ? (wa.m + log2f(wa.l)) * LN2 : -INFINITY;
    if (p.nkeys) p.nkeys[qid] = total;
  }
}

// ------------------------------------------------------------------------------------------------ sparse_attn
// fastseg.py:173 sparse_attn forward: candidate positions per query (int32 or int64), -1 = unused.
struct SparseAttnParams {
  const void *q, *k, *v;
  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  const void* cand;       // (B,H,T,Kc) contiguous
  int cand64;             // 1: int64, 0: int32
  int B, H, T, Kc, T_kv;
  float scale;
  void* o;
  int64_t o_sb, o_sh, o_st;
  float* lse;
};

template <typename T, int DH>
__global__ void __launch_bounds__(128) sparse_attn_kernel(SparseAttnParams p) {
  using WA = WarpAttn<T, DH>;
  constexpr int U = (WA::RPW >= 8) ? 2 : 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.B * p.H * p.T) return;
  const int n = (int)(qid % p.T);
  const int bh = (int)(qid / p.T);
  const int b = bh / p.H, h = bh % p.H;
  const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + n * p.q_st;
  const T* kb = reinterpret_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
  const T* vb = reinterpret_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
  const int64_t cbase = qid * p.Kc;
  WA wa;
  wa.init(qrow, p.scale * LOG2E, lane);
  for (int base = 0; base < p.Kc; base += WA::RPW * U) {
    const T* kr[U];
    const T* vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * WA::RPW + wa.sub;
      kr[u] = vr[u] = nullptr;
      if (g < p.Kc) {
        const int64_t pos = p.cand64 ? reinterpret_cast<const int64_t*>(p.cand)[cbase + g]
                                     : (int64_t)reinterpret_cast<const int32_t*>(p.cand)[cbase + g];
        if (pos >= 0 && pos < p.T_kv) {
          kr[u] = kb + pos * p.k_st;
          vr[u] = vb + pos * p.v_st;
        } else if (pos >= p.T_kv) {
          record_error(DEV_INDEX_RANGE, K_SPARSE_ATTN, (int)pos, p.T_kv);
        }
      }
    }
    wa.template rows_global<U>(kr, vr);
  }
  wa.reduce_rows();
  const float inv = wa.l > 0.f ? 1.f / wa.l : 0.f;
  if (wa.sub == 0) {
    float outv[WA::VEC];
#pragma unroll
    for (int i = 0; i < WA::VEC; ++i) outv[i] = wa.acc[i] * inv;
    T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + n * p.o_st;
    store_vec_from_f32<T>(orow + wa.c * WA::VEC, outv);
  }
  if (lane == 0 && p.lse) p.lse[qid] = wa.l > 0.f ? (wa.m + log2f(wa.l)) * LN2 : -INFINITY;
}

// ------------------------------------------------------------------------------------------------ sparse_attn bwd
// fastseg.py:80-110 _attn_bwd / 158-170 _SparseAttnFn.backward: with p = exp(scale q.k - lse) over the query's
// candidate keys (-1 unused), di = o . do, dp = do . v and ds = p (dp - di):
//   dq = sum_keys ds scale k          (fp32, stored in q's dtype)
//   dk[key] += ds scale q, dv[key] += p do   (fp32 accumulators shared by all queries: vector atomics, as the
//                                             reference accumulates them; the caller zeroes them)
// One warp per query, LPR lanes per key row (16-byte chunks), RPW keys per warp step; dot products reduced within
// the row's lanes, dq across the rows at the end. All tensors dense: q, o, do, dq (B, H, T, dh); k, v, dk, dv
// (B, H, T_kv, dh).
struct SparseAttnBwdParams {
  const void *q, *k, *v, *o, *dout;
  const float* lse;       // (B,H,T) natural log
  const void* cand;       // (B,H,T,Kc) contiguous, int32 or int64
  int cand64;
  int B, H, T, Kc, T_kv;
  float scale;
  void* dq;
  float* dk;
  float* dv;
};

__device__ __forceinline__ void atomic_add_vec(float* dst, const float* v, int n) {
  // n = 4 or 8, dst 16-byte aligned (sm_90+: one vector atomic per 16 bytes)
  for (int i = 0; i < n; i += 4) atomicAdd(reinterpret_cast<float4*>(dst + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
}

template <typename T, int DH>
__global__ void __launch_bounds__(128) sparse_attn_bwd_kernel(SparseAttnBwdParams p) {
  constexpr int VEC = TypeInfo<T>::VEC;
  constexpr int LPR = DH / VEC;  // lanes per key row
  constexpr int RPW = 32 / LPR;  // key rows per warp step
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.B * p.H * p.T) return;
  const int64_t bh = qid / p.T;
  const int c = lane % LPR, sub = lane / LPR;
  const int64_t row = qid * DH + c * VEC;
  float q[VEC], dov[VEC], ov[VEC], dq[VEC];
  load_vec_f32<T>(reinterpret_cast<const T*>(p.q) + row, q);
  load_vec_f32<T>(reinterpret_cast<const T*>(p.dout) + row, dov);
  load_vec_f32<T>(reinterpret_cast<const T*>(p.o) + row, ov);
  float di = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    di = fmaf(ov[i], dov[i], di);
    dq[i] = 0.f;
  }
  di = warp_sum_sub(di, LPR);
  const float lse = p.lse[qid];
  const T* kb = reinterpret_cast<const T*>(p.k) + bh * (int64_t)p.T_kv * DH + c * VEC;
  const T* vb = reinterpret_cast<const T*>(p.v) + bh * (int64_t)p.T_kv * DH + c * VEC;
  float* dkb = p.dk + bh * (int64_t)p.T_kv * DH + c * VEC;
  float* dvb = p.dv + bh * (int64_t)p.T_kv * DH + c * VEC;
  const int64_t cbase = qid * p.Kc;
  for (int base = 0; base < p.Kc; base += RPW) {
    const int g = base + sub;
    int64_t pos = -1;
    if (g < p.Kc) {
      pos = p.cand64 ? reinterpret_cast<const int64_t*>(p.cand)[cbase + g]
                     : (int64_t)reinterpret_cast<const int32_t*>(p.cand)[cbase + g];
      if (pos >= p.T_kv) {
        if (c == 0) record_error(DEV_INDEX_RANGE, K_SPARSE_ATTN, (int)pos, p.T_kv);
        pos = -1;
      }
    }
    const bool valid = pos >= 0;
    float kv[VEC], vv[VEC];
    if (valid) {
      load_vec_f32<T>(kb + pos * DH, kv);
      load_vec_f32<T>(vb + pos * DH, vv);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) kv[i] = vv[i] = 0.f;
    }
    float sdot = 0.f, pdot = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      sdot = fmaf(q[i], kv[i], sdot);
      pdot = fmaf(dov[i], vv[i], pdot);
    }
    sdot = warp_sum_sub(sdot, LPR);
    pdot = warp_sum_sub(pdot, LPR);
    const float pr = valid ? expf(sdot * p.scale - lse) : 0.f;
    const float ds = pr * (pdot - di);
    const float dss = ds * p.scale;
    if (valid) {
      float gk[VEC], gv[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        dq[i] = fmaf(dss, kv[i], dq[i]);
        gk[i] = dss * q[i];
        gv[i] = pr * dov[i];
      }
      atomic_add_vec(dkb + pos * DH, gk, VEC);
      atomic_add_vec(dvb + pos * DH, gv, VEC);
    }
  }
  // dq: sum over the RPW row slots (lanes with the same chunk c)
#pragma unroll
  for (int i = 0; i < VEC; ++i)
    for (int o = LPR; o < 32; o <<= 1) dq[i] += __shfl_xor_sync(0xffffffffu, dq[i], o);
  if (sub == 0) store_vec_from_f32<T>(reinterpret_cast<T*>(p.dq) + row, dq);
}

// ------------------------------------------------------------------------------------------------ gather_dot
// fastseg.py:118-130: out[b,h,n,c] = scale * q[b,h,n] . S[b,h,cand[b,h,n,c]] in fp32; ids clamped to [0, M-1]
// as the reference does. One warp per query row.
struct GatherDotParams {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const void* S;
  int64_t s_sb, s_sh, s_st;
  const void* cand;  // (B,H,N,C) contiguous, int32 or int64
  int cand64;
  int B, H, N, C, M;
  float scale;
  float* out;        // (B,H,N,C)
};

template <typename T, int DH>
__global__ void __launch_bounds__(128) gather_dot_kernel(GatherDotParams p) {
  using WA = WarpAttn<T, DH>;
  constexpr int VEC = WA::VEC, LPR = WA::LPR, RPW = WA::RPW;
  constexpr int U = (RPW >= 8) ? 2 : 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qid = (int64_t)blockIdx.x * 4 + warp;
  if (qid >= (int64_t)p.B * p.H * p.N) return;
  const int n = (int)(qid % p.N);
  const int bh = (int)(qid / p.N);
  const int b = bh / p.H, h = bh % p.H;
  const int sub = lane / LPR, c = lane % LPR;
  float qv[VEC];
  load_vec_f32<T>(reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + n * p.q_st + c * VEC, qv);
  const T* sb = reinterpret_cast<const T*>(p.S) + b * p.s_sb + h * p.s_sh;
  const int64_t cbase = qid * p.C;
  for (int base = 0; base < p.C; base += RPW * U) {
    float kf[U][VEC];
    int gi[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * RPW + sub;
      gi[u] = g;
      if (g < p.C) {
        int64_t id = p.cand64 ? reinterpret_cast<const int64_t*>(p.cand)[cbase + g]
                              : (int64_t)reinterpret_cast<const int32_t*>(p.cand)[cbase + g];
        id = id < 0 ? 0 : (id >= p.M ? p.M - 1 : id);
        ldg_vec_f32<T>(sb + id * p.s_st + c * VEC, kf[u]);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) kf[u][i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) s = fmaf(qv[i], kf[u][i], s);
      s = warp_sum_sub(s, LPR);
      if (c == 0 && gi[u] < p.C) p.out[cbase + gi[u]] = s * p.scale;
    }
  }
}

// Block form (selected key blocks of `blk` contiguous rows): each CTA stages NB_CTA blocks of one (b, h) into
// shared memory with 1-D bulk copies (one mbarrier), then 4 warps score the rows from shared memory.
struct GatherDotBlocksParams {
  const void* q;            // (B,H,dh) query rows (strides)
  int64_t q_sb, q_sh;
  const void* k;            // (B,H,T,dh) keys (strides; rows must be 16-byte aligned)
  int64_t k_sb, k_sh, k_st;
  const int32_t* blocks;    // (B,H,nblk) block ids
  int B, H, T, nblk, blk, nb_cta;
  float scale;
  float* out;               // (B,H,nblk*blk)
};

template <typename T, int DH>
__global__ void __launch_bounds__(128) gather_dot_blocks_kernel(GatherDotBlocksParams p) {
  using WA = WarpAttn<T, DH>;
  constexpr int VEC = WA::VEC, LPR = WA::LPR, RPW = WA::RPW;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar;
  T* rows = reinterpret_cast<T*>(smem_raw);
  const int groups = ceil_div(p.nblk, p.nb_cta);
  const int bh = blockIdx.x / groups, grp = blockIdx.x % groups;
  const int b = bh / p.H, h = bh % p.H;
  const int j0 = grp * p.nb_cta;
  const int nb = min(p.nb_cta, p.nblk - j0);
  const int row_bytes = DH * (int)sizeof(T);
  const int32_t* bl = p.blocks + (int64_t)bh * p.nblk + j0;
  const T* kbase = reinterpret_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
  // launched with programmatic stream serialization: wait (before the first global read) until the previous grid
  // of the stream has completed and its writes are visible; the next grid may be scheduled once every CTA of this
  // one has its rows in flight
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t pol = l2_policy_evict_first();
    uint32_t bytes = 0;
    int okb[64];
    for (int j = 0; j < nb; ++j) {
      const int id = bl[j];
      okb[j & 63] = (id >= 0 && (int64_t)(id + 1) * p.blk <= p.T);
      if (okb[j & 63]) bytes += (uint32_t)(p.blk * row_bytes);
      else record_error(DEV_INDEX_RANGE, K_GATHER_DOT_BLOCKS, id, p.T / p.blk);
    }
    mbar_arrive_expect_tx(&bar, bytes);
    for (int j = 0; j < nb; ++j) {
      if (!okb[j & 63]) continue;
      bulk_g2s_hint(rows + (size_t)j * p.blk * DH, kbase + (int64_t)bl[j] * p.blk * p.k_st,
                    (uint32_t)(p.blk * row_bytes), &bar, pol);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, c = lane % LPR;
  float qv[VEC];
  load_vec_f32<T>(reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + c * VEC, qv);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const bool ok = mbar_wait_bounded(&bar, 0, K_GATHER_DOT_BLOCKS, 0);
  if (!ok) return;  // the wait gave up; an error is recorded (copies may still land in this CTA's smem)
  const int nrows = nb * p.blk;
  float* outp = p.out + (int64_t)bh * p.nblk * p.blk + (int64_t)j0 * p.blk;
  for (int base = warp * RPW; base < nrows; base += 4 * RPW) {
    const int r = base + sub;
    float s = 0.f;
    if (r < nrows) {
      float kf[VEC];
      load_vec_f32<T>(rows + (size_t)r * DH + c * VEC, kf);
#pragma unroll
      for (int i = 0; i < VEC; ++i) s = fmaf(qv[i], kf[i], s);
    }
    s = warp_sum_sub(s, LPR);
    if (c == 0 && r < nrows) outp[r] = s * p.scale;
  }
}

// ------------------------------------------------------------------------------------------------ dedupe
// keep[r, j] = valid[r, j] and no earlier valid entry of row r holds the same value. One CTA per row.
__global__ void dedupe_kernel(const int64_t* __restrict__ cand, const uint8_t* __restrict__ valid, uint8_t* keep,
                              int64_t rows, int Kc) {
  extern __shared__ int64_t s_key[];
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  for (int j = threadIdx.x; j < Kc; j += blockDim.x) {
    const bool v = valid[r * Kc + j] != 0;
    s_key[j] = v ? cand[r * Kc + j] : INT64_MIN;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < Kc; j += blockDim.x) {
    const int64_t x = s_key[j];
    bool kp = x != INT64_MIN;
    for (int i = 0; i < j && kp; ++i) kp = (s_key[i] != x);
    keep[r * Kc + j] = kp ? 1 : 0;
  }
}

}  // namespace ta
