// Segment-tree node summaries ("index vectors") in HBM, and the kernels that build them.
//
// Layout. For every (batch b, head h) the stored levels L0..Lm are packed one after the other:
//   nodes[b*s_b + h*s_h + (off[l] + m) * DH + d]      (fp32)
// where level l holds cap >> l nodes (node m covers positions [m*2^l, (m+1)*2^l)) and
// off[L0] = 0, off[l+1] = off[l] + (cap >> l). A parent is the fp32 SUM of its two children, formed in the
// adjacent-pair order of the reference (seg.py:35 level_sums, engine.py:48-54 SegState.add), so node values
// are bit-identical to the reference's. The key at position 0 (the sink) enters the sums as 0
// (seg.py:128-130, engine.py:44, engine.py:62). Only levels >= L0 (the leaf-block level, 2^L0 tokens) are kept.
#pragma once
#include "common.cuh"

namespace ta {

constexpr int MAX_LEVELS = 32;

struct LevelView {
  const float* nodes;   // (b=0, h=0) base
  int64_t s_b, s_h;     // strides (in floats) between batch rows / heads
  int cap;              // capacity in positions
  int L0, Lm;           // stored levels
  int off[MAX_LEVELS];  // node offset of level l (valid for L0 <= l <= Lm)
};

// Host/device helper: level offsets for a given capacity. Returns total nodes per (b, h).
__host__ __device__ inline int64_t level_offsets(int cap, int L0, int Lm, int* off) {
  int64_t o = 0;
  for (int l = L0; l <= Lm; ++l) {
    off[l] = (int)o;
    o += (cap >> l);
  }
  return o;
}

// Binary-counter pairwise accumulator: feeding x_0, x_1, ..., x_{2^L-1} in order leaves the
// balanced adjacent-pair sum ((x0+x1)+(x2+x3))+... in stk[L] - the exact order of repeated
// reshape(..., 2, d).sum over levels 1..L.
struct PairwiseAcc {
  float stk[16];
  __device__ __forceinline__ void push(int i, float v) {
    int j = 0;
    while ((i >> j) & 1) {
      v = stk[j] + v;  // left sibling + right sibling
      ++j;
    }
    stk[j] = v;
  }
};

// The mean-log gate's statistic of one key value (seg.py:31): log(|x| + 1e-6) in fp32 (the sum rounded once, the
// logarithm evaluated in double and rounded once).
__device__ __forceinline__ float log_mag(float x) { return (float)log((double)__fadd_rn(fabsf(x), 1e-6f)); }

// Leaf level: one thread per (bh, leaf node m, dim d). Reads 2^L0 keys of dim d; with zero_sink the key at
// position 0 enters as 0. LOGMAG sums log_mag of the keys instead (the gate's log-magnitude tree).
template <typename T, bool LOGMAG = false>
__global__ void build_leaf_level_kernel(const T* __restrict__ k, int64_t k_sb, int64_t k_sh, int64_t k_st, int H,
                                        int T_len, int dh, int L0, float* __restrict__ nodes, int64_t n_sb,
                                        int64_t n_sh, int n_leaf_nodes, int64_t total_threads, int zero_sink) {
  int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= total_threads) return;
  const int d = (int)(gid % dh);
  int64_t r = gid / dh;
  const int m = (int)(r % n_leaf_nodes);
  r /= n_leaf_nodes;
  const int h = (int)(r % H);
  const int b = (int)(r / H);
  const int leaf = 1 << L0;
  const T* kp = k + b * k_sb + h * k_sh + d;
  PairwiseAcc acc;
  const int p0 = m * leaf;
  auto key_at = [&](int p) -> float {
    const float x = ((p != 0 || !zero_sink) && p < T_len) ? to_f32(kp[(int64_t)p * k_st]) : 0.f;
    return LOGMAG ? log_mag(x) : x;
  };
  if (leaf >= 8) {
    for (int i0 = 0; i0 < leaf; i0 += 8) {  // 8 independent loads in flight, then the ordered pairwise adds
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = key_at(p0 + i0 + j);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc.push(i0 + j, v[j]);
    }
  } else {
    for (int i = 0; i < leaf; ++i) acc.push(i, key_at(p0 + i));
  }
  nodes[b * n_sb + h * n_sh + (int64_t)m * dh + d] = acc.stk[L0];
}

// Upper levels of one (b, h) per CTA in shared memory: the complete leaf-level nodes are staged, then every level
// L0+1..Lm is formed in parallel over (node, dim) as parent = left + right (the same fp32 adds, in the same
// order, as the reference's repeated pairwise sums) and written out. Only nodes complete within the first T_len
// positions are formed (m < T_len >> l).
__global__ void __launch_bounds__(256) build_upper_levels_smem_kernel(float* __restrict__ nodes, int64_t n_sb,
                                                                      int64_t n_sh, int H, int dh, LevelView lv,
                                                                      int T_len) {
  extern __shared__ __align__(16) float lvl_smem[];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  float* base = nodes + b * n_sb + h * n_sh;
  const int n_leaf = T_len >> lv.L0;
  // stage the leaf level; level l (> L0) is then built in place at offset 0 of the buffer's second half
  float* cur = lvl_smem;
  float* nxt = lvl_smem + (size_t)n_leaf * dh;
  const float* src0 = base + (int64_t)lv.off[lv.L0] * dh;
  for (int x = threadIdx.x; x < n_leaf * dh / 4; x += blockDim.x)
    reinterpret_cast<float4*>(cur)[x] = reinterpret_cast<const float4*>(src0)[x];
  __syncthreads();
  for (int l = lv.L0 + 1; l <= lv.Lm; ++l) {
    const int n = T_len >> l;
    if (n == 0) break;
    float* dst = base + (int64_t)lv.off[l] * dh;
    for (int x = threadIdx.x; x < n * dh; x += blockDim.x) {
      const int m = x / dh, d = x - (x / dh) * dh;
      const float v = cur[(2 * m) * dh + d] + cur[(2 * m + 1) * dh + d];
      nxt[x] = v;
      dst[x] = v;
    }
    __syncthreads();
    float* tmp = cur; cur = nxt; nxt = tmp;
  }
}

// Upper levels: one thread per (bh, dim) walks levels L0+1..Lm, parent = left + right.
// Only nodes that are complete within the first T_len positions are formed (m < T_len >> l).
__global__ void build_upper_levels_kernel(float* __restrict__ nodes, int64_t n_sb, int64_t n_sh, int H, int dh,
                                          LevelView lv, int n_bh, int T_len) {
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= n_bh * dh) return;
  const int d = gid % dh;
  const int bh = gid / dh;
  const int b = bh / H, h = bh % H;
  float* base = nodes + b * n_sb + h * n_sh + d;
  for (int l = lv.L0 + 1; l <= lv.Lm; ++l) {
    const int n = T_len >> l;
    const float* src = base + (int64_t)lv.off[l - 1] * dh;
    float* dst = base + (int64_t)lv.off[l] * dh;
    for (int m = 0; m < n; ++m) dst[(int64_t)m * dh] = src[(int64_t)(2 * m) * dh] + src[(int64_t)(2 * m + 1) * dh];
  }
}

// ------------------------------------------------------------------------------------------------ mean-log gate
// seg.py:16-23 gate_apply on one node with a warp: ml = lg / size; thr = torch.quantile(ml, q) (ranks q (dh - 1)
// in fp32, the values at floor / ceil of the rank by a stable rank count, torch's fused two-sided lerp); kept =
// #{ml >= thr}; out = (raw * [ml >= thr]) * (dh / max(kept, 1)). NPL = ceil(dh / 32) values per lane; with
// dh = 16 the upper half-warp holds no element (ranked last, never counted).
// torch.quantile(ml, q) over the DH values of a warp (NPL per lane, element (i, lane) = index i * 32 + lane, absent
// elements +inf): ranks q (DH - 1) in fp32, the values at floor / ceil of the rank by a stable rank count, torch's
// fused two-sided lerp.
template <int DH>
__device__ __forceinline__ float warp_quantile(const float (&ml)[(DH + 31) / 32], float gate_q, int lane) {
  constexpr int NPL = (DH + 31) / 32;
  const float rank = __fmul_rn(gate_q, (float)(DH - 1));
  const int lo = (int)floorf(rank), hi = (int)ceilf(rank);
  const float w = __fsub_rn(rank, (float)lo);
  int rk[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) rk[i] = 0;
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    for (int src = 0; src < 32; ++src) {
      const float o = __shfl_sync(0xffffffffu, ml[j], src);
      const int oi = j * 32 + src;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int mi = i * 32 + lane;
        rk[i] += (o < ml[i] || (o == ml[i] && oi < mi)) ? 1 : 0;
      }
    }
  }
  float vlo = 0.f, vhi = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const unsigned blo = __ballot_sync(0xffffffffu, rk[i] == lo), bhi = __ballot_sync(0xffffffffu, rk[i] == hi);
    if (blo) vlo = __shfl_sync(0xffffffffu, ml[i], __ffs(blo) - 1);
    if (bhi) vhi = __shfl_sync(0xffffffffu, ml[i], __ffs(bhi) - 1);
  }
  const float d = __fsub_rn(vhi, vlo);
  return w < 0.5f ? fmaf(w, d, vlo) : fmaf(-__fsub_rn(1.f, w), d, vhi);
}

template <int DH>
__device__ __forceinline__ void gate_node_warp(const float* raw, const float* lg, float* out, float inv_size,
                                               float gate_q, int lane) {
  constexpr int NPL = (DH + 31) / 32;
  float r[NPL], ml[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const bool on = i * 32 + lane < DH;
    r[i] = on ? raw[i * 32 + lane] : 0.f;
    ml[i] = on ? lg[i * 32 + lane] * inv_size : INFINITY;  // size is a power of two: exact
  }
  const float thr = warp_quantile<DH>(ml, gate_q, lane);
  int kept = 0;
#pragma unroll
  for (int i = 0; i < NPL; ++i) kept += __popc(__ballot_sync(0xffffffffu, ml[i] >= thr && i * 32 + lane < DH));
  const float scale = __fdiv_rn((float)DH, (float)(kept > 1 ? kept : 1));
#pragma unroll
  for (int i = 0; i < NPL; ++i)
    if (i * 32 + lane < DH) out[i * 32 + lane] = __fmul_rn(ml[i] >= thr ? r[i] : 0.f, scale);
}

// Gated copy of the levels [L0, Lm]: one warp per complete node (m < T_len >> l); levels below gate_min are copied.
template <int DH>
__global__ void __launch_bounds__(128) gate_levels_kernel(const float* __restrict__ raw, const float* __restrict__ lg,
                                                         float* __restrict__ out, int64_t n_sb, int64_t n_sh, int H,
                                                         LevelView lv, int T_len, int n_bh, float gate_q,
                                                         int gate_min, int64_t nodes_per_bh) {
  constexpr int NPL = (DH + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (int64_t)n_bh * nodes_per_bh) return;
  const int bh = (int)(wid / nodes_per_bh);
  int m = (int)(wid % nodes_per_bh);
  int l = lv.L0;
  while (l < lv.Lm && m >= (lv.cap >> l)) {  // packed node index -> (level, node)
    m -= lv.cap >> l;
    ++l;
  }
  if (m >= (T_len >> l)) return;
  const int b = bh / H, h = bh % H;
  const int64_t row = b * n_sb + h * n_sh + (int64_t)(lv.off[l] + m) * DH;
  if (l >= gate_min) {
    gate_node_warp<DH>(raw + row, lg + row, out + row, __int_as_float((127 - l) << 23), gate_q, lane);
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (i * 32 + lane < DH) out[row + i * 32 + lane] = raw[row + i * 32 + lane];
  }
}

// Decoding: after position pos[b] was appended (and, when it completed a leaf block, its raw nodes formed), form
// the log-magnitude nodes of the same leaf block and right-spine ancestors and their gated copies. One warp per
// (b, h); the block's keys are read from the cache (position pos[b] included).
template <typename T, int DH>
__global__ void __launch_bounds__(128) gate_append_kernel(const T* __restrict__ kc, int64_t c_sb, int64_t c_sh,
                                                         int64_t c_st, const float* __restrict__ raw,
                                                         float* __restrict__ lg, float* __restrict__ out,
                                                         int64_t n_sb, int64_t n_sh, int B, int H, LevelView lv,
                                                         const int32_t* __restrict__ pos, float gate_q, int gate_min) {
  constexpr int NPL = (DH + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (int64_t)B * H) return;
  const int b = (int)(wid / H), h = (int)(wid % H);
  const int t = pos[b];
  const int leaf = 1 << lv.L0;
  if (t < 0 || t >= lv.cap || ((t + 1) & (leaf - 1)) != 0) return;
  const T* kb = kc + b * c_sb + h * c_sh;
  const int64_t base = b * n_sb + h * n_sh;
  const int n0 = t >> lv.L0;
  // leaf node: pairwise sums (adjacent-pair order) of log_mag over the block, one PairwiseAcc per dim
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int d = i * 32 + lane;
    if (d >= DH) continue;
    PairwiseAcc acc;
    for (int j = 0; j < leaf; ++j) {
      const int p = n0 * leaf + j;
      const float x = p == 0 ? 0.f : to_f32(kb[(int64_t)p * c_st + d]);
      acc.push(j, log_mag(x));
    }
    lg[base + (int64_t)(lv.off[lv.L0] + n0) * DH + d] = acc.stk[lv.L0];
  }
  __syncwarp();
  for (int l = lv.L0 + 1; l <= lv.Lm; ++l) {  // complete right-spine ancestors
    if (((t + 1) & ((1 << l) - 1)) != 0) break;
    const int m = t >> l;
    if (m >= (lv.cap >> l)) break;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = i * 32 + lane;
      if (d >= DH) continue;
      lg[base + (int64_t)(lv.off[l] + m) * DH + d] = lg[base + (int64_t)(lv.off[l - 1] + 2 * m) * DH + d] +
                                                     lg[base + (int64_t)(lv.off[l - 1] + 2 * m + 1) * DH + d];
    }
    __syncwarp();
  }
  for (int l = lv.L0; l <= lv.Lm; ++l) {
    if (((t + 1) & ((1 << l) - 1)) != 0) break;
    const int m = t >> l;
    if (m >= (lv.cap >> l)) break;
    const int64_t row = base + (int64_t)(lv.off[l] + m) * DH;
    if (l >= gate_min) {
      gate_node_warp<DH>(raw + row, lg + row, out + row, __int_as_float((127 - l) << 23), gate_q, lane);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i)
        if (i * 32 + lane < DH) out[row + i * 32 + lane] = raw[row + i * 32 + lane];
    }
    __syncwarp();
  }
}

}  // namespace ta
