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

// Leaf level: one thread per (bh, leaf node m, dim d). Reads 2^L0 keys of dim d; with zero_sink the key at
// position 0 enters as 0.
template <typename T>
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
    return ((p != 0 || !zero_sink) && p < T_len) ? to_f32(kp[(int64_t)p * k_st]) : 0.f;
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

}  // namespace ta
