// Small fused row kernels of the decode step around the attention (the callers of the hot path): token + position
// embedding with the first layer norm, residual add with the next layer norm, and greedy argmax with the
// token/position advance. Each replaces 2-4 separate elementwise launches per layer.
//
// Reference: model.py:12-18 (LayerNorm: no bias, eps 1e-5), model.py:75-77 / engine.py:165 (x = wte[tok] +
// wpe[t]), engine.py:168/176 (ln1 / ln2 before the matmuls), phase2.py:61-62 (greedy argmax of the logits).
#pragma once
#include "common.cuh"

namespace ta {

constexpr int ROW_THREADS = 256;

// Block-wide sum of two values (all ROW_THREADS threads call it).
__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (lane == 0) red[warp] = make_float2(a, b);
  __syncthreads();
  float2 r = make_float2(0.f, 0.f);
  for (int w = 0; w < ROW_THREADS / 32; ++w) {
    r.x += red[w].x;
    r.y += red[w].y;
  }
  __syncthreads();
  return r;
}

// Layer norm of one fp32 row held in registers (vals[i] = x[tid + i*ROW_THREADS]); writes w * (x - mean) / sqrt(var +
// eps) as T. Mean and variance in fp32, two passes over the registers.
template <typename T, int MAXV>
__device__ __forceinline__ void ln_row_store(const float (&vals)[MAXV], int C, const float* __restrict__ w, float eps,
                                             T* __restrict__ out, float2* red) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * ROW_THREADS;
    if (c < C) s += vals[i];
  }
  const float mean = block_sum2(s, 0.f, red).x / (float)C;
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * ROW_THREADS;
    if (c < C) {
      const float d = vals[i] - mean;
      v = fmaf(d, d, v);
    }
  }
  const float var = block_sum2(v, 0.f, red).x / (float)C;
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * ROW_THREADS;
    if (c < C) out[c] = from_f32<T>((vals[i] - mean) * rstd * w[c]);
  }
}

// x[b] = wte[tok[b]] + wpe[pos[b]] (fp32), h[b] = LN(x[b]) * w (T). One CTA per row.
template <typename T, int MAXV>
__global__ void __launch_bounds__(ROW_THREADS) embed_ln_kernel(const T* __restrict__ wte, const T* __restrict__ wpe,
                                                               const int64_t* __restrict__ tok,
                                                               const int32_t* __restrict__ pos, int V, int P, int C,
                                                               const float* __restrict__ w, float eps, float* x,
                                                               T* h) {
  __shared__ float2 red[ROW_THREADS / 32];
  pdl_wait();  // tokens and positions come from the previous step's greedy argmax
  pdl_launch_dependents();
  const int b = blockIdx.x;
  int64_t tk = tok[b];
  int ps = pos[b];
  if (tk < 0 || tk >= V || ps < 0 || ps >= P) {
    if (threadIdx.x == 0) record_error(DEV_INDEX_RANGE, K_ROWS, (int)tk, ps);
    tk = tk < 0 ? 0 : (tk >= V ? V - 1 : tk);
    ps = ps < 0 ? 0 : (ps >= P ? P - 1 : ps);
  }
  float vals[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * ROW_THREADS;
    vals[i] = 0.f;
    if (c < C) {
      vals[i] = to_f32(wte[tk * C + c]) + to_f32(wpe[(int64_t)ps * C + c]);
      x[(int64_t)b * C + c] = vals[i];
    }
  }
  ln_row_store<T, MAXV>(vals, C, w, eps, h + (int64_t)b * C, red);
}

// x[b] += y[b] (y in T, may be null), h[b] = LN(x[b]) * w (T). One warp per row, shuffle reductions only,
// 16-byte vector accesses (C a multiple of 8, rows 16-byte aligned; checked by the caller).
template <typename T, int NV>  // NV = 16-byte chunks (8 elements) per lane: C <= 256 * NV
__global__ void __launch_bounds__(128) add_ln_warp_kernel(float* x, const T* __restrict__ y, int B, int C,
                                                          const float* __restrict__ w, float eps, T* h) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= B) return;
  float* xr = x + (int64_t)warp * C;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + i * 32) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    if (c < C) {
      const float4 a = *reinterpret_cast<const float4*>(xr + c);
      const float4 bq = *reinterpret_cast<const float4*>(xr + c + 4);
      v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
      v[i][4] = bq.x; v[i][5] = bq.y; v[i][6] = bq.z; v[i][7] = bq.w;
      if (y) {
        float yv[8];
        load_vec_f32<T>(y + (int64_t)warp * C + c, yv);
        if constexpr (sizeof(T) == 4) load_vec_f32<T>(y + (int64_t)warp * C + c + 4, yv + 4);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] += yv[e];
        *reinterpret_cast<float4*>(xr + c) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        *reinterpret_cast<float4*>(xr + c + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[i][e];
    }
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + i * 32) * 8;
    if (c < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mean;
        q = fmaf(d, d, q);
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / (float)C + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + i * 32) * 8;
    if (c < C) {
      float o8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o8[e] = (v[i][e] - mean) * rstd * w[c + e];
      if constexpr (sizeof(T) == 2) {
        store_vec_from_f32<T>(h + (int64_t)warp * C + c, o8);
      } else {
        store_vec_from_f32<T>(h + (int64_t)warp * C + c, o8);
        store_vec_from_f32<T>(h + (int64_t)warp * C + c + 4, o8 + 4);
      }
    }
  }
}

// Exact (erf) GELU in place on n elements (F.gelu default), 16-byte vectors; n a multiple of 8.
template <typename T>
__global__ void __launch_bounds__(256) gelu_kernel(T* x, int64_t n) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= n) return;
  float v[8];
  if constexpr (sizeof(T) == 2) {
    load_vec_f32<T>(x + i, v);
  } else {
    load_vec_f32<T>(x + i, v);
    load_vec_f32<T>(x + i + 4, v + 4);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.5f * v[e] * (1.f + erff(v[e] * 0.70710678118654752f));
  if constexpr (sizeof(T) == 2) {
    store_vec_from_f32<T>(x + i, v);
  } else {
    store_vec_from_f32<T>(x + i, v);
    store_vec_from_f32<T>(x + i + 4, v + 4);
  }
}

// tok[b] = argmax_v logits[b, v] (the first maximum, NaN counted as the largest value as torch.argmax does),
// pos[b] += 1. One CTA of ARG_THREADS per row, 16-byte vector loads.
constexpr int ARG_THREADS = 1024;

__device__ __forceinline__ bool arg_better(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  return a > b || (a == b && ia < ib);
}

template <typename T>
__global__ void __launch_bounds__(ARG_THREADS) argmax_advance_kernel(const T* __restrict__ logits, int V,
                                                                     int64_t* tok, int32_t* pos) {
  __shared__ float sv[ARG_THREADS / 32];
  __shared__ int si[ARG_THREADS / 32];
  constexpr int VEC = TypeInfo<T>::VEC;
  const int b = blockIdx.x;
  const T* row = logits + (int64_t)b * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int nvec = ((V % VEC) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) ? V / VEC : 0;
  for (int j = threadIdx.x; j < nvec; j += ARG_THREADS) {
    float f[VEC];
    ldg_vec_f32<T>(row + (int64_t)j * VEC, f);
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      if (arg_better(f[e], j * VEC + e, best, bi)) { best = f[e]; bi = j * VEC + e; }
  }
  for (int v = nvec * VEC + threadIdx.x; v < V; v += ARG_THREADS) {
    const float f = to_f32(row[v]);
    if (arg_better(f, v, best, bi)) { best = f; bi = v; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (arg_better(ob, oi, best, bi)) { best = ob; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = sv[lane];
    bi = si[lane];
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (arg_better(ob, oi, best, bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) {
      tok[b] = bi;
      pos[b] += 1;
    }
  }
}

}  // namespace ta
