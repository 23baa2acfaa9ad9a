// The decode step's linear layers on the tensor cores (the callers around the hot path): out = act W^T for the
// batch's rows, W an nn.Linear weight (N out features x K in features, K contiguous), bf16 or f16 operands, fp32
// accumulation in tensor memory. Reference: model.py:21-44 (c_attn, c_proj, c_fc + GELU, c_mlp), model.py:90 /
// engine.py:177 (the lm_head on the tied embedding), phase2.py:61-62 (greedy argmax).
//
// The batch is small (64 rows in configuration 4), so the weights are the stream and the rows are the MMA's N:
//   CTA tile  128 output features (MMA M = TMEM lanes) x BN rows (the batch padded to a multiple of 16, MMA N)
//             over a K slice; grid = ceil(N / 128) x splits.
//   warp 4    TMA producer: the weight tile in copies of nb 64-wide K blocks (nb x 16 KB, 128-byte swizzle: few large
//             copies, since an SM's copy throughput grows with the copy size) into an NST-stage ring.
//             The first NST blocks are requested before the kernel waits for the grid it depends on (programmatic
//             dependent launch): the weights do not depend on it, so they stream while the previous kernel ends.
//             After that wait it also requests the CTA's K slice of the rows (one box of BN rows per K block, the
//             rows past B filled with zeros by the copy), all on one barrier.
//   warps 0-3 read the accumulator out of TMEM (thread = output feature) and write the epilogue.
//   warp 5    allocates TMEM; one thread issues tcgen05.mma (K = 16 each) as the weight blocks land.
// Epilogues: STORE (out rows in T), GELU (exact erf GELU of the T-rounded sum, as F.gelu(F.linear(...)) in T),
// PARTIAL (the split's fp32 sums into part[split] - the residual kernel adds the splits in order), ARGMAX (STORE
// plus, per row, the tile's largest T-rounded value and its first index as one 64-bit key in keys[tile, row], which
// argmax_finish_kernel reduces over the tiles). STORE / GELU / ARGMAX with K splits: every split writes its fp32
// tile to a workspace and the last split of the tile to arrive (an arrival counter, no waiting) adds them in split
// order and writes the epilogue, so the result does not depend on the arrival order.
// Every wait is a bounded mbarrier wait; on a timeout the CTA records the error, waits (bounded) for its copies and
// MMAs in flight, frees its TMEM and returns.
#pragma once
#include <type_traits>
#include "common.cuh"
#include "tc.cuh"

namespace ta {

constexpr int LIN_THREADS = 192;
constexpr int LIN_MT = 128;        // output features per CTA (MMA M)
constexpr int LIN_KB = 64;         // K per block (one 128-byte swizzled row of 16-bit elements)
constexpr int LIN_W_BYTES = LIN_MT * LIN_KB * 2;  // one weight block
constexpr int LIN_MAX_BN = 256;    // MMA N limit
constexpr int K_LINEAR = 14;

enum LinearMode : int { LIN_STORE = 0, LIN_GELU = 1, LIN_PARTIAL = 2, LIN_ARGMAX = 3 };

struct LinearParams {
  int B, BN;             // rows; rows padded to a multiple of 16 (MMA N)
  int N, K, Ks;          // out features, in features, K per split (a multiple of 64)
  int nb;                // 64-wide K blocks per weight copy (one TMA box of nb x 16 KB)
  int na;                // 64-wide K blocks per copy of the rows
  int nst;               // weight ring stages (nb blocks each)
  void* out;             // STORE / GELU / ARGMAX: (B, N) T, row stride out_ld
  int64_t out_ld;
  float* part;           // PARTIAL: (splits, B, N) fp32
  unsigned long long* keys;  // ARGMAX: (ceil(N / 128), B) per-tile row keys
  float* ws;             // other modes with K splits: (tiles, splits, B, 128) fp32 tile sums
  int* counters;         // ... and (tiles,) arrival counts, zero between launches
};

constexpr int LIN_MAX_NST = 8;

struct LinBars {
  uint64_t act_full, mma_done;
  uint64_t w_full[LIN_MAX_NST], w_empty[LIN_MAX_NST];
  uint32_t tmem_base;
  int abort_flag;
  int last;    // this CTA completes its tile (the last of the K splits to arrive)
  int epi_ok;  // the MMAs completed: the epilogue warps write their tile
};

// Operand space (weight ring, then the rows' slice); once the MMAs are done the same space holds the fp32 output
// tile (BN rows x 128 features, row-major) on its way out.
__host__ __device__ inline size_t linear_operand_bytes(int BN, int Ks, int nst, int nb) {
  const size_t ops = (size_t)nst * nb * LIN_W_BYTES + (size_t)(Ks / LIN_KB) * BN * 128;
  const size_t tile = (size_t)BN * LIN_MT * 4;
  return ops > tile ? ops : tile;
}

__host__ __device__ inline size_t linear_smem_bytes(int BN, int Ks, int nst, int nb) {
  return 1024 + linear_operand_bytes(BN, Ks, nst, nb) + sizeof(LinBars) + 16;
}

// Tiled 3-D load of the tensor map's box at (c0 innermost, c1, c2) into dst, completing on bar.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Order-preserving map of an fp32 value to an unsigned key (NaN above everything, as torch.argmax ranks it).
__device__ __forceinline__ uint32_t f32_order_key(float v) {
  if (v != v) return 0xffffffffu;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

// Both tensor maps view a (rows, K) 16-bit matrix as (64, rows, K / 64): a box of (64, R, n) is n consecutive
// 64-wide K blocks of R rows, each landing as one 128-byte-swizzled K-major tile of R x 128 bytes.
template <typename T, int MODE>
__global__ void __launch_bounds__(LIN_THREADS, 1)
    linear_rows_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                       LinearParams p) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char lin_smem_raw[];
  const uint32_t raw_a = smem_u32(lin_smem_raw);
  unsigned char* base = lin_smem_raw + (((raw_a + 1023u) & ~1023u) - raw_a);
  const int nkb = p.Ks / LIN_KB;           // K blocks of this CTA
  const int NB = p.nb, NST = p.nst;
  const int nstage = nkb / NB;             // weight copies
  const uint32_t stage_bytes = (uint32_t)NB * LIN_W_BYTES;
  unsigned char* sW = base;
  unsigned char* sA = sW + (size_t)NST * stage_bytes;
  LinBars& bar = *reinterpret_cast<LinBars*>(base + linear_operand_bytes(p.BN, p.Ks, NST, NB));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int f0 = (int)blockIdx.x * LIN_MT;
  const int split = (int)blockIdx.y;
  const int kb0 = split * nkb;             // first K block of the slice
  const uint32_t tcols = p.BN <= 32 ? 32u : (p.BN <= 64 ? 64u : (p.BN <= 128 ? 128u : 256u));

  if (tid == 0) {
    mbar_init(&bar.act_full, 1);
    mbar_init(&bar.mma_done, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&bar.w_full[s], 1);
      mbar_init(&bar.w_empty[s], 1);
    }
    bar.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_map(&tm_w);
    tma_prefetch_map(&tm_a);
  }
  if (warp == 5) {
    tmem_alloc(&bar.tmem_base, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // the next kernel of the chain may start its own weight prefetch wherever this grid leaves room
  pdl_launch_dependents();

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      bool rows = false;
      // the rows, once the grid they come from has completed (the weights do not depend on it)
      auto load_rows = [&]() {
        rows = true;
        pdl_wait();
        mbar_arrive_expect_tx(&bar.act_full, (uint32_t)(nkb * p.BN * 128));
        for (int kb = 0; kb < nkb; kb += p.na)
          tma_load_3d(sA + (size_t)kb * p.BN * 128, &tm_a, 0, 0, kb0 + kb, &bar.act_full);
      };
      for (; issued < nstage; ++issued) {
        const int s = issued % NST;
        if (issued == NST) load_rows();  // after the weight ring's first fill
        if (issued >= NST) {
          if (!mbar_wait_bounded(&bar.w_empty[s], ((issued / NST) - 1) & 1, K_LINEAR, 1)) {
            atomicExch(&bar.abort_flag, 1);
            break;
          }
          if (*reinterpret_cast<volatile int*>(&bar.abort_flag)) break;
        }
        mbar_arrive_expect_tx(&bar.w_full[s], stage_bytes);
        tma_load_3d(sW + (size_t)s * stage_bytes, &tm_w, 0, f0, kb0 + issued * NB, &bar.w_full[s]);
      }
      if (!rows) load_rows();  // the whole slice fit in the ring
      // no copy of this CTA may still be in flight when it exits
      mbar_wait_bounded(&bar.act_full, 0, K_LINEAR, 7);
      for (int i = max(issued - NST, 0); i < issued; ++i)
        mbar_wait_bounded(&bar.w_full[i % NST], (i / NST) & 1, K_LINEAR, 2);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(LIN_MT, p.BN, BF, false);
      const uint32_t aW = smem_u32(sW), aA = smem_u32(sA);
      bool ok = mbar_wait_bounded(&bar.act_full, 0, K_LINEAR, 3);
      for (int st = 0; ok && st < nstage; ++st) {
        const int s = st % NST;
        if (!(ok = mbar_wait_bounded(&bar.w_full[s], (st / NST) & 1, K_LINEAR, 4))) break;
        if (*reinterpret_cast<volatile int*>(&bar.abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < NB; ++j) {
          const int kb = st * NB + j;
          const uint32_t wa = aW + s * stage_bytes + j * LIN_W_BYTES, xa = aA + kb * p.BN * 128;
#pragma unroll
          for (int k = 0; k < LIN_KB / 16; ++k)
            umma_f16(bar.tmem_base, sw128_desc(wa + k * 32, 16, 1024), sw128_desc(xa + k * 32, 16, 1024), idesc,
                     kb > 0 || k > 0);
        }
        umma_commit(&bar.w_empty[s]);
      }
      if (!ok) atomicExch(&bar.abort_flag, 1);
      umma_commit(&bar.mma_done);
      mbar_wait_bounded(&bar.mma_done, 0, K_LINEAR, 5);  // every MMA of this CTA has completed
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ accumulator out (warps 0-3)
    pdl_wait();  // the outputs may still be read by the grid this one follows
    if (!mbar_wait_bounded(&bar.mma_done, 0, K_LINEAR, 6)) atomicExch(&bar.abort_flag, 1);
    named_bar_sync(1, 128);
    if (tid == 0) bar.epi_ok = *reinterpret_cast<volatile int*>(&bar.abort_flag) == 0;
    named_bar_sync(1, 128);
    const bool ok = bar.epi_ok != 0;  // one outcome for the 4 warps (the named barriers below need all of them)
    tc_fence_after();
    const uint32_t lane_base = bar.tmem_base + ((uint32_t)(warp * 32) << 16);
    // The accumulator goes through a row-major fp32 tile in shared memory (the operand space is free once the MMAs
    // are done): a thread holds one feature of every row, the rows leave in 16-byte pieces.
    float* tile = reinterpret_cast<float*>(base);
    const int fl = warp * 32 + lane;  // this thread's feature in the tile (its TMEM lane)
    for (int c0 = 0; ok && c0 < p.BN; c0 += 32) {
      float v[32];
      tmem_ld32(lane_base + c0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c0 + i < p.B) tile[(c0 + i) * LIN_MT + fl] = v[i];
    }
    tc_fence_before();
    named_bar_sync(1, 128);
    const int S = (int)gridDim.y;
    const int n4 = p.B * (LIN_MT / 4);  // float4 pieces of the tile
    if (ok && MODE == LIN_PARTIAL) {
      float* dst = p.part + (int64_t)split * p.B * p.N + f0;
      for (int id = tid; id < n4; id += 128) {
        const int r = id >> 5, c = (id & 31) * 4;
        if (f0 + c < p.N)
          *reinterpret_cast<float4*>(dst + (int64_t)r * p.N + c) = *reinterpret_cast<const float4*>(tile + r * LIN_MT + c);
      }
    } else if (ok) {
      if (S > 1) {
        // this split's sums to the workspace; the last split of the tile to arrive adds them all, in split order
        float* ws = p.ws + (int64_t)blockIdx.x * S * p.B * LIN_MT;
        for (int id = tid; id < n4; id += 128)
          reinterpret_cast<float4*>(ws + (int64_t)split * p.B * LIN_MT)[id] = reinterpret_cast<const float4*>(tile)[id];
        __threadfence();
        named_bar_sync(1, 128);
        if (tid == 0) bar.last = atomicAdd(p.counters + blockIdx.x, 1) == S - 1;
        named_bar_sync(1, 128);
        if (bar.last) {
          __threadfence();
          // 8 pieces per thread in flight at a time (the loads of one split are independent of each other)
          constexpr int U = 8;
          for (int id0 = tid; id0 < n4; id0 += 128 * U) {
            float4 a[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (id0 + u * 128 < n4) a[u] = __ldcg(reinterpret_cast<const float4*>(ws) + id0 + u * 128);
            for (int sp = 1; sp < S; ++sp) {
              const float4* src = reinterpret_cast<const float4*>(ws + (int64_t)sp * p.B * LIN_MT) + id0;
              float4 b4[U];
#pragma unroll
              for (int u = 0; u < U; ++u)
                if (id0 + u * 128 < n4) b4[u] = __ldcg(src + u * 128);
#pragma unroll
              for (int u = 0; u < U; ++u) {
                a[u].x += b4[u].x; a[u].y += b4[u].y; a[u].z += b4[u].z; a[u].w += b4[u].w;
              }
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (id0 + u * 128 < n4) reinterpret_cast<float4*>(tile)[id0 + u * 128] = a[u];
          }
          if (tid == 0) p.counters[blockIdx.x] = 0;  // ready for the next launch
          named_bar_sync(1, 128);
        }
      }
      if (S == 1 || bar.last) {
        // 8 features per thread: rounded (GELU), packed, stored; ARGMAX also folds the row's best (rounded value,
        // first index) over the 16 threads that hold the row
        T* out = reinterpret_cast<T*>(p.out);
        const int n8 = p.B * (LIN_MT / 8);
        for (int j = 0; j < (p.BN * (LIN_MT / 8) + 127) / 128; ++j) {
          const int id = tid + j * 128;
          const int r = id >> 4, c = (id & 15) * 8, f = f0 + c;
          const bool live = id < n8 && f < p.N;
          unsigned long long key = 0ull;
          if (live) {
            const float4 lo = *reinterpret_cast<const float4*>(tile + r * LIN_MT + c);
            const float4 hi = *reinterpret_cast<const float4*>(tile + r * LIN_MT + c + 4);
            float o[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            if (MODE == LIN_GELU) {
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = gelu_erf(to_f32(from_f32<T>(o[e])));
            }
            store_vec_from_f32<T>(out + (int64_t)r * p.out_ld + f, o);
            if (MODE == LIN_ARGMAX) {
              // key = value order << 32 | ~index: the larger key is the larger rounded value, then the smaller index
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const unsigned long long k = ((unsigned long long)f32_order_key(to_f32(from_f32<T>(o[e]))) << 32) |
                                             (unsigned long long)(0xffffffffu - (uint32_t)(f + e));
                key = k > key ? k : key;
              }
            }
          }
          if (MODE == LIN_ARGMAX) {
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) {
              const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, sh);
              key = other > key ? other : key;
            }
            if ((id & 15) == 0 && id < n8) p.keys[(int64_t)blockIdx.x * p.B + r] = key;
          }
        }
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(bar.tmem_base, tcols);
  }
}

// tok[b] = the index in the largest of keys[0 .. n_tiles-1, b] (the row's largest logit, its first index on ties),
// pos[b] += 1. One warp per row.
__global__ void __launch_bounds__(128) argmax_finish_kernel(const unsigned long long* __restrict__ keys, int n_tiles,
                                                            int B, int V, int64_t* tok, int32_t* pos) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (b >= B) return;
  unsigned long long key = 0ull;
  for (int t = lane; t < n_tiles; t += 32) {
    const unsigned long long k = keys[(int64_t)t * B + b];
    key = k > key ? k : key;
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, s);
    key = other > key ? other : key;
  }
  if (lane == 0) {
    int64_t idx = (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    if (key == 0ull || idx >= V) {
      record_error(DEV_INDEX_RANGE, K_ROWS, (int)idx, V);
      idx = 0;
    }
    tok[b] = idx;
    pos[b] += 1;
  }
}

// x[b] += round_T(sum over the splits s = 0 .. S-1 of part[s, b]) (the projection's output rounded to the model
// dtype, as F.linear returns it, added to the fp32 residual), h[b] = LN(x[b]) * w (T). One CTA per row, one thread
// per 8 features (C a multiple of 8, at most 8 x 256), 16-byte accesses; each thread requests the splits' pieces
// eight at a time before adding them, in split order.
constexpr int ASL_MAX_WARPS = 8;

__device__ __forceinline__ float block_sum_rows(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  __syncthreads();
  return t;
}

template <typename T>
__global__ void __launch_bounds__(256) add_splits_ln_kernel(float* x, const float* __restrict__ part, int S, int B,
                                                             int C, const float* __restrict__ w, float eps, T* h) {
  __shared__ float red[ASL_MAX_WARPS];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x, c = threadIdx.x * 8;
  const bool live = c < C;
  const int64_t sstride = (int64_t)B * C;
  float v[8];
  float sum = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
  if (live) {
    const float* pr = part + (int64_t)row * C + c;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    constexpr int G = 8;
    for (int s0 = 0; s0 < S; s0 += G) {
      float4 q[G][2];
#pragma unroll
      for (int u = 0; u < G; ++u)
        if (s0 + u < S) {
          q[u][0] = __ldcg(reinterpret_cast<const float4*>(pr + (s0 + u) * sstride));
          q[u][1] = __ldcg(reinterpret_cast<const float4*>(pr + (s0 + u) * sstride + 4));
        }
#pragma unroll
      for (int u = 0; u < G; ++u)
        if (s0 + u < S) {
          // the first split starts the sum (0 + a == a exactly), the others follow in order
          acc[0] += q[u][0].x; acc[1] += q[u][0].y; acc[2] += q[u][0].z; acc[3] += q[u][0].w;
          acc[4] += q[u][1].x; acc[5] += q[u][1].y; acc[6] += q[u][1].z; acc[7] += q[u][1].w;
        }
    }
    float* xr = x + (int64_t)row * C + c;
    const float4 x0 = *reinterpret_cast<const float4*>(xr), x1 = *reinterpret_cast<const float4*>(xr + 4);
    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[e] = xs[e] + to_f32(from_f32<T>(acc[e]));
      sum += v[e];
    }
    *reinterpret_cast<float4*>(xr) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(xr + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  const float mean = block_sum_rows(sum, red) / (float)C;
  float q2 = 0.f;
  if (live) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = v[e] - mean;
      q2 = fmaf(d, d, q2);
    }
  }
  const float rstd = rsqrtf(block_sum_rows(q2, red) / (float)C + eps);
  if (live) {
    float o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = (v[e] - mean) * rstd * w[c + e];
    store_vec_from_f32<T>(h + (int64_t)row * C + c, o8);
  }
}

}  // namespace ta
