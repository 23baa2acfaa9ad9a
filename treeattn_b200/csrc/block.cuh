// The decode step's block tail in one launch: everything a transformer block does after its attention, plus the next
// block's q/k/v projection, for the batch's rows (reference: model.py:21-44 - Block.forward's x + attn.c_proj(y),
// ln_2, mlp.c_fc, GELU, mlp.c_proj, x + mlp(...); the next block's ln_1 and c_attn; engine.py:161-177 runs that
// chain once per decoded token):
//
//   P1  part_proj[s] = att W_proj^T over K slice s                  (tcgen05, fp32 partial sums)
//   P2  x += round(sum_s part_proj[s]);  h2 = ln_2(x)               (one CTA per row)
//   P3  fc = round(gelu(round(h2 W_fc^T)))                          (tcgen05, K splits summed by the tile's last split)
//   P4  part_mlp[s] = fc W_mlp^T over K slice s                     (tcgen05)
//   P5  x += round(sum_s part_mlp[s]);  h = ln_next(x)              (the next block's ln_1, or ln_f after the last)
//   P6  qkv = round(h W_attn^T)                                     (the next block's c_attn; absent after the last)
//
// The separate launches this replaces (four GEMMs, two residual + layer-norm kernels and a GELU per block) are each a
// few microseconds of latency on 64 rows; here every GEMM is cut into units of (128 output features x a K slice)
// spread over one CTA per SM, and the phases are ordered by counters in global memory instead of kernel boundaries:
// a unit waits only for what it reads (P3 for all of P2's rows, a P4 unit for the P3 tiles holding its K slice, P6
// for all of P5's rows). All CTAs are resident at once (one per SM, the launcher checks the occupancy), so these
// waits always end; each is bounded anyway (TA_WAIT_LIMIT_NS), and a CTA that gives up records the error and raises
// an abort word that ends every other CTA's waits.
//
// Weights: each CTA streams its units' weight slices, K block by K block (128 x 64, 128-byte swizzle), through a
// ring of shared-memory slots in unit order; the first ring-full is requested at launch, before the CTA waits for
// the attention kernel it follows (programmatic dependent launch), so most of the layer's ~14 MB streams in while
// the attention drains. Rows (the MMA's N, the batch padded to 16) come with one TMA copy per unit.
//
// Warps: 0-3 workers (dependency waits, row staging, TMEM epilogues, layer norms, signals), 4 TMA producer, 5 TMEM
// owner + MMA issuer. Sync words (int32, zero between launches; the last CTA to leave zeroes them):
//   [0] P1 units done  [1] P2 rows done  [2] P4 units done  [3] P5 rows done  [4] CTAs left  [5] abort
//   [8 .. 8+Tf) P3 split arrivals per tile, [8+Tf .. 8+2Tf) P3 tiles written, [8+2Tf .. 8+2Tf+Tq) P6 split arrivals.
#pragma once
#include <type_traits>
#include "common.cuh"
#include "tc.cuh"
#include "linear.cuh"

namespace ta {

constexpr int BT_THREADS = 192;
constexpr int BT_MAXU = 8;          // GEMM units one CTA may hold
constexpr int BT_MAX_SLOTS = 16;    // weight ring slots (one 128 x 64 block each)
constexpr int BT_MAX_BN = 128;      // rows (padded) per launch
constexpr int BT_MAX_C = 2048;      // row width the layer-norm phases take (8 features per worker thread, 2 passes)
constexpr int K_BLOCK_TAIL = 15;

#ifdef TA_TAIL_TRACE
// Profiling build only: per CTA, %globaltimer at the phase boundaries (slot meanings at the TAIL_MARK calls).
__device__ unsigned long long g_tail_trace[256][32];
#define TAIL_MARK(i)                                                                        \
  do {                                                                                      \
    if (blockIdx.x < 256) g_tail_trace[blockIdx.x][(i)] = global_timer_ns();                \
  } while (0)
#else
#define TAIL_MARK(i) \
  do {               \
  } while (0)
#endif

enum TailGemmId : int { TG_PROJ = 0, TG_FC = 1, TG_MLP = 2, TG_QKV = 3 };
enum TailSyncWord : int { TW_PROJ = 0, TW_LN2 = 1, TW_MLP = 2, TW_LN1 = 3, TW_EXIT = 4, TW_ABORT = 5, TW_FIXED = 8 };

// One GEMM phase: unit u = (tile u / S, split u % S) covers output features [128 tile, 128 tile + 128) over K blocks
// [kc split, kc (split + 1)) and runs on CTA (off + u) % G.
struct TailGemm {
  int N, K;   // out features, in features
  int S;      // K splits
  int kc;     // 64-wide K blocks per unit
  int n;      // units = N / 128 * S
  int off;
};

struct BlockTailParams {
  int B, BN, C, G;
  int nslot;                // weight ring slots
  TailGemm g[4];
  int off_ln;               // layer-norm row r runs on CTA (off_ln + r) % G
  int nsync;                // sync words
  const void* att;          // (B, C) T, row stride C: the attention output
  float* x;                 // (B, C) fp32 residual stream, updated in place
  const float* ln2;         // (C,) ln_2 weight
  const float* ln_next;     // (C,) the next block's ln_1 weight (ln_f after the last block)
  float eps;
  void* h2;                 // (B, C) T scratch: ln_2 output
  void* fc;                 // (B, 4C) T scratch: GELU output
  void* h;                  // (B, C) T: ln_next output
  void* qkv;                // (B, 3C) T: the next block's projection (g[3].n == 0: none)
  float* part_proj;         // (S_proj, B, C)
  float* ws_fc;             // (4C / 128, S_fc, BN, 128): per tile and split, its fp32 tile row-major
  float* part_mlp;          // (S_mlp, B, C)
  float* ws_qkv;            // (3C / 128, S_qkv, BN, 128)
  int* sync;
};

// Tensor maps of one launch: the four weights (box 64 x 128: one K block) and the four row sources the GEMMs read
// (att, h2, fc, h: box 64 x BN, one K block; rows past B read as zeros).
struct TailMaps {
  CUtensorMap w[4];
  CUtensorMap a[4];
};

struct TailBars {
  uint64_t w_full[BT_MAX_SLOTS], w_empty[BT_MAX_SLOTS];
  uint64_t act_full, mma_done, fin, ln_full;
  uint32_t tmem_base;
  int abort_flag;           // this CTA gave up (workers or MMA issuer)
  int nu;                   // this CTA's units, in phase order
  int u_gemm[BT_MAXU], u_id[BT_MAXU];
  float red[4];
};

__host__ __device__ inline size_t tail_act_bytes(int BN, int kc_max) { return (size_t)kc_max * BN * 128; }

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// bar.sync on a named barrier that also returns the OR of every participant's predicate: one decision for all.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Wait for an mbarrier phase, giving up when this CTA's abort flag is raised or after TA_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, const int* abort_flag, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<const volatile int*>(abort_flag)) return false;
    if ((++spins & 3u) == 0 && global_timer_ns() - t0 > TA_WAIT_LIMIT_NS) {
      record_error(DEV_WAIT_TIMEOUT, K_BLOCK_TAIL, where, (int)parity);
      return false;
    }
  }
}

// Worker thread 0 waits until every counter in ctr[0 .. n) reaches `target` (acquire), then the 128 workers agree on
// the outcome. False: this CTA gives up (a wait ran out, or another CTA raised the abort word).
__device__ __forceinline__ bool tail_wait(const BlockTailParams& p, const int* ctr, int n, int target, int where) {
  bool bad = false;
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    for (int i = 0; i < n && !bad; ++i) {
      while (ld_acquire_gpu(ctr + i) < target) {
        if (ld_acquire_gpu(p.sync + TW_ABORT)) { bad = true; break; }
        if ((++spins & 15u) == 0 && global_timer_ns() - t0 > TA_WAIT_LIMIT_NS) {
          record_error(DEV_WAIT_TIMEOUT, K_BLOCK_TAIL, where, target);
          atomicExch(p.sync + TW_ABORT, 1);
          bad = true;
          break;
        }
      }
    }
  }
  return !named_bar_or(1, 128, bad);
}

__device__ __forceinline__ void red_release_gpu(int* p, int n) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(n) : "memory");
}

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int n) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(n) : "memory");
  return old;
}

// After the workers' global writes: one release increment of ctr by n (the barrier orders the other workers'
// writes before it). The writes are fenced for the async proxy first (the consumers read rows with TMA copies).
__device__ __forceinline__ void tail_signal(int* ctr, int n) {
  fence_proxy_async_global();
  named_bar_sync(1, 128);
  if (threadIdx.x == 0) red_release_gpu(ctr, n);
}

__device__ __forceinline__ float workers_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  named_bar_sync(1, 128);
  const float t = red[0] + red[1] + red[2] + red[3];
  named_bar_sync(1, 128);
  return t;
}

// Bytes of the stage area: a unit's rows (kc_max K blocks of BN rows), a layer-norm row's inputs (the S partial
// rows and the residual row, fp32) or a unit's fp32 output tile, whichever is largest.
__host__ __device__ inline size_t tail_stage_bytes(int BN, int kc_max, int C, int s_ln) {
  size_t a = tail_act_bytes(BN, kc_max);
  const size_t l = (size_t)(s_ln + 1) * C * 4, t = (size_t)BN * LIN_MT * 4;  // layer-norm inputs, fp32 out tile
  a = a > l ? a : l;
  a = a > t ? a : t;
  return (a + 1023) / 1024 * 1024;
}

// x[r] += round_T(sum over s of part[s, r]) (in split order), out[r] = LN(x[r]) * w. The S partial rows and the
// residual row come into the stage with one bulk copy each (written by other CTAs' generic stores, observed through
// the counter the caller waited on); then 8 features per worker thread.
// False: the copies did not land (this CTA gives up).
template <typename T>
__device__ __forceinline__ bool tail_ln_row(const BlockTailParams& p, TailBars& bar, float* stage, uint32_t parity,
                                            int r, const float* part, int S, const float* w, T* out) {
  const int C = p.C, tid = threadIdx.x;
  if (tid == 0) mbar_arrive_expect_tx(&bar.ln_full, (uint32_t)((S + 1) * C * 4));
  named_bar_sync(1, 128);
  if ((tid & 31) == 0) {  // the copies issued by the four worker warps in turn
    fence_proxy_async_global();
    fence_proxy_async_smem();
    for (int s = tid >> 5; s <= S; s += 4)
      bulk_g2s(stage + s * C, s < S ? part + ((int64_t)s * p.B + r) * C : p.x + (int64_t)r * C, (uint32_t)C * 4,
               &bar.ln_full);
  }
  const bool landed = mbar_wait_or_abort(&bar.ln_full, parity, &bar.abort_flag, 6);
  if (named_bar_or(1, 128, !landed)) return false;
  float v[2][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = (tid + i * 128) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    if (c < C) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int s = 0; s < S; ++s) {
        // the first split starts the sum (0 + a == a exactly), the others follow in order
        const float4 a = *reinterpret_cast<const float4*>(stage + s * C + c);
        const float4 b = *reinterpret_cast<const float4*>(stage + s * C + c + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
      const float4 x0 = *reinterpret_cast<const float4*>(stage + S * C + c);
      const float4 x1 = *reinterpret_cast<const float4*>(stage + S * C + c + 4);
      const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[i][e] = xs[e] + to_f32(from_f32<T>(acc[e]));
        sum += v[i][e];
      }
      float* xr = p.x + (int64_t)r * C + c;
      *reinterpret_cast<float4*>(xr) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
      *reinterpret_cast<float4*>(xr + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
    }
  }
  const float mean = workers_sum(sum, bar.red) / (float)C;
  float q2 = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if ((tid + i * 128) * 8 < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mean;
        q2 = fmaf(d, d, q2);
      }
    }
  const float rstd = rsqrtf(workers_sum(q2, bar.red) / (float)C + p.eps);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int c = (tid + i * 128) * 8;
    if (c < C) {
      float o8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o8[e] = (v[i][e] - mean) * rstd * w[c + e];
      store_vec_from_f32<T>(out + (int64_t)r * C + c, o8);
    }
  }
  return true;
}

// The CTA's units in phase order (GEMM g's units u with (off + u) % G == this CTA).
__device__ __forceinline__ int tail_first_unit(const TailGemm& g, int cta, int G) {
  return ((cta - g.off) % G + G) % G;
}

template <typename T, int MAXC>
__global__ void __launch_bounds__(BT_THREADS, 1)
    block_tail_kernel(const __grid_constant__ TailMaps maps, BlockTailParams p) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ unsigned char bt_smem_raw[];
  const uint32_t raw_a = smem_u32(bt_smem_raw);
  unsigned char* base = bt_smem_raw + (((raw_a + 1023u) & ~1023u) - raw_a);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = (int)blockIdx.x, G = p.G;

  // shared memory: the weight ring, then the rows' stage, then the barriers
  int kc_max = 1, nu = 0;
#pragma unroll 1
  for (int gi = 0; gi < 4; ++gi) {
    const TailGemm& g = p.g[gi];
    if (g.n > 0) kc_max = max(kc_max, g.kc);
    for (int u = tail_first_unit(g, cta, G); u < g.n; u += G) ++nu;
  }
  const int NS = p.nslot;
  unsigned char* sW = base;
  unsigned char* sA = base + (size_t)NS * LIN_W_BYTES;
  TailBars& bar = *reinterpret_cast<TailBars*>(
      sA + tail_stage_bytes(p.BN, kc_max, p.C, max(p.g[TG_PROJ].S, p.g[TG_MLP].S)));
  const uint32_t tcols = MAXC <= 32 ? 32u : (MAXC <= 64 ? 64u : 128u);

  if (tid == 0) {
    int k = 0;
    for (int gi = 0; gi < 4; ++gi) {
      const TailGemm& g = p.g[gi];
      for (int u = tail_first_unit(g, cta, G); u < g.n && k < BT_MAXU; u += G, ++k) {
        bar.u_gemm[k] = gi;
        bar.u_id[k] = u;
      }
    }
    bar.nu = k;
    bar.abort_flag = 0;
    if (nu > BT_MAXU || NS < 2 || NS > BT_MAX_SLOTS) {
      record_error(DEV_INDEX_RANGE, K_BLOCK_TAIL, nu, NS);
      bar.abort_flag = 1;
    }
    for (int i = 0; i < BT_MAX_SLOTS; ++i) {
      mbar_init(&bar.w_full[i], 1);
      mbar_init(&bar.w_empty[i], 1);
    }
    mbar_init(&bar.act_full, 1);
    mbar_init(&bar.mma_done, 1);
    mbar_init(&bar.fin, 1);
    mbar_init(&bar.ln_full, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&bar.tmem_base, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const int NU = bar.abort_flag ? 0 : bar.nu;
  if (tid == 0) TAIL_MARK(0);

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer: the weight ring
    if (lane == 0) {
      for (int i = 0; i < 4; ++i) {
        tma_prefetch_map(&maps.w[i]);
        tma_prefetch_map(&maps.a[i]);
      }
      int k = 0;  // K blocks issued
      bool ok = true;
      for (int u = 0; ok && u < NU; ++u) {
        const int gi = bar.u_gemm[u];
        const TailGemm& g = p.g[gi];
        const int tile = bar.u_id[u] / g.S, split = bar.u_id[u] % g.S;
        for (int j = 0; j < g.kc; ++j, ++k) {
          const int slot = k % NS;
          if (k >= NS && !(ok = mbar_wait_or_abort(&bar.w_empty[slot], ((k / NS) - 1) & 1, &bar.abort_flag, 1)))
            break;
          mbar_arrive_expect_tx(&bar.w_full[slot], (uint32_t)LIN_W_BYTES);
          tma_load_3d(sW + (size_t)slot * LIN_W_BYTES, &maps.w[gi], 0, tile * LIN_MT, split * g.kc + j,
                      &bar.w_full[slot]);
        }
      }
      // no copy of this CTA may still be in flight when it exits
      for (int i = max(k - NS, 0); i < k; ++i) mbar_wait_bounded(&bar.w_full[i % NS], (i / NS) & 1, K_BLOCK_TAIL, 7);
      TAIL_MARK(30);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(LIN_MT, p.BN, BF, false);
      const uint32_t aW = smem_u32(sW), aA = smem_u32(sA);
      int k = 0;  // K blocks consumed
      bool ok = true;
      for (int u = 0; ok && u < NU; ++u) {
        if (!(ok = mbar_wait_or_abort(&bar.act_full, u & 1, &bar.abort_flag, 2))) break;
        const int kc = p.g[bar.u_gemm[u]].kc;
        for (int j = 0; j < kc; ++j, ++k) {
          const int slot = k % NS;
          if (!(ok = mbar_wait_or_abort(&bar.w_full[slot], (k / NS) & 1, &bar.abort_flag, 3))) break;
          tc_fence_after();
          const uint32_t wa = aW + slot * LIN_W_BYTES, xa = aA + j * p.BN * 128;
#pragma unroll
          for (int kk = 0; kk < LIN_KB / 16; ++kk)
            umma_f16(bar.tmem_base, sw128_desc(wa + kk * 32, 16, 1024), sw128_desc(xa + kk * 32, 16, 1024), idesc,
                     j > 0 || kk > 0);
          umma_commit(&bar.w_empty[slot]);  // the slot is free once these MMAs have read it
        }
        if (ok) umma_commit(&bar.mma_done);
      }
      if (!ok) atomicExch(&bar.abort_flag, 1);
      umma_commit(&bar.fin);
      mbar_wait_bounded(&bar.fin, 0, K_BLOCK_TAIL, 4);  // every MMA of this CTA has completed
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ workers (warps 0-3)
    pdl_wait();  // the attention output and the residual come from the grids this one follows
    if (tid == 0) TAIL_MARK(1);
    const uint32_t lane_base = bar.tmem_base + ((uint32_t)(warp * 32) << 16);
    const int fl = warp * 32 + lane;  // this thread's output feature in a unit's tile (its TMEM lane)
    const int F = p.g[TG_FC].N;
    const int Tf = F / LIN_MT;
    int* fc_cnt = p.sync + TW_FIXED;
    int* fc_ready = fc_cnt + Tf;
    int* q_cnt = fc_ready + Tf;
    bool alive = NU > 0 || bar.nu == 0;
    int u = 0;
    // layer-norm rows of this CTA: r = (cta - off_ln) mod G, + G, ...
    const int r0 = ((cta - p.off_ln) % G + G) % G;
    int nrows = 0, n_ln = 0;
    for (int r = r0; r < p.B; r += G) ++nrows;

    for (int ph = 0; ph < 4 && alive; ++ph) {
      if (ph == TG_FC || ph == TG_QKV) {
        // P2 (ln_2) before the fc units, P5 (ln_next) before the qkv units
        const bool first = ph == TG_FC;
        if (nrows > 0) {
          if (!(alive = tail_wait(p, p.sync + (first ? TW_PROJ : TW_MLP), 1, p.g[first ? TG_PROJ : TG_MLP].n,
                                  first ? 10 : 11)))
            break;
          if (tid == 0) TAIL_MARK(first ? 22 : 24);
          for (int r = r0; alive && r < p.B; r += G, ++n_ln)
            alive = tail_ln_row<T>(p, bar, reinterpret_cast<float*>(sA), n_ln & 1, r,
                                   first ? p.part_proj : p.part_mlp, p.g[first ? TG_PROJ : TG_MLP].S,
                                   first ? p.ln2 : p.ln_next, reinterpret_cast<T*>(first ? p.h2 : p.h));
          if (!alive) break;
          tail_signal(p.sync + (first ? TW_LN2 : TW_LN1), nrows);
          if (tid == 0) TAIL_MARK(first ? 23 : 25);
        }
      }
      const TailGemm& g = p.g[ph];
      for (; alive && u < NU && bar.u_gemm[u] == ph; ++u) {
        const int tile = bar.u_id[u] / g.S, split = bar.u_id[u] % g.S;
        const int kb0 = split * g.kc;
        // ---- what this unit reads must be complete
        if (ph == TG_FC) {
          if (!(alive = tail_wait(p, p.sync + TW_LN2, 1, p.B, 12))) break;
        } else if (ph == TG_MLP) {
          const int t_lo = (kb0 * 64) / LIN_MT, t_hi = ((kb0 + g.kc) * 64 - 1) / LIN_MT;
          if (!(alive = tail_wait(p, fc_ready + t_lo, t_hi - t_lo + 1, 1, 13))) break;
        } else if (ph == TG_QKV) {
          if (!(alive = tail_wait(p, p.sync + TW_LN1, 1, p.B, 14))) break;
        }
        // ---- the unit's rows: one TMA copy per K block of its slice (att, h2, fc or h) into the stage, issued by
        // the four worker warps in turn (an SM moves more bytes at once when several warps issue copies)
        if (tid == 0) {
          TAIL_MARK(2 + ph * 5);
          mbar_arrive_expect_tx(&bar.act_full, (uint32_t)(g.kc * p.BN * 128));
        }
        named_bar_sync(1, 128);
        if (lane == 0) {
          fence_proxy_async_global();  // rows other CTAs stored, observed through the counter above
          fence_proxy_async_smem();    // the stage was last read / written by the workers (generic proxy)
          for (int j = warp; j < g.kc; j += 4)
            tma_load_3d(sA + (size_t)j * p.BN * 128, &maps.a[ph], 0, 0, kb0 + j, &bar.act_full);
        }
        if (tid == 0) TAIL_MARK(3 + ph * 5);
        const bool waited = mbar_wait_or_abort(&bar.mma_done, u & 1, &bar.abort_flag, 5);
        if (named_bar_or(1, 128, !waited)) {
          if (tid == 0) atomicExch(&bar.abort_flag, 1);
          alive = false;
          break;
        }
        tc_fence_after();
        if (tid == 0) TAIL_MARK(4 + ph * 5);
        // ---- the accumulator (thread = output feature, columns = rows) into a row-major fp32 tile [BN][128] in
        // the stage (its rows were consumed by the MMAs that just completed)
        float* tl = reinterpret_cast<float*>(sA);
#pragma unroll
        for (int c0 = 0; c0 < MAXC; c0 += 32)
          if (c0 < p.BN) {
            float v[32];
            tmem_ld32(lane_base + c0, v);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c0 + i < p.BN) tl[(c0 + i) * LIN_MT + fl] = v[i];  // the tile holds BN rows
          }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (tid == 0) TAIL_MARK(27);
        const int f0 = tile * LIN_MT;
        if (ph == TG_PROJ || ph == TG_MLP) {
          // ---- fp32 partial sums of this K slice: part[split, b, f0 ..], 16-byte pieces
          float* dst = (ph == TG_PROJ ? p.part_proj : p.part_mlp) + (int64_t)split * p.B * g.N + f0;
          for (int id = tid; id < p.B * (LIN_MT / 4); id += 128) {
            const int r = id >> 5, c = (id & 31) * 4;
            *reinterpret_cast<float4*>(dst + (int64_t)r * g.N + c) = *reinterpret_cast<const float4*>(tl + r * LIN_MT + c);
          }
          if (tid == 0) TAIL_MARK(28);
          tail_signal(p.sync + (ph == TG_PROJ ? TW_PROJ : TW_MLP), 1);
        } else {
          // ---- c_fc (+ GELU) / c_attn: with K splits every split leaves its tile in the workspace and the tile's
          // last split to arrive adds them all in split order
          bool write = true;
          if (g.S > 1) {
            const int n4 = p.BN * (LIN_MT / 4);
            float4* ws = reinterpret_cast<float4*>((ph == TG_FC ? p.ws_fc : p.ws_qkv) +
                                                   (int64_t)tile * g.S * p.BN * LIN_MT);
            for (int id = tid; id < n4; id += 128) ws[(int64_t)split * n4 + id] = reinterpret_cast<const float4*>(tl)[id];
            named_bar_sync(1, 128);
            bool last = false;
            if (tid == 0)  // release this split's sums, acquire the others' (the counter is zeroed at exit)
              last = atom_add_acq_rel_gpu((ph == TG_FC ? fc_cnt : q_cnt) + tile, 1) == g.S - 1;
            write = named_bar_or(1, 128, last);
            if (write) {
              constexpr int U = 8;
              for (int id0 = tid; id0 < n4; id0 += 128 * U) {
                float4 a[U];
#pragma unroll
                for (int e = 0; e < U; ++e) a[e] = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int sp = 0; sp < g.S; ++sp) {
                  float4 q[U];
#pragma unroll
                  for (int e = 0; e < U; ++e) {
                    const int id = id0 + e * 128;
                    if (id < n4)
                      q[e] = sp == split ? reinterpret_cast<const float4*>(tl)[id] : __ldcg(ws + (int64_t)sp * n4 + id);
                  }
#pragma unroll
                  for (int e = 0; e < U; ++e) {
                    a[e].x += q[e].x; a[e].y += q[e].y; a[e].z += q[e].z; a[e].w += q[e].w;
                  }
                }
#pragma unroll
                for (int e = 0; e < U; ++e)
                  if (id0 + e * 128 < n4) reinterpret_cast<float4*>(tl)[id0 + e * 128] = a[e];
              }
              named_bar_sync(1, 128);
            }
          }
          if (write) {
            // 8 features of a row per thread: rounded to T, GELU'd (c_fc) and rounded again, one 16-byte store
            T* out = reinterpret_cast<T*>(ph == TG_FC ? p.fc : p.qkv) + f0;
            for (int id = tid; id < p.B * (LIN_MT / 8); id += 128) {
              const int r = id >> 4, c = (id & 15) * 8;
              const float4 lo = *reinterpret_cast<const float4*>(tl + r * LIN_MT + c);
              const float4 hi = *reinterpret_cast<const float4*>(tl + r * LIN_MT + c + 4);
              float o[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                o[e] = to_f32(from_f32<T>(o[e]));
                if (ph == TG_FC) o[e] = gelu_erf(o[e]);
              }
              store_vec_from_f32<T>(out + (int64_t)r * g.N + c, o);
            }
            if (tid == 0) TAIL_MARK(28);
            if (ph == TG_FC) tail_signal(fc_ready + tile, 1);
          }
        }
        if (tid == 0) TAIL_MARK(5 + ph * 5);
      }
    }
    if (tid == 0) TAIL_MARK(26);
    if (!alive && tid == 0) {
      atomicExch(&bar.abort_flag, 1);
      atomicExch(p.sync + TW_ABORT, 1);  // the other CTAs' waits end now instead of at their limits
    }
    // ---- leave: the last CTA out zeroes the sync words for the next launch
    named_bar_sync(1, 128);
    if (tid == 0) {
      __threadfence();
      if (atomicAdd(p.sync + TW_EXIT, 1) == G - 1) {
        for (int i = 0; i < p.nsync; ++i) p.sync[i] = 0;
        __threadfence();
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

}  // namespace ta
