// Tensor-core tile kernel for segment-tree sparse attention over whole sequences (prefill): the key assembly +
// dedupe + sparse attention of SegAttention.sparse_attend (fastseg.py:367-383, static keys 372-381,
// dedupe_fast 227-234, _attn_fwd 49-78) for 128 queries at a time.
//
// One CTA owns the 128 queries [q0, q0 + 128) of one (b, h). Every query has its own key set - the positions of
// its used leaf blocks that lie before its window, the sink (position 0) and the window [t - Lw + 1, t] - so the
// CTA streams the UNION of those sets in 64-key tiles and masks each query's row:
//   key tile list : a shared-memory bitmap over 64-key tiles (used leaves of any query, the window tiles, tile 0)
//   per query     : a leaf bitmap (bit m = leaf m used); the mask of key p is
//                   (w0 <= p <= t) || p == 0 || (p < w0 && leaf bit p >> L0)      (w0 = max(t - Lw + 1, 0))
//                   which is exactly the deduplicated key set of the reference (every position once).
// Warp roles (192 threads):
//   warps 0-3  softmax: thread r owns query row r = TMEM lane r. Reads S = Q K^T of a tile from TMEM, masks,
//              softmax in the log2 domain against a per-row reference max, writes P (16-bit, 128-byte-swizzled
//              K-major) to shared memory. The reference max moves only when a tile's max exceeds it by more than
//              TAU (P then stays below 2^TAU); only then does the warp wait for the last P V and rescale its O rows
//              in TMEM. The output row is read from TMEM once, at the end.
//   warp 4     TMA producer: the Q tile once, then K and V tiles into an NS-stage ring.
//   warp 5     allocates TMEM; one thread issues tcgen05.mma: S(n) = Q K(n)^T into S[n % 2], then
//              O += P(n-1) V(n-1) into the one O accumulator, committing to mbarriers.
// Every wait is a bounded mbarrier wait; on a timeout the CTA records the error, stops, waits (bounded) for its
// copies and MMAs in flight and frees its TMEM.
#pragma once
#include <type_traits>
#include "attn.cuh"
#include "tc.cuh"

namespace ta {

constexpr int PF_QT = 128;                // queries per CTA tile (TMEM lanes, MMA M)
constexpr int PF_KT = 64;                 // keys per key tile (MMA N of S, K of P V)
constexpr int PF_MAX_LEAF_WORDS = 32;     // per-query leaf bitmap: at most 1024 leaves
constexpr int PF_MAX_TILE_WORDS = 512;    // key-tile bitmap: at most 16384 tiles (T_kv <= 2^20)
constexpr int PF_THREADS = 192;

struct PrefillParams {
  const int64_t* tq;
  int64_t tq_sb, tq_st;
  const int64_t* ids;     // (B,H,Nq,wl) leaf ids, best first
  const uint8_t* vld;     // (B,H,Nq,wl)
  const int64_t* n_tree;  // (B,H,Nq) or null -> ntree_const
  int ntree_const;
  int B, H, Nq, wl, L0, Lw, T_kv;
  int n_qtiles, leaf_words, tile_words;
  float scale_log2;       // softmax scale * log2(e)
  void* o;                // (B,H,Nq,dh) with strides
  int64_t o_sb, o_sh, o_st;
  float* lse;             // natural-log LSE (B,H,Nq), may be null
  int32_t* nkeys;         // keys attended (B,H,Nq), may be null
};

template <int DH, int NS>
struct PfCfg {
  static constexpr int NHALF = DH / 64;                 // 128-byte column blocks of a 16-bit row
  static constexpr int Q_BYTES = PF_QT * DH * 2;        // Q tile
  static constexpr int KT_BYTES = PF_KT * DH * 2;       // one K or V tile
  static constexpr int STAGE_BYTES = 2 * KT_BYTES;      // K then V
  static constexpr int P_BYTES = PF_QT * PF_KT * 2;     // one P buffer
  static constexpr int TM_S = 0;                        // TMEM columns: S[2] (64 each) then the O accumulator
  static constexpr int TM_O = 2 * PF_KT;
  static constexpr int TM_COLS = (2 * PF_KT + DH) <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC_QK_BF16 = umma_idesc_f16(PF_QT, PF_KT, true, false);
  static constexpr uint32_t IDESC_QK_F16 = umma_idesc_f16(PF_QT, PF_KT, false, false);
  static constexpr uint32_t IDESC_PV_BF16 = umma_idesc_f16(PF_QT, DH, true, true);
  static constexpr uint32_t IDESC_PV_F16 = umma_idesc_f16(PF_QT, DH, false, true);
  static constexpr size_t fixed_bytes() { return (size_t)Q_BYTES + (size_t)NS * STAGE_BYTES + 2 * (size_t)P_BYTES; }
};

template <int NS>
struct PfBars {
  uint64_t q_full, mma_done;
  uint64_t kv_full[NS], kv_empty[NS];
  uint64_t s_full[2], s_free[2], p_full[2], o_full[2];  // o_full[j % 2]: P(j) V(j) has been added to O
  uint32_t tmem_base;
  int abort_flag;
};

template <int DH, int NS>
__host__ __device__ inline size_t prefill_smem_bytes(int leaf_words, int tile_words) {
  return 1024 + PfCfg<DH, NS>::fixed_bytes() + (size_t)PF_QT * leaf_words * 4 + (size_t)tile_words * 4 + 16 +
         sizeof(PfBars<NS>);
}

// Walks the set bits of the key-tile bitmap in increasing order (each role keeps its own cursor).
struct TileIter {
  const uint32_t* bits;
  int nw, w;
  uint32_t cur;
  __device__ __forceinline__ TileIter(const uint32_t* b, int n) : bits(b), nw(n), w(0), cur(n > 0 ? b[0] : 0u) {}
  __device__ __forceinline__ int next() {
    while (cur == 0u) {
      if (++w >= nw) return -1;
      cur = bits[w];
    }
    const int bit = __ffs(cur) - 1;
    cur &= cur - 1u;
    return w * 32 + bit;
  }
};

// Set bits [a, c] (inclusive) of a shared bitmap.
__device__ __forceinline__ void bitmap_set_range(uint32_t* bits, int a, int c) {
  for (int w = a >> 5; w <= (c >> 5); ++w) {
    const int lo = max(a - w * 32, 0), hi = min(c - w * 32, 31);
    const uint32_t m = (hi == 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u);
    atomicOr(&bits[w], m);
  }
}

// Mask of positions [lo, hi] (0 <= lo <= hi <= 63) of a 64-key tile.
__device__ __forceinline__ uint64_t range_mask64(int lo, int hi) {
  const uint64_t upto = hi == 63 ? ~0ull : ((1ull << (hi + 1)) - 1ull);
  return upto & ~((1ull << lo) - 1ull);
}

// 2^x by the hardware's approximate base-2 exponential (ex2.approx.ftz: 2^-inf = 0, relative error ~2^-22,
// below the 16-bit rounding of P that follows).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

template <typename T, int DH, int NS>
__global__ void __launch_bounds__(PF_THREADS, DH == 64 ? 2 : 1)
    prefill_tile_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, PrefillParams p) {
  using C = PfCfg<DH, NS>;
  using Bars = PfBars<NS>;
  constexpr bool BF = sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_QK = BF ? C::IDESC_QK_BF16 : C::IDESC_QK_F16;
  constexpr uint32_t IDESC_PV = BF ? C::IDESC_PV_BF16 : C::IDESC_PV_F16;

  extern __shared__ unsigned char pf_smem_raw[];
  const uint32_t raw_a = smem_u32(pf_smem_raw);
  unsigned char* base = pf_smem_raw + (((raw_a + 1023u) & ~1023u) - raw_a);
  unsigned char* sQ = base;
  unsigned char* sKV = sQ + C::Q_BYTES;
  unsigned char* sP = sKV + NS * C::STAGE_BYTES;
  uint32_t* qbits = reinterpret_cast<uint32_t*>(sP + 2 * C::P_BYTES);
  uint32_t* tbits = qbits + PF_QT * p.leaf_words;
  int* tmeta = reinterpret_cast<int*>(tbits + p.tile_words);  // [0] = number of key tiles
  Bars& bar = *reinterpret_cast<Bars*>(reinterpret_cast<unsigned char*>(tmeta) + 16 -
                                       (reinterpret_cast<uintptr_t>(tmeta) & 7u));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nbh = p.B * p.H;
  const int qt = p.n_qtiles - 1 - (int)(blockIdx.x / nbh);  // late (heavier) query tiles first
  const int bh = (int)(blockIdx.x % nbh);
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qt * PF_QT;
  const int L0 = p.L0;

  // ---------------------------------------------------------------- set-up
  if (tid == 0) {
    mbar_init(&bar.q_full, 1);
    mbar_init(&bar.mma_done, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bar.kv_full[s], 1);
      mbar_init(&bar.kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar.s_full[s], 1);
      mbar_init(&bar.s_free[s], 4);
      mbar_init(&bar.p_full[s], 4);
      mbar_init(&bar.o_full[s], 1);
    }
    bar.abort_flag = 0;
    tmeta[0] = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < p.tile_words; i += PF_THREADS) tbits[i] = 0u;
  if (warp < 4)
    for (int i = 0; i < p.leaf_words; ++i) qbits[i * PF_QT + tid] = 0u;
  if (warp == 4 && lane == 0) {
    tma_prefetch_map(&tm_q);
    tma_prefetch_map(&tm_k);
    tma_prefetch_map(&tm_v);
  }
  if (warp == 5) {
    tmem_alloc(&bar.tmem_base, C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // this thread's query (softmax warps)
  const int qi = q0 + tid;
  const int64_t qid = (int64_t)bh * p.Nq + qi;
  int t = -1, w0 = 0;
  if (warp < 4 && qi < p.Nq) {
    const int64_t tt = p.tq[b * p.tq_sb + (int64_t)qi * p.tq_st];
    if (tt < 0 || tt >= p.T_kv) {
      record_error(DEV_POS_RANGE, K_PREFILL, (int)tt, p.T_kv);
    } else {
      t = (int)tt;
      w0 = max(t - p.Lw + 1, 0);
      const int ntree = p.n_tree ? (int)p.n_tree[qid] : p.ntree_const;
      const int64_t sb = qid * p.wl;
      const int64_t leaf = 1ll << L0;
      uint32_t* qb = qbits + tid;  // word i of this query's leaf bitmap at qb[i * PF_QT] (conflict-free)
      for (int i = 0; i < p.wl && i < ntree; ++i) {
        if (!p.vld[sb + i]) continue;
        const int64_t m = p.ids[sb + i];
        if (m < 0 || m * leaf >= (int64_t)w0) continue;  // only the part before the window counts
        qb[(m >> 5) * PF_QT] |= 1u << (m & 31);
        const int a = (int)(m * leaf), c = (int)min(m * leaf + leaf, (int64_t)w0) - 1;
        bitmap_set_range(tbits, a >> 6, c >> 6);
      }
      bitmap_set_range(tbits, w0 >> 6, t >> 6);  // window
      if (w0 > 0) atomicOr(&tbits[0], 1u);        // sink
    }
  }
  __syncthreads();
  if (warp == 0) {
    int cnt = 0;
    for (int i = lane; i < p.tile_words; i += 32) cnt += __popc(tbits[i]);
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) tmeta[0] = cnt;
  }
  __syncthreads();
  const int ntiles = tmeta[0];

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    int issued = 0;
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(&bar.q_full, (uint32_t)C::Q_BYTES);
#pragma unroll
      for (int hh = 0; hh < C::NHALF; ++hh) tma_load_4d(sQ + hh * (PF_QT * 128), &tm_q, hh * 64, q0, h, b, &bar.q_full);
      TileIter it(tbits, p.tile_words);
      for (int kt; (kt = it.next()) >= 0; ++issued) {
        const int s = issued % NS;
        if (issued >= NS && !mbar_wait_bounded(&bar.kv_empty[s], ((issued / NS) - 1) & 1, K_PREFILL, 20)) {
          atomicExch(&bar.abort_flag, 1);
          break;
        }
        if (*reinterpret_cast<volatile int*>(&bar.abort_flag)) break;
        unsigned char* st = sKV + s * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&bar.kv_full[s], (uint32_t)C::STAGE_BYTES);
#pragma unroll
        for (int hh = 0; hh < C::NHALF; ++hh) {
          tma_load_4d(st + hh * (PF_KT * 128), &tm_k, hh * 64, kt * PF_KT, h, b, &bar.kv_full[s]);
          tma_load_4d(st + C::KT_BYTES + hh * (PF_KT * 128), &tm_v, hh * 64, kt * PF_KT, h, b, &bar.kv_full[s]);
        }
      }
      // no copy of this CTA may still be in flight when it exits
      mbar_wait_bounded(&bar.q_full, 0, K_PREFILL, 21);
      for (int i = max(issued - NS, 0); i < issued; ++i)
        mbar_wait_bounded(&bar.kv_full[i % NS], (i / NS) & 1, K_PREFILL, 22);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t tS = bar.tmem_base + C::TM_S, tO = bar.tmem_base + C::TM_O;
      const uint32_t aQ = smem_u32(sQ), aKV = smem_u32(sKV), aP = smem_u32(sP);
      bool ok = mbar_wait_bounded(&bar.q_full, 0, K_PREFILL, 23);
      auto issue_pv = [&](int j) -> bool {
        // P(j) written (and any rescale of O the softmax warps made before it, ordered by their arrival)
        if (!mbar_wait_bounded(&bar.p_full[j & 1], (j >> 1) & 1, K_PREFILL, 24)) return false;
        tc_fence_after();
        const uint32_t pa = aP + (j & 1) * C::P_BYTES;
        const uint32_t va = aKV + (j % NS) * C::STAGE_BYTES + C::KT_BYTES;
#pragma unroll
        for (int k = 0; k < PF_KT / 16; ++k)
          umma_f16(tO, sw128_desc(pa + k * 32, 16, 1024), sw128_desc(va + k * 2048, PF_KT * 128, 1024), IDESC_PV,
                   j > 0 || k > 0);
        umma_commit(&bar.o_full[j & 1]);
        umma_commit(&bar.kv_empty[j % NS]);
        return true;
      };
      int n = 0;
      for (; ok && n < ntiles; ++n) {
        const int s = n % NS;
        if (!(ok = mbar_wait_bounded(&bar.kv_full[s], (n / NS) & 1, K_PREFILL, 26))) break;
        if (n >= 2 && !(ok = mbar_wait_bounded(&bar.s_free[n & 1], ((n >> 1) - 1) & 1, K_PREFILL, 27))) break;
        if (*reinterpret_cast<volatile int*>(&bar.abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = aKV + s * C::STAGE_BYTES;
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) {
          const uint32_t off = (k >> 2) * (PF_QT * 128) + (k & 3) * 32;   // Q: 128-row blocks of 64 columns
          const uint32_t koff = (k >> 2) * (PF_KT * 128) + (k & 3) * 32;  // K: 64-row blocks of 64 columns
          umma_f16(tS + (n & 1) * PF_KT, sw128_desc(aQ + off, 16, 1024), sw128_desc(ka + koff, 16, 1024), IDESC_QK,
                   k > 0);
        }
        umma_commit(&bar.s_full[n & 1]);
        if (n >= 1 && !(ok = issue_pv(n - 1))) break;
      }
      if (ok && n == ntiles) ok = issue_pv(ntiles - 1);
      if (!ok) atomicExch(&bar.abort_flag, 1);
      umma_commit(&bar.mma_done);
      mbar_wait_bounded(&bar.mma_done, 0, K_PREFILL, 28);  // every MMA of this CTA has completed
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax warps (thread = query row)
    const uint32_t lane_base = bar.tmem_base + ((uint32_t)(warp * 32) << 16);
    // a row's weights are p = 2^(s * scale_log2 - m_ref); m_ref follows the row's running max lazily: it moves to a
    // tile's max only when that exceeds it by more than TAU, so p < 2^TAU (far inside the 16-bit and fp32 ranges)
    constexpr float TAU = 8.f;
    float m_ref = -INFINITY, l_run = 0.f;
    int keys = 0;
    bool ok = true;
    unsigned char* prow_base = sP + (tid >> 3) * 1024 + (tid & 7) * 128;
    const uint32_t* qb = qbits + tid;
    // warp-uniform: every lane waits for the same phase
    auto pv_done = [&](int j, int where) -> bool {
      return __all_sync(0xffffffffu, mbar_wait_bounded(&bar.o_full[j & 1], (j >> 1) & 1, K_PREFILL, where));
    };

    TileIter it(tbits, p.tile_words);
    int n = 0;
    for (int kt; ok && (kt = it.next()) >= 0; ++n) {
      if (!(ok = __all_sync(0xffffffffu, mbar_poll_bounded(&bar.s_full[n & 1], (n >> 1) & 1, K_PREFILL, 31)))) break;
      tc_fence_after();
      float s[64];
      {
        float v[32];
        tmem_ld32(lane_base + C::TM_S + (n & 1) * PF_KT, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = v[i];
        tmem_ld32(lane_base + C::TM_S + (n & 1) * PF_KT + 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 + i] = v[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.s_free[n & 1]);

      // mask of this query over the tile's 64 positions
      const int P0 = kt * PF_KT;
      uint64_t vm = 0ull;
      if (t >= 0) {
        if (t >= P0 && w0 <= P0 + 63) vm |= range_mask64(max(w0, P0) - P0, min(t, P0 + 63) - P0);
        if (P0 == 0) vm |= 1ull;  // sink
        if (P0 < w0) {
          uint64_t lm;
          if (L0 >= 6) {
            const int m = P0 >> L0;
            lm = ((qb[(m >> 5) * PF_QT] >> (m & 31)) & 1u) ? ~0ull : 0ull;
          } else {
            const int m0 = P0 >> L0, nb = 64 >> L0;  // leaves of this tile (L0 >= 1: nb <= 32, in one word)
            const uint32_t field = (qb[(m0 >> 5) * PF_QT] >> (m0 & 31)) & (nb == 32 ? 0xffffffffu : ((1u << nb) - 1u));
            lm = 0ull;
            for (int i = 0; i < nb; ++i)
              if ((field >> i) & 1u) lm |= range_mask64(i << L0, ((i + 1) << L0) - 1);
          }
          const int lim = w0 - P0;
          if (lim < 64) lm &= (1ull << lim) - 1ull;
          vm |= lm;
        }
      }
      keys += __popcll(vm);
      // warp-uniform shortcut: a tile masked for all 32 queries of the warp contributes nothing (its P rows are
      // zero and the reference max is unchanged)
      const bool none = __all_sync(0xffffffffu, vm == 0ull);
      float mt = -INFINITY;  // this tile's max in the log2 domain
      if (!none) {
        // max over the raw scores (scaling by a positive constant is monotone under rounding: max commutes)
        // (four independent chains: the max is exact in any order)
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] = ((vm >> i) & 1ull) ? s[i] : -INFINITY;
          m4[i & 3] = fmaxf(m4[i & 3], s[i]);
        }
        mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
      }
      const bool bump = mt > m_ref + TAU;            // a new reference (never for a masked row)
      const bool resc = bump && m_ref != -INFINITY;  // O and l hold weights of the old reference
      const float m_new = bump ? mt : m_ref;
      const float f = resc ? ex2_approx(m_ref - m_new) : 1.f;
      if (__any_sync(0xffffffffu, resc)) {
        // rescale this warp's O rows once the last P V has landed in them (factor 1 for the other lanes)
        if (n >= 1 && !(ok = pv_done(n - 1, 30))) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DH / 32; ++c) {
          float v[32];
          tmem_ld32(lane_base + C::TM_O + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= f;
          tmem_st32(lane_base + C::TM_O + c * 32, v);
        }
        tmem_wait_st();
        tc_fence_before();
      }
      l_run *= f;
      m_ref = m_new;
      // P buffer n % 2 was last read by P(n-2) V(n-2)
      if (n >= 2 && !(ok = pv_done(n - 2, 32))) break;
      unsigned char* prow = prow_base + (n & 1) * C::P_BYTES;
      if (none) {
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(prow + ((c ^ (tid & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
      } else {
        const float mu = m_ref == -INFINITY ? 0.f : m_ref;
        // P row (16-bit, rounded for the tensor-core P.V) into the swizzled K-major P buffer; the denominator l sums
        // the fp32 weights p = 2^(s * scale_log2 - mu) (the scaling fused into one FMA), as the reference's _attn_fwd
        // sums them, in four independent chains
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = ex2_approx(fmaf(s[c * 8 + 2 * e], p.scale_log2, -mu));
            const float p1 = ex2_approx(fmaf(s[c * 8 + 2 * e + 1], p.scale_log2, -mu));
            l4[e] += p0 + p1;
            w[e] = pack2<T>(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + ((c ^ (tid & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_run += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.p_full[n & 1]);
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&bar.abort_flag) != 0)) { ok = false; break; }
    }
    // the output row: O / l once the last P V has landed
    if (ok && n > 0) ok = pv_done(n - 1, 33);
    if (!ok) atomicExch(&bar.abort_flag, 1);
    if (ok && n > 0) {
      tc_fence_after();
      const float fin = l_run > 0.f ? 1.f / l_run : 0.f;
      T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + (int64_t)qi * p.o_st;
#pragma unroll
      for (int c = 0; c < DH / 32; ++c) {
        float v[32];
        tmem_ld32(lane_base + C::TM_O + c * 32, v);  // the whole warp (a lane without a query discards its row)
        if (t >= 0) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            float v8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v8[e] = v[q8 * 8 + e] * fin;
            if constexpr (sizeof(T) == 2) store_vec_from_f32<T>(orow + c * 32 + q8 * 8, v8);
          }
        }
      }
    }
    if (t >= 0) {
      if (!(ok && n > 0)) {  // nothing attended (a failed launch): zero rows
        T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + (int64_t)qi * p.o_st;
        float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < DH / 8; ++c)
          if constexpr (sizeof(T) == 2) store_vec_from_f32<T>(orow + c * 8, z);
      }
      if (p.lse) p.lse[qid] = l_run > 0.f ? (m_ref + log2f(l_run)) * LN2 : -INFINITY;
      if (p.nkeys) p.nkeys[qid] = keys;
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(bar.tmem_base, C::TM_COLS);
  }
}

}  // namespace ta
