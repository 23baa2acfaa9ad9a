// C ABI of the treeattn_b200 kernels: argument checks, launch shapes, dispatch over dtype x head dim.
// Single translation unit: every kernel header is included here.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "../../include/treeattn_b200.h"
#include <cudaTypedefs.h>

#include "block.cuh"
#include "decode.cuh"
#include "dyn.cuh"
#include "forest.cuh"
#include "linear.cuh"
#include "model_ops.cuh"
#include "prefill.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return TA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// a row of dh elements of `esize` bytes read in 16-byte chunks: base and every stride must keep 16-byte
// alignment
bool rows_aligned(const void* base, int esize, std::initializer_list<int64_t> strides) {
  if (!aligned16(base)) return false;
  for (int64_t s : strides)
    if ((s * esize) % 16 != 0) return false;
  return true;
}

int esize_of(int dtype) { return dtype == TA_F32 ? 4 : 2; }

bool valid_dtype(int dtype) { return dtype == TA_F32 || dtype == TA_BF16 || dtype == TA_F16; }

bool valid_dh(int dh) { return dh == 16 || dh == 32 || dh == 64 || dh == 128; }

cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Per-device state of one launcher. cudaFuncSetAttribute and the occupancy and SM-count queries answer for the
// current device only, so a process that drives several GPUs keeps one entry per device (the first 64 devices
// are cached; others are asked again on every call).
constexpr int kDevCache = 64;

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  return dev;
}

// The dynamic shared-memory size a call site has allowed for its kernel, per device (0 = not yet).
struct SmemAttr {
  std::atomic<size_t> bytes[kDevCache];
};

// Allow `bytes` of dynamic shared memory for kern on the current device. The attribute is always set to the most
// the device gives one block beside the kernel's static shared memory: a kernel launched from several call sites
// (or launcher instantiations) then never has its limit lowered by one of them under another's launch.
template <typename K>
int allow_smem(SmemAttr& a, K* kern, size_t bytes, const char* what) {
  const int dev = current_device();
  const bool cached = dev >= 0 && dev < kDevCache;
  if (cached) {
    const size_t have = a.bytes[dev].load(std::memory_order_relaxed);
    if (have >= bytes) return TA_OK;
    if (have != 0) return fail(TA_ERR_ARG, "%s: %zu B of dynamic shared memory, above the %zu B a block can have",
                               what, bytes, have);
  }
  int optin = 0;
  cudaFuncAttributes fa;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev < 0 ? 0 : dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, kern) != cudaSuccess)
    return check_launch(what);
  const size_t most = (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
  if (bytes > most)
    return fail(TA_ERR_ARG, "%s: %zu B of dynamic shared memory, above the %zu B a block can have", what, bytes, most);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)most) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    return fail(TA_ERR_CUDA, "%s: dynamic shared memory limit of %zu B refused: %s", what, most, cudaGetErrorString(e));
  }
  if (cached) a.bytes[dev].store(most, std::memory_order_relaxed);
  return TA_OK;
}

// Launch with programmatic stream serialization: the kernel may start while the previous kernel of the stream is
// still running (it calls griddepcontrol.wait before reading anything that kernel writes).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Dispatch F<T, DH>::run(args...) over the runtime dtype and head dim.
template <template <typename, int> class F, typename T, typename... Args>
int by_dh(int dh, Args&&... args) {
  switch (dh) {
    case 16: return F<T, 16>::run(args...);
    case 32: return F<T, 32>::run(args...);
    case 64: return F<T, 64>::run(args...);
    case 128: return F<T, 128>::run(args...);
    default: return fail(TA_ERR_ARG, "unsupported head dim %d (16, 32, 64, 128)", dh);
  }
}

template <template <typename, int> class F, typename... Args>
int by_type_dh(int dtype, int dh, Args&&... args) {
  switch (dtype) {
    case TA_F32: return by_dh<F, float>(dh, args...);
    case TA_BF16: return by_dh<F, __nv_bfloat16>(dh, args...);
    case TA_F16: return by_dh<F, __half>(dh, args...);
    default: return fail(TA_ERR_ARG, "unsupported dtype code %d", dtype);
  }
}

int check_levels(int cap, int L0, int Lm) {
  if (cap <= 0) return fail(TA_ERR_ARG, "capacity must be positive (got %d)", cap);
  if (L0 < 1 || L0 > 12) return fail(TA_ERR_ARG, "leaf level L0=%d outside [1, 12]", L0);
  if (Lm < L0 || Lm > 30) return fail(TA_ERR_ARG, "top level Lm=%d outside [L0=%d, 30]", Lm, L0);
  return TA_OK;
}

ta::LevelView make_lv(const float* nodes, int64_t n_sb, int64_t n_sh, int cap, int L0, int Lm) {
  ta::LevelView lv{};
  lv.nodes = nodes;
  lv.s_b = n_sb;
  lv.s_h = n_sh;
  lv.cap = cap;
  lv.L0 = L0;
  lv.Lm = Lm;
  ta::level_offsets(cap, L0, Lm, lv.off);
  return lv;
}

// ------------------------------------------------------------------------------------------------ launchers
template <typename T, int DH>
struct BuildLevels {
  static int run(const void* k, int B, int H, int T_len, int64_t k_sb, int64_t k_sh, int64_t k_st, int cap, int L0,
                 int Lm, int zero_sink, float* nodes, int64_t n_sb, int64_t n_sh, cudaStream_t st,
                 bool logmag = false) {
    const ta::LevelView lv = make_lv(nodes, n_sb, n_sh, cap, L0, Lm);
    const int n_leaf = T_len >> L0;
    const int64_t total = (int64_t)B * H * n_leaf * DH;
    if (total > 0) {
      const int threads = 256;
      auto kern = logmag ? ta::build_leaf_level_kernel<T, true> : ta::build_leaf_level_kernel<T, false>;
      kern<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(
          reinterpret_cast<const T*>(k), k_sb, k_sh, k_st, H, T_len, DH, L0, nodes + (int64_t)lv.off[L0] * DH, n_sb,
          n_sh, n_leaf, total, zero_sink);
      if (int r = check_launch("ta_build_levels(leaf)")) return r;
    }
    if (Lm > L0 && n_leaf > 1) {
      // one CTA per (b, h) in shared memory (the leaf level and the level being formed) when it fits and the node
      // rows are 16-byte aligned, else one thread per (b, h, dim) walking the levels
      const size_t smem = (size_t)2 * n_leaf * DH * sizeof(float);
      const bool aligned = (reinterpret_cast<uintptr_t>(nodes) & 15u) == 0 && (n_sb * 4) % 16 == 0 &&
                           (n_sh * 4) % 16 == 0;
      if (aligned && smem <= 200 * 1024 && (int64_t)B * H <= 0x7fffffff) {
        static SmemAttr smem_attr;
        if (int r = allow_smem(smem_attr, ta::build_upper_levels_smem_kernel, smem, "ta_build_levels(upper)")) return r;
        if (B * H > 0)
          ta::build_upper_levels_smem_kernel<<<(unsigned)(B * H), 256, smem, st>>>(nodes, n_sb, n_sh, H, DH, lv, T_len);
      } else {
        const int n = B * H * DH;
        ta::build_upper_levels_kernel<<<(n + 127) / 128, 128, 0, st>>>(nodes, n_sb, n_sh, H, DH, lv, B * H, T_len);
      }
      if (int r = check_launch("ta_build_levels(upper)")) return r;
    }
    return TA_OK;
  }
};

template <typename T, int DH>
struct BuildLogLevels {
  static int run(const void* k, int B, int H, int T_len, int64_t k_sb, int64_t k_sh, int64_t k_st, int cap, int L0,
                 int Lm, int zero_sink, float* nodes, int64_t n_sb, int64_t n_sh, cudaStream_t st) {
    return BuildLevels<T, DH>::run(k, B, H, T_len, k_sb, k_sh, k_st, cap, L0, Lm, zero_sink, nodes, n_sb, n_sh, st,
                                   true);
  }
};

template <typename T, int DH>
struct GateAppend {
  static int run(const void* kc, int B, int H, int64_t c_sb, int64_t c_sh, int64_t c_st, const float* raw, float* lg,
                 float* out, int64_t n_sb, int64_t n_sh, const ta::LevelView& lv, const int32_t* pos, float gate_q,
                 int gate_min, cudaStream_t st) {
    const int64_t threads = (int64_t)B * H * 32;
    if (threads == 0) return TA_OK;
    ta::gate_append_kernel<T, DH><<<(unsigned)((threads + 127) / 128), 128, 0, st>>>(
        reinterpret_cast<const T*>(kc), c_sb, c_sh, c_st, raw, lg, out, n_sb, n_sh, B, H, lv, pos, gate_q, gate_min);
    return check_launch("ta_gate_append");
  }
};

template <typename QT, int DH>
struct Select {
  static int run(ta::SelectParams p, cudaStream_t st) {
    // whole sequences (many queries per (b, h)) on trees whose leaf level fits the score table: the tile kernel
    const int rmax = p.lv.cap >> p.lv.L0;
    const int64_t qs = (int64_t)sizeof(QT);
    const bool q_aligned = (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0 && (p.q_sb * qs) % 16 == 0 &&
                           (p.q_sh * qs) % 16 == 0 && (p.q_st * qs) % 16 == 0;
    if (DH >= 32 && p.Nq >= ta::TS_QT / 4 && rmax <= ta::TS_RMAX && p.wmax <= ta::TS_WMAX && p.wl <= p.wmax &&
        q_aligned)
      return p.wmax <= 4 ? tile<4>(p, st, rmax) : (p.wmax <= 8 ? tile<8>(p, st, rmax) : tile<16>(p, st, rmax));
    // 4 warps (queries) per CTA unless their staging rows would not fit in shared memory
    int warps = 4;
    auto smem_for = [&](int w) {
      return sizeof(ta::DescentScratch) * w + (size_t)w * (2 * p.wmax + 1) * ta::stage_row_floats<DH>() * sizeof(float);
    };
    while (warps > 1 && smem_for(warps) > 200 * 1024) warps >>= 1;
    const size_t smem = smem_for(warps);
    if (smem > 200 * 1024) return fail(TA_ERR_ARG, "ta_select: wmax %d too large for head dim %d", p.wmax, DH);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, ta::select_kernel<QT, DH>, smem, "ta_select")) return r;
    const int64_t nq = (int64_t)p.B * p.H * p.Nq;
    if (nq == 0) return TA_OK;
    ta::select_kernel<QT, DH><<<(unsigned)((nq + warps - 1) / warps), warps * 32, smem, st>>>(p);
    return check_launch("ta_select");
  }

  template <int W>
  static int tile(ta::SelectParams p, cudaStream_t st, int rmax) {
    auto kern = ta::select_tile_kernel<QT, DH, W>;
    const size_t smem = ta::select_tile_smem_bytes<DH>(rmax);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, kern, smem, "ta_select")) return r;
    if ((int64_t)p.B * p.H == 0 || p.Nq == 0) return TA_OK;
    const dim3 grid((unsigned)((p.Nq + ta::TS_QT - 1) / ta::TS_QT), (unsigned)(p.B * p.H), 1);
    kern<<<grid, ta::TS_THREADS, smem, st>>>(p);
    return check_launch("ta_select(tile)");
  }
};

template <typename T, int DH>
struct SegAttn {
  static int run(ta::SegAttnParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.B * p.H * p.Nq;
    if (nq == 0) return TA_OK;
    ta::seg_attn_kernel<T, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_seg_attn");
  }
};

// ---------------------------------------------------------------------------------------------- prefill tiles
// cuTensorMapEncodeTiled from the driver, looked up once (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

int get_encode_tiled() {
  if (g_encode_tiled) return TA_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qr = cudaDriverEntryPointSymbolNotFound;
  const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr);
  if (e != cudaSuccess || qr != cudaDriverEntryPointSuccess || !fn)
    return fail(TA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
  g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return TA_OK;
}

// 4-D tensor map over a (B, H, rows, dh) 16-bit tensor with element strides (sb, sh, st) and a contiguous head
// dim: dims (dh, rows, H, B), box 64 x box_rows x 1 x 1, 128-byte swizzle, zero fill outside the tensor. The
// stride of a size-1 dim is replaced by a valid one (it is never stepped).
int make_rows_map(CUtensorMap* m, const void* ptr, int dtype, int dh, int rows, int H, int B, int64_t st, int64_t sh,
                  int64_t sb, int box_rows, const char* what) {
  if (H == 1) sh = st * rows;
  if (B == 1) sb = sh * H;
  const cuuint64_t dims[4] = {(cuuint64_t)dh, (cuuint64_t)rows, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = g_encode_tiled(
      m, dtype == TA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
      const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TA_ERR_ARG, "ta_prefill_attn: tensor map for %s rejected (CUresult %d)", what, (int)r);
  return TA_OK;
}

template <typename T, int DH>
struct Prefill {
  static constexpr int NS = 3;  // K/V ring stages (dh 64: still two CTAs per SM)
  static int run(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const ta::PrefillParams& p,
                 cudaStream_t st) {
    auto kern = ta::prefill_tile_kernel<T, DH, NS>;
    const size_t smem = ta::prefill_smem_bytes<DH, NS>(p.leaf_words, p.tile_words);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, kern, smem, "ta_prefill_attn")) return r;
    const int64_t grid = (int64_t)p.B * p.H * p.n_qtiles;
    kern<<<(unsigned)grid, ta::PF_THREADS, smem, st>>>(mq, mk, mv, p);
    return check_launch("ta_prefill_attn");
  }
};

template <typename T, int DH>
struct SparseAttn {
  static int run(ta::SparseAttnParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.B * p.H * p.T;
    if (nq == 0) return TA_OK;
    ta::sparse_attn_kernel<T, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_sparse_attn");
  }
};

template <typename T, int DH>
struct SparseAttnBwd {
  static int run(ta::SparseAttnBwdParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.B * p.H * p.T;
    if (nq == 0) return TA_OK;
    ta::sparse_attn_bwd_kernel<T, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_sparse_attn_bwd");
  }
};

template <typename QT, int DH>
struct NeighborPass {
  static int run(ta::NeighborParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.B * p.H * p.Nq;
    if (nq == 0) return TA_OK;
    ta::neighbor_pass_kernel<QT, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_neighbor_pass");
  }
};

template <typename T, int DH>
struct LaneSearch {
  static int run(ta::LaneSearchParams p, cudaStream_t st) {
    if (p.P == 0) return TA_OK;
    ta::lane_search_kernel<DH><<<(unsigned)((p.P + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_lane_search");
  }
};

// One level of the 2-means build: groups of > 256 slots one per CTA, smaller groups one per warp.
__global__ void lane_init_kernel(const int64_t* n, int first, int P, int C, int32_t* perm, uint8_t* valid) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)P * C) return;
  const int s = (int)(i % C);
  perm[i] = s;
  valid[i] = (s >= first && s < n[i / C]) ? 1 : 0;
}

// One level of the 2-means build for groups of more than ta::SUBTREE_SLOTS slots (one group per CTA, rows from
// L2), or, from the first level whose groups are that small, all the remaining levels at once (ta::Subtree).
template <typename T, int DH>
struct LaneSplit {
  static int run(ta::LaneSplitParams p, int levels_left, cudaStream_t st) {
    const int S = p.C >> p.lvl;
    const int64_t groups = (int64_t)p.P << p.lvl;
    if (groups == 0) return TA_OK;
    if (S > ta::SUBTREE_SLOTS) {
      const size_t smem = ta::SplitSmem<8, DH>::bytes(S);
      static SmemAttr smem_attr;
      if (int r = allow_smem(smem_attr, ta::lane_split_cta_kernel<DH>, smem, "ta_lane_order")) return r;
      ta::lane_split_cta_kernel<DH><<<(unsigned)groups, 256, smem, st>>>(p);
    } else {
      const size_t smem = ta::Subtree<DH>::bytes(S);
      static SmemAttr smem_attr;
      if (int r = allow_smem(smem_attr, ta::lane_subtree_kernel<DH>, smem, "ta_lane_order")) return r;
      ta::lane_subtree_kernel<DH><<<(unsigned)groups, 256, smem, st>>>(p, levels_left);
    }
    return check_launch("ta_lane_order");
  }
};

template <typename T, int DH>
struct ForestLevels {
  static int run(ta::ForestLevelsParams p, cudaStream_t st) {
    if (p.P == 0) return TA_OK;
    const size_t smem = (size_t)3 * p.B / 2 * DH * sizeof(float);
    if (smem > 200 * 1024) return fail(TA_ERR_ARG, "ta_forest_levels: blocks of %d keys need %zu B of shared memory", p.B, smem);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, ta::forest_levels_kernel<T, DH>, smem, "ta_forest_levels")) return r;
    ta::forest_levels_kernel<T, DH><<<(unsigned)p.P, 256, smem, st>>>(p);
    return check_launch("ta_forest_levels");
  }
};

template <typename T, int DH>
struct SoftGate {
  static int run(const void* sm, const void* grp, void* out, int64_t N, int S, float q, float temp, cudaStream_t st) {
    if (N == 0) return TA_OK;
    ta::soft_gate_kernel<T, DH><<<(unsigned)((N + 3) / 4), 128, 0, st>>>(
        reinterpret_cast<const T*>(sm), reinterpret_cast<const T*>(grp), reinterpret_cast<T*>(out), N, S, q, temp);
    return check_launch("ta_soft_gate");
  }
};

template <typename T, int DH>
struct ForestSelect {
  static int run(ta::ForestSelectParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.Bn * p.H * p.T;
    if (nq == 0) return TA_OK;
    ta::forest_select_kernel<T, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_forest_select");
  }
};

template <typename T, int DH>
struct LaneInsert {
  static int run(ta::LaneInsertParams p, cudaStream_t st) {
    if (p.P == 0) return TA_OK;
    ta::lane_insert_kernel<DH><<<(unsigned)((p.P + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_lane_insert");
  }
};

template <typename T, int DH>
struct LaneSelect {
  static int run(ta::LaneSelectParams p, cudaStream_t st) {
    const int64_t P = (int64_t)p.B * p.H * p.nl;
    if (P == 0) return TA_OK;
    constexpr size_t smem = ta::lane_select_smem_bytes<DH>();
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, ta::lane_select_kernel<DH>, smem, "ta_lane_select")) return r;
    ta::lane_select_kernel<DH><<<(unsigned)((P + 3) / 4), 128, smem, st>>>(p);
    return check_launch("ta_lane_select");
  }
};

template <typename T, int DH>
struct GatherDot {
  static int run(ta::GatherDotParams p, cudaStream_t st) {
    const int64_t nq = (int64_t)p.B * p.H * p.N;
    if (nq == 0 || p.C == 0) return TA_OK;
    ta::gather_dot_kernel<T, DH><<<(unsigned)((nq + 3) / 4), 128, 0, st>>>(p);
    return check_launch("ta_gather_dot");
  }
};

template <typename T, int DH>
struct GatherDotBlocks {
  static int run(ta::GatherDotBlocksParams p, cudaStream_t st) {
    const size_t smem = (size_t)p.nb_cta * p.blk * DH * sizeof(T);
    if (smem > 200 * 1024)
      return fail(TA_ERR_ARG, "ta_gather_dot_blocks: nb_cta*blk rows need %zu B of shared memory (max 200 KiB)", smem);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, ta::gather_dot_blocks_kernel<T, DH>, smem, "ta_gather_dot_blocks")) return r;
    const int groups = ta::ceil_div(p.nblk, p.nb_cta);
    const int64_t grid = (int64_t)p.B * p.H * groups;
    if (grid == 0) return TA_OK;
    // programmatic dependent launch: a chain of these short, latency-bound calls overlaps each launch with the
    // previous call (the kernel waits for the previous grid before its first global read)
    const cudaError_t e = launch_pdl(ta::gather_dot_blocks_kernel<T, DH>, dim3((unsigned)grid), dim3(128), smem, st, p);
    if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_gather_dot_blocks: launch failed: %s", cudaGetErrorString(e));
    return check_launch("ta_gather_dot_blocks");
  }
};

template <typename T, int DH>
struct Append {
  static int run(ta::AppendParams p, cudaStream_t st) {
    const size_t smem = ta::APPEND_SMEM_FLOATS * sizeof(float);
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, ta::append_kernel<T, DH>, smem, "ta_append")) return r;
    if (p.B * p.H == 0) return TA_OK;
    ta::append_kernel<T, DH><<<p.B * p.H, ta::APPEND_THREADS, smem, st>>>(p);
    return check_launch("ta_append");
  }
};

// Decode ring shape per (dtype, head dim): CH rows per stage, NST stages, 4 consumer warps.
template <typename T, int DH>
struct DecodeShape {
  static constexpr int ROWB = DH * (int)sizeof(T);
  static constexpr int CH = ROWB <= 128 ? 64 : 32;
  static constexpr int NST = 3;
  static constexpr int NCW = 4;
};

std::atomic<int> g_num_sms[kDevCache];

int num_sms() {
  const int dev = current_device();
  const bool cached = dev >= 0 && dev < kDevCache;
  int n = cached ? g_num_sms[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev < 0 ? 0 : dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    if (cached) g_num_sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Decode mode for B*H (b, h) pairs of row_bytes-wide K/V rows: -1 = persistent pipelined kernel (rows of at most
// 128 bytes, so that two CTAs share an SM, or enough pairs for every SM), otherwise the number of CTAs per (b, h)
// of the cluster kernel (~4 resident CTAs per SM). With wider rows the persistent kernel runs one CTA per SM and
// its consumer warps cannot hide their latency, so the cluster kernel (several CTAs per SM) streams faster once
// there are about three pairs per SM; below that (e.g. 320 pairs of 32768-token contexts, dh 128: 0.54 vs 0.47
// of HBM bandwidth measured; 512 pairs: 0.66 vs 0.72) the persistent kernel's one-item-ahead descent wins.
int default_splits(int B, int H, int row_bytes) {
  const int pairs = B * H;
  if (pairs <= 0) return 1;
  if (pairs >= num_sms()) return (row_bytes <= 128 || pairs < 3 * num_sms()) ? -1 : 1;
  // fewer pairs than SMs with narrow rows: the persistent kernel cutting every item into parts (given the split
  // scratch) descends from one round trip of node rows; the cluster kernel descends level by level (configuration-4
  // rows, 96 pairs: 19.9 us against 35.8 us)
  if (row_bytes <= 128) return -1;
  const int target = 4 * num_sms();
  int s = 1;
  while (s < 8 && pairs * s < target) s <<= 1;
  return s;
}

template <typename T, int DH>
struct Decode {
  static int run(ta::DecodeParams p, cudaStream_t st) {
    if (p.B * p.H == 0) return TA_OK;
    if (p.splits < 0) return persistent(p, st);
    using Sh = DecodeShape<T, DH>;
    auto kern = ta::decode_kernel<T, DH, Sh::CH, Sh::NST, Sh::NCW>;
    const size_t smem = ta::decode_smem_bytes<T, DH, Sh::CH, Sh::NST, Sh::NCW>(p.wmax);
    if (smem > 220 * 1024) return fail(TA_ERR_ARG, "ta_decode_step: %zu B of shared memory needed", smem);
    constexpr int RING_FLOATS = (int)(ta::DecodeCfg<T, DH, Sh::CH, Sh::NST, Sh::NCW>::RING_BYTES / sizeof(float));
    if ((1 << p.lv.L0) > RING_FLOATS) return fail(TA_ERR_ARG, "ta_decode_step: leaf block too large");
    static SmemAttr smem_attr;
    if (int r = allow_smem(smem_attr, kern, smem, "ta_decode_step")) return r;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.splits, (unsigned)(p.B * p.H), 1);
    cfg.blockDim = dim3((Sh::NCW + 1) * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // set up while the kernel before ends
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.splits > 1 ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_decode_step: launch failed: %s", cudaGetErrorString(e));
    return check_launch("ta_decode_step");
  }

  // Pipeline shape of the persistent kernel for 256-byte rows (bf16/f16 dh=128, f32 dh=64), which run one CTA
  // per SM: rows per stage, ring stages and consumer groups (compile-time; NST must be a multiple of NCG).
#ifndef TA_MAX_PSPLIT
#define TA_MAX_PSPLIT 8  // most parts per split decode item (persistent kernel); 1 turns splitting off
#endif
#ifndef TA_WIDE_CH
#define TA_WIDE_CH 32
#endif
#ifndef TA_WIDE_NST
#define TA_WIDE_NST 6
#endif
#ifndef TA_WIDE_NCG
#define TA_WIDE_NCG 2
#endif
  static int persistent(ta::DecodeParams p, cudaStream_t st) {
    constexpr int ROWB = DH * (int)sizeof(T);
    constexpr int CH = ROWB <= 128 ? 64 : (ROWB == 256 ? TA_WIDE_CH : 32);  // rows per stage
    constexpr int NST = ROWB == 256 ? TA_WIDE_NST : 4;                        // ring stages
    constexpr int NCG = ROWB == 256 ? TA_WIDE_NCG : 2, WPG = 4;               // consumer groups x warps
    using Cfg = ta::PCfg<T, DH, CH, NST, NCG, WPG>;
    auto kern = ta::decode_persistent_kernel<T, DH, CH, NST, NCG, WPG, false>;
    auto kern_split = ta::decode_persistent_kernel<T, DH, CH, NST, NCG, WPG, true>;
    // descent staging rows: whatever keeps two CTAs per SM (111 KiB each) when at least one full level
    // (2*wmax+1 rows) fits that way, else what one CTA per SM allows
    const size_t row_bytes = (size_t)ta::stage_row_floats<DH>() * 4;
    const size_t base = Cfg::smem_bytes(0);
    const size_t budget = base + (size_t)(2 * p.wmax + 1) * row_bytes <= 111 * 1024 ? 111 * 1024 : 218 * 1024;
    const int fit = budget > base ? (int)((budget - base) / row_bytes) : 0;
    const int stage_rows = std::max(2 * p.wmax + 1, std::min(fit, 256));
    const size_t smem = Cfg::smem_bytes(stage_rows);
    if (smem > 220 * 1024) return fail(TA_ERR_ARG, "ta_decode_step: %zu B of shared memory needed", smem);
    if ((1 << p.lv.L0) > Cfg::TU_FLOATS) return fail(TA_ERR_ARG, "ta_decode_step: leaf block too large");
    static SmemAttr smem_attr, smem_attr_split;
    if (int r = allow_smem(smem_attr, kern, smem, "ta_decode_step(persistent)")) return r;
    if (int r = allow_smem(smem_attr_split, kern_split, smem, "ta_decode_step(persistent)")) return r;
    // CTAs per SM at this shared-memory size, per device
    static std::atomic<int64_t> occ[kDevCache];
    const int dev = current_device();
    const bool cached = dev >= 0 && dev < kDevCache;
    int per_sm = 0;
    const int64_t hit = cached ? occ[dev].load(std::memory_order_relaxed) : 0;
    if (hit != 0 && (size_t)(hit >> 8) == smem) {
      per_sm = (int)(hit & 0xff);
    } else {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Cfg::NTHREADS, smem) != cudaSuccess)
        return check_launch("ta_decode_step(persistent) occupancy");
      per_sm = std::min(std::max(per_sm, 1), 255);
      if (cached) occ[dev].store(((int64_t)smem << 8) | per_sm, std::memory_order_relaxed);
    }
    const int items = p.B * p.H;
    const int gmax = per_sm * num_sms();
    // With one CTA per SM (256-byte rows) whole items leave the last round of CTAs part-empty (e.g. 320 items on 148
    // SMs: 3 rounds, the third for 24 items). The items of that last round are cut into parts (window and leaf rows
    // shared out, partial states merged by the last part to finish) spread over every CTA. Measured on the
    // configuration-5 shape: whole items 204 us; every item in 2 / 3 parts 177 / 195 us (each part repeats its
    // item's descent and pipeline fill); 296 whole items + the 24 others in 6 parts: see the decode profile.
    p.psplit = 1;
    p.n_whole = items;
    int grid;
    if (p.part && p.part_cnt && per_sm == 1 && items % gmax != 0) {
      // full rounds of whole items, then the remaining `tail` items cut into PT parts each so that the last round
      // spreads them over (nearly) every CTA: per CTA R whole items and at most one part of 1/PT item
      const int R = items / gmax, tail = items - R * gmax;
      const int PT = std::min(TA_MAX_PSPLIT, gmax / tail);
      if (PT > 1 && (int64_t)tail * PT <= (int64_t)items * 4) {  // the scratch holds 4 parts per item
        p.psplit = PT;
        p.n_whole = R * gmax;
      }
    } else if (p.part && p.part_cnt && items < gmax) {
      // fewer items than CTA slots (small batches): every item in PT parts, so that each CTA streams a share of one
      // item and the items' descents run side by side. Two parts measured best (every part repeats its item's
      // descent): 8-sequence configuration-4 steps 0.563 ms with 2 parts, 0.574 with 3, 0.607 with 4; with 16 or
      // 24 sequences (under 2 items per CTA slot) whole items stay faster (0.566 / 0.601 ms vs 0.663 / 0.707)
      const int PT = std::min(std::min(TA_MAX_PSPLIT, 2), gmax / items);
      if (PT > 1) {
        p.psplit = PT;
        p.n_whole = 0;
      }
    }
    const int units = p.n_whole + (items - p.n_whole) * p.psplit;
    if (p.psplit > 1) {
      grid = std::min(units, gmax);  // unit u runs on CTA u % grid
    } else {
      const int per_cta = (units + gmax - 1) / gmax;  // units per CTA (equal for all but the last few)
      grid = (units + per_cta - 1) / per_cta;
    }
    // programmatic dependent launch: the CTAs set up while the projection before them ends
    const cudaError_t e = launch_pdl(p.psplit > 1 ? kern_split : kern, dim3(grid), dim3(Cfg::NTHREADS), smem, st, p,
                                     stage_rows);
    if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_decode_step(persistent): launch failed: %s", cudaGetErrorString(e));
    return check_launch("ta_decode_step(persistent)");
  }
};

template <typename T, int MAXV>
int launch_embed(const void* wte, const void* wpe, const int64_t* tok, const int32_t* pos, int B, int V, int P, int C,
                 const float* w, float eps, float* x, void* h, cudaStream_t st) {
  const cudaError_t e = launch_pdl(ta::embed_ln_kernel<T, MAXV>, dim3(B), dim3(ta::ROW_THREADS), 0, st,
                                   reinterpret_cast<const T*>(wte), reinterpret_cast<const T*>(wpe), tok, pos, V, P,
                                   C, w, eps, x, reinterpret_cast<T*>(h));
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_embed_ln: launch failed: %s", cudaGetErrorString(e));
  return check_launch("ta_embed_ln");
}

template <typename T>
int embed_by_c(const void* wte, const void* wpe, const int64_t* tok, const int32_t* pos, int B, int V, int P, int C,
               const float* w, float eps, float* x, void* h, cudaStream_t st) {
  const int need = (C + ta::ROW_THREADS - 1) / ta::ROW_THREADS;
  if (need <= 1) return launch_embed<T, 1>(wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, st);
  if (need <= 2) return launch_embed<T, 2>(wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, st);
  if (need <= 4) return launch_embed<T, 4>(wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, st);
  if (need <= 8) return launch_embed<T, 8>(wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, st);
  if (need <= 16) return launch_embed<T, 16>(wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, st);
  return fail(TA_ERR_ARG, "row width %d above 4096", C);
}

template <typename T>
int add_ln_by_c(float* x, const void* y, int B, int C, const float* w, float eps, void* h, cudaStream_t st) {
  const int need = (C + 255) / 256;  // 16-byte chunks per lane
  const int blocks = (B + 3) / 4;
  const T* yy = reinterpret_cast<const T*>(y);
  T* hh = reinterpret_cast<T*>(h);
  if (need <= 1) ta::add_ln_warp_kernel<T, 1><<<blocks, 128, 0, st>>>(x, yy, B, C, w, eps, hh);
  else if (need <= 2) ta::add_ln_warp_kernel<T, 2><<<blocks, 128, 0, st>>>(x, yy, B, C, w, eps, hh);
  else if (need <= 4) ta::add_ln_warp_kernel<T, 4><<<blocks, 128, 0, st>>>(x, yy, B, C, w, eps, hh);
  else if (need <= 8) ta::add_ln_warp_kernel<T, 8><<<blocks, 128, 0, st>>>(x, yy, B, C, w, eps, hh);
  else return fail(TA_ERR_ARG, "ta_add_ln: row width %d above 2048", C);
  return check_launch("ta_add_ln");
}

int rows_dispatch(int dtype, int kind, const void* a0, const void* a1, const int64_t* tok, const int32_t* pos, int B,
                  int V, int P, int C, const float* w, float eps, float* x, void* h, cudaStream_t st) {
  if (kind == 1 && (C % 8 != 0 || !aligned16(x) || !aligned16(h) || (a1 && !aligned16(a1))))
    return fail(TA_ERR_ARG, "ta_add_ln: rows must be multiples of 8 elements and 16-byte aligned");
  switch (dtype) {
    case TA_F32:
      return kind == 0 ? embed_by_c<float>(a0, a1, tok, pos, B, V, P, C, w, eps, x, h, st)
                       : add_ln_by_c<float>(x, a1, B, C, w, eps, h, st);
    case TA_BF16:
      return kind == 0 ? embed_by_c<__nv_bfloat16>(a0, a1, tok, pos, B, V, P, C, w, eps, x, h, st)
                       : add_ln_by_c<__nv_bfloat16>(x, a1, B, C, w, eps, h, st);
    case TA_F16:
      return kind == 0 ? embed_by_c<__half>(a0, a1, tok, pos, B, V, P, C, w, eps, x, h, st)
                       : add_ln_by_c<__half>(x, a1, B, C, w, eps, h, st);
    default: return fail(TA_ERR_ARG, "bad dtype %d", dtype);
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------------- linear rows
// Shared memory a linear_rows_kernel block may use (the B200's 227 KiB opt-in limit).
constexpr size_t kLinearSmem = 227 * 1024;

// Copy shape of a linear_rows_kernel CTA with BN rows and a Ks slice: nb K blocks per weight copy (large copies
// stream faster), na per copy of the rows, nst ring stages. nst = 0 when nothing fits in shared memory.
struct LinShape {
  int nb, na, nst;
};

LinShape linear_shape(int BN, int Ks) {
  const int nkb = Ks / ta::LIN_KB;
  LinShape sh{1, 1, 0};
  for (int d = 8; d >= 1; --d)
    if (nkb % d == 0) { sh.na = d; break; }
  for (int nb = 4; nb >= 1; --nb) {
    if (nkb % nb != 0) continue;
    const int nstage = nkb / nb;
    for (int nst = std::min(nstage, ta::LIN_MAX_NST); nst >= 1; --nst)
      if (ta::linear_smem_bytes(BN, Ks, nst, nb) <= kLinearSmem && (nst >= 2 || nstage == 1)) {
        sh.nb = nb;
        sh.nst = nst;
        return sh;
      }
  }
  return sh;
}

// 3-D tensor map viewing a (rows, K) 16-bit matrix with a row stride of ld elements as (64, rows, K / 64): box
// (64, box_rows, nblk) = nblk consecutive 64-wide K blocks of box_rows rows; 128-byte swizzle, zeros outside.
int make_blocks_map(CUtensorMap* m, const void* ptr, int dtype, int rows, int K, int64_t ld, int box_rows, int nblk,
                    const char* what) {
  if (int r = get_encode_tiled()) return r;
  const cuuint64_t dims[3] = {(cuuint64_t)ta::LIN_KB, (cuuint64_t)rows, (cuuint64_t)(K / ta::LIN_KB)};
  const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ta::LIN_KB * 2};
  const cuuint32_t box[3] = {(cuuint32_t)ta::LIN_KB, (cuuint32_t)box_rows, (cuuint32_t)nblk};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode_tiled(m, dtype == TA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                    3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TA_ERR_ARG, "tensor map of the %s rejected (CUresult %d)", what, (int)r);
  return TA_OK;
}

template <typename T, int MODE>
int launch_linear(const CUtensorMap& tw, const CUtensorMap& ta_, const ta::LinearParams& p, dim3 grid, size_t smem,
                  cudaStream_t st) {
  static SmemAttr attr;
  if (int r = allow_smem(attr, ta::linear_rows_kernel<T, MODE>, smem, "ta_linear_rows")) return r;
  const cudaError_t e = launch_pdl(ta::linear_rows_kernel<T, MODE>, grid, dim3(ta::LIN_THREADS), smem, st, tw, ta_, p);
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_linear_rows: launch failed: %s", cudaGetErrorString(e));
  return check_launch("ta_linear_rows");
}

template <typename T>
int launch_linear_mode(int mode, const CUtensorMap& tw, const CUtensorMap& ta_, const ta::LinearParams& p, dim3 grid,
                       size_t smem, cudaStream_t st) {
  switch (mode) {
    case ta::LIN_STORE: return launch_linear<T, ta::LIN_STORE>(tw, ta_, p, grid, smem, st);
    case ta::LIN_GELU: return launch_linear<T, ta::LIN_GELU>(tw, ta_, p, grid, smem, st);
    case ta::LIN_PARTIAL: return launch_linear<T, ta::LIN_PARTIAL>(tw, ta_, p, grid, smem, st);
    default: return launch_linear<T, ta::LIN_ARGMAX>(tw, ta_, p, grid, smem, st);
  }
}

// ---------------------------------------------------------------------------------------------- block tail
// Launch plan of block_tail_kernel for B rows of width C on G CTAs (one per SM): K splits per GEMM, the CTA offset of
// each GEMM's units, the shared memory of the busiest CTA and the caller's workspace layout.
struct TailPlan {
  int BN = 0, maxc = 0, nslot = 0;
  ta::TailGemm g[4] = {};
  int off_ln = 0, nsync = 0;
  size_t smem = 0;
  size_t o_part_proj = 0, o_ws_fc = 0, o_part_mlp = 0, o_ws_qkv = 0, o_h2 = 0, o_fc = 0, ws_bytes = 0;
};

// Shared memory a block_tail_kernel block may use (the B200's 227 KiB opt-in limit).
constexpr size_t kTailSmem = 227 * 1024;

// Units of GEMM g that land on CTA c when its first unit sits on CTA `off`.
int tail_units_on(const ta::TailGemm& g, int c, int off, int G) {
  const int first = ((c - off) % G + G) % G;
  return first < g.n ? (g.n - first + G - 1) / G : 0;
}

// Place every GEMM's units (largest units first) at the CTA offset that keeps the busiest CTA's weight bytes lowest
// (ties: the most even spread), so that units of one phase land on different CTAs where they can. Returns the
// busiest CTA's weight bytes, or SIZE_MAX if some CTA would hold more than BT_MAXU units.
size_t place_tail_units(ta::TailGemm (&g)[4], int G) {
  std::vector<size_t> bytes(G, 0);
  std::vector<int> units(G, 0);
  int order[4] = {0, 1, 2, 3};
  std::sort(order, order + 4, [&](int a, int b) { return g[a].kc > g[b].kc || (g[a].kc == g[b].kc && a < b); });
  for (int oi = 0; oi < 4; ++oi) {
    ta::TailGemm& t = g[order[oi]];
    t.off = 0;
    if (t.n == 0) continue;
    const size_t ub = (size_t)t.kc * ta::LIN_W_BYTES;
    size_t best_max = SIZE_MAX;
    double best_sq = 0.0;
    for (int off = 0; off < G; ++off) {
      size_t mx = 0;
      double sq = 0.0;
      for (int c = 0; c < G; ++c) {
        const size_t b = bytes[c] + (size_t)tail_units_on(t, c, off, G) * ub;
        mx = std::max(mx, b);
        sq += (double)b * (double)b;
      }
      if (mx < best_max || (mx == best_max && sq < best_sq)) {
        best_max = mx;
        best_sq = sq;
        t.off = off;
      }
    }
    for (int c = 0; c < G; ++c) {
      const int k = tail_units_on(t, c, t.off, G);
      bytes[c] += (size_t)k * ub;
      units[c] += k;
    }
  }
  size_t mx = 0;
  for (int c = 0; c < G; ++c) {
    if (units[c] > ta::BT_MAXU) return SIZE_MAX;
    mx = std::max(mx, bytes[c]);
  }
  return mx;
}

// Smallest K split of nk 64-wide blocks whose units hold at most kc_cap blocks.
int split_for(int nk, int kc_cap) {
  for (int d = 1; d <= nk; ++d)
    if (nk % d == 0 && nk / d <= kc_cap) return d;
  return nk;
}

bool make_tail_plan(int B, int C, bool with_qkv, int G, int esize, TailPlan& pl) {
  pl = TailPlan{};
  if (B < 1 || C < 128 || C % 128 != 0 || C > ta::BT_MAX_C || G < 1) return false;
  pl.BN = (B + 15) / 16 * 16;
  if (pl.BN > ta::BT_MAX_BN) return false;
  pl.maxc = pl.BN <= 32 ? 32 : (pl.BN <= 64 ? 64 : 128);
  const int F = 4 * C;
  const int N[4] = {C, F, C, 3 * C}, K[4] = {C, C, F, C};
  const int T[4] = {C / 128, F / 128, C / 128, 3 * C / 128};
  // K splits: c_proj and c_mlp in slices of at most 6 / 8 blocks (their partial sums meet in the layer norm's
  // rows); c_fc and c_attn whole when the rows' stage fits (no partial sums to exchange), else split with the
  // tile's last split adding the others' sums
  const int s_proj = split_for(K[0] / 64, 6), s_mlp = split_for(K[2] / 64, 8);
  const int whole_opts[] = {1, 2, 3, 4, 6};
  for (int sf : whole_opts)
    for (int sq : whole_opts) {
      const int S[4] = {s_proj, sf, s_mlp, with_qkv ? sq : 1};
      bool ok = true;
      for (int i = 0; i < 4 && ok; ++i) ok = (K[i] / 64) % S[i] == 0;
      if (!ok) continue;
      ta::TailGemm g[4];
      int kc_max = 1;
      for (int i = 0; i < 4; ++i) {
        g[i].N = N[i];
        g[i].K = K[i];
        g[i].S = S[i];
        g[i].kc = K[i] / 64 / S[i];
        g[i].n = (i == ta::TG_QKV && !with_qkv) ? 0 : T[i] * S[i];
        if (g[i].n > 0) kc_max = std::max(kc_max, g[i].kc);
      }
      if (place_tail_units(g, G) == SIZE_MAX) continue;
      const size_t fixed = 1024 + ta::tail_stage_bytes(pl.BN, kc_max, C, std::max(S[0], S[2])) +
                           sizeof(ta::TailBars) + 16;
      if (fixed + 2 * (size_t)ta::LIN_W_BYTES > kTailSmem) continue;
      const int nslot = (int)std::min<size_t>(ta::BT_MAX_SLOTS, (kTailSmem - fixed) / ta::LIN_W_BYTES);
      std::copy(g, g + 4, pl.g);
      pl.nslot = nslot;
      pl.smem = fixed + (size_t)nslot * ta::LIN_W_BYTES;
      pl.off_ln = 0;
      pl.nsync = ta::TW_FIXED + 2 * T[1] + T[3];
      // workspace: fp32 sums, then the 16-bit layer-norm and GELU rows (each piece 256-byte aligned)
      size_t o = 0;
      auto take = [&](size_t bytes) {
        const size_t at = o;
        o += (bytes + 255) / 256 * 256;
        return at;
      };
      pl.o_part_proj = take((size_t)S[0] * B * C * 4);
      pl.o_ws_fc = take(S[1] > 1 ? (size_t)T[1] * S[1] * pl.BN * 128 * 4 : 0);
      pl.o_part_mlp = take((size_t)S[2] * B * C * 4);
      pl.o_ws_qkv = take(with_qkv && S[3] > 1 ? (size_t)T[3] * S[3] * pl.BN * 128 * 4 : 0);
      pl.o_h2 = take((size_t)B * C * esize);
      pl.o_fc = take((size_t)B * F * esize);
      pl.ws_bytes = o;
      return true;
    }
  return false;
}

// Plans are cached per (rows, width, with c_attn, CTAs, element size).
std::mutex g_tail_mu;
std::map<std::tuple<int, int, int, int, int>, TailPlan> g_tail_plans;

bool tail_plan(int B, int C, bool with_qkv, int esize, TailPlan& pl) {
  const int G = num_sms();
  const auto key = std::make_tuple(B, C, (int)with_qkv, G, esize);
  std::lock_guard<std::mutex> lk(g_tail_mu);
  auto it = g_tail_plans.find(key);
  if (it != g_tail_plans.end()) {
    pl = it->second;
    return pl.BN > 0;
  }
  const bool ok = make_tail_plan(B, C, with_qkv, G, esize, pl);
  if (!ok) pl = TailPlan{};
  g_tail_plans[key] = pl;
  return ok;
}

template <typename T, int MAXC>
int launch_tail(const ta::TailMaps& m, const ta::BlockTailParams& p, size_t smem, cudaStream_t st) {
  auto kern = ta::block_tail_kernel<T, MAXC>;
  static SmemAttr attr;
  if (int r = allow_smem(attr, kern, smem, "ta_block_tail")) return r;
  // every CTA must be resident at once (the phases wait on each other's counters)
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, ta::BT_THREADS, smem) != cudaSuccess)
    return check_launch("ta_block_tail");
  if ((int64_t)per_sm * num_sms() < p.G)
    return fail(TA_ERR_ARG, "ta_block_tail: %d CTAs cannot all be resident (%d per SM)", p.G, per_sm);
  const cudaError_t e = launch_pdl(kern, dim3((unsigned)p.G), dim3(ta::BT_THREADS), smem, st, m, p);
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_block_tail: launch failed: %s", cudaGetErrorString(e));
  return check_launch("ta_block_tail");
}

template <typename T>
int launch_tail_by_c(int maxc, const ta::TailMaps& m, const ta::BlockTailParams& p, size_t smem, cudaStream_t st) {
  switch (maxc) {
    case 32: return launch_tail<T, 32>(m, p, smem, st);
    case 64: return launch_tail<T, 64>(m, p, smem, st);
    default: return launch_tail<T, 128>(m, p, smem, st);
  }
}

// ================================================================================================== C ABI
// Scratch of ta_lane_order_noalloc, in the library's own device memory: the second slot-order buffer that the
// 2-means build ping-pongs with the caller's output. 2^21 slots (P * C at most): 8 MiB of int32 + 2 MiB of flags,
// held by every GPU that loads the library until the process exits. Every slot of it is written before it is read in
// a call, so it never needs clearing; all calls share it, so calls that overlap on the GPU race.
constexpr int64_t kLaneScratchSlots = int64_t(1) << 21;
static __device__ __align__(256) int32_t g_lane_perm_scratch[kLaneScratchSlots];
static __device__ __align__(256) uint8_t g_lane_valid_scratch[kLaneScratchSlots];

namespace {
// Device addresses of the scratch. An address belongs to one CUDA context (the module is loaded per context), not
// to a device number: after cudaDeviceReset, or with another context current (a driver-API caller with its own
// context), the old address is stale. So every call made outside stream capture looks the address up again with
// the calling thread's context current, and records it against that context; a call made while its stream is
// capturing (where a lookup could load the module, which capture forbids) uses the address recorded for the current
// context, and fails if there is none. In host code the arrays' names stand for host-side shadows, never for the
// device memory, so only these addresses may reach a kernel.
struct LaneScratch {
  CUcontext ctx;
  int32_t* perm;
  uint8_t* valid;
};
constexpr int kMaxScratchContexts = 64;
std::mutex g_scratch_mu;
LaneScratch g_scratch[kMaxScratchContexts];
int g_scratch_n = 0;
PFN_cuCtxGetCurrent_v4000 g_ctx_get_current = nullptr;

int current_context(CUcontext* ctx) {
  if (!g_ctx_get_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &qr);
    if (e != cudaSuccess || qr != cudaDriverEntryPointSuccess || !fn)
      return fail(TA_ERR_CUDA, "ta_lane_order_noalloc: cuCtxGetCurrent unavailable (%s)", cudaGetErrorString(e));
    g_ctx_get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  }
  *ctx = nullptr;
  const CUresult r = g_ctx_get_current(ctx);
  if (r != CUDA_SUCCESS) return fail(TA_ERR_CUDA, "ta_lane_order_noalloc: cuCtxGetCurrent failed (CUresult %d)", (int)r);
  return TA_OK;
}

int lane_scratch(cudaStream_t st, int32_t** perm, uint8_t** valid) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_lane_order_noalloc: stream state: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  CUcontext ctx = nullptr;
  if (cs == cudaStreamCaptureStatusNone) {
    void* pa = nullptr;
    void* va = nullptr;
    e = cudaGetSymbolAddress(&pa, g_lane_perm_scratch);  // makes the device's primary context current if none is
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&va, g_lane_valid_scratch);
    if (e != cudaSuccess || !pa || !va)
      return fail(TA_ERR_CUDA, "ta_lane_order_noalloc: scratch address: %s", cudaGetErrorString(e));
    if (int r = current_context(&ctx)) return r;
    int i = 0;
    while (i < g_scratch_n && g_scratch[i].ctx != ctx) ++i;
    if (i == g_scratch_n && g_scratch_n < kMaxScratchContexts) ++g_scratch_n;
    if (i < kMaxScratchContexts) g_scratch[i] = {ctx, static_cast<int32_t*>(pa), static_cast<uint8_t*>(va)};
    *perm = static_cast<int32_t*>(pa);
    *valid = static_cast<uint8_t*>(va);
    return TA_OK;
  }
  if (int r = current_context(&ctx)) return r;
  for (int i = 0; i < g_scratch_n; ++i)
    if (g_scratch[i].ctx == ctx) {
      *perm = g_scratch[i].perm;
      *valid = g_scratch[i].valid;
      return TA_OK;
    }
  return fail(TA_ERR_ARG, "ta_lane_order_noalloc: called during stream capture before any call outside capture in "
              "this context (the scratch address is looked up outside capture)");
}
}  // namespace

extern "C" {

int ta_version(void) { return 100; }

const char* ta_last_error(void) { return g_err.c_str(); }

int ta_device_error(int* out4) {
  if (!out4) return fail(TA_ERR_ARG, "ta_device_error: null output");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_device_error: %s", cudaGetErrorString(e));
  e = cudaMemcpyFromSymbol(out4, ta::g_dev_err, 4 * sizeof(int));
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_device_error: %s", cudaGetErrorString(e));
  const int zero[4] = {0, 0, 0, 0};
  e = cudaMemcpyToSymbol(ta::g_dev_err, zero, 4 * sizeof(int));
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_device_error: %s", cudaGetErrorString(e));
  return TA_OK;
}

int ta_wait_probe(int64_t limit_ns, void* stream) {
  g_err.clear();
  if (limit_ns < 1000 || limit_ns > 10000000000ll)
    return fail(TA_ERR_ARG, "ta_wait_probe: limit %lld ns outside [1 us, 10 s]", (long long)limit_ns);
  ta::wait_probe_kernel<<<1, 32, 0, S(stream)>>>((uint64_t)limit_ns);
  return check_launch("ta_wait_probe");
}

int64_t ta_level_nodes(int cap, int L0, int Lm) {
  if (cap <= 0 || L0 < 0 || Lm < L0 || Lm > 30) return 0;
  int off[ta::MAX_LEVELS];
  return ta::level_offsets(cap, L0, Lm, off);
}

int ta_build_levels(const void* k, int dtype, int B, int H, int T_len, int dh, int64_t k_sb, int64_t k_sh,
                    int64_t k_st, int cap, int L0, int Lm, int zero_sink, float* nodes, int64_t n_sb, int64_t n_sh,
                    void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_build_levels: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_build_levels: unsupported head dim %d", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (B < 0 || H <= 0 || T_len < 0 || T_len > cap)
    return fail(TA_ERR_ARG, "ta_build_levels: bad sizes B=%d H=%d T=%d cap=%d", B, H, T_len, cap);
  if (!k || !nodes) return fail(TA_ERR_ARG, "ta_build_levels: null pointer");
  return by_type_dh<BuildLevels>(dtype, dh, k, B, H, T_len, k_sb, k_sh, k_st, cap, L0, Lm, zero_sink, nodes, n_sb,
                                 n_sh, S(stream));
}

int ta_build_log_levels(const void* k, int dtype, int B, int H, int T_len, int dh, int64_t k_sb, int64_t k_sh,
                        int64_t k_st, int cap, int L0, int Lm, int zero_sink, float* nodes, int64_t n_sb,
                        int64_t n_sh, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_build_log_levels: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_build_log_levels: unsupported head dim %d", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (B < 0 || H <= 0 || T_len < 0 || T_len > cap)
    return fail(TA_ERR_ARG, "ta_build_log_levels: bad sizes B=%d H=%d T=%d cap=%d", B, H, T_len, cap);
  if (!k || !nodes) return fail(TA_ERR_ARG, "ta_build_log_levels: null pointer");
  return by_type_dh<BuildLogLevels>(dtype, dh, k, B, H, T_len, k_sb, k_sh, k_st, cap, L0, Lm, zero_sink, nodes, n_sb,
                                    n_sh, S(stream));
}

int ta_gate_levels(const float* raw, const float* lg, float* out, int B, int H, int dh, int T_len, int64_t n_sb,
                   int64_t n_sh, int cap, int L0, int Lm, float gate_q, int gate_min, void* stream) {
  g_err.clear();
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_gate_levels: head dim %d (16, 32, 64, 128)", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (B < 0 || H <= 0 || T_len < 0 || T_len > cap) return fail(TA_ERR_ARG, "ta_gate_levels: bad sizes");
  if (!(gate_q >= 0.f && gate_q <= 1.f)) return fail(TA_ERR_ARG, "ta_gate_levels: gate_q outside [0, 1]");
  if (!raw || !lg || !out) return fail(TA_ERR_ARG, "ta_gate_levels: null pointer");
  const ta::LevelView lv = make_lv(raw, n_sb, n_sh, cap, L0, Lm);
  const int64_t per_bh = ta_level_nodes(cap, L0, Lm);
  const int64_t threads = (int64_t)B * H * per_bh * 32;
  if (threads == 0) return TA_OK;
  const unsigned grid = (unsigned)((threads + 127) / 128);
  cudaStream_t st = S(stream);
  auto kern = dh == 16 ? ta::gate_levels_kernel<16>
              : dh == 32 ? ta::gate_levels_kernel<32> : dh == 64 ? ta::gate_levels_kernel<64> : ta::gate_levels_kernel<128>;
  kern<<<grid, 128, 0, st>>>(raw, lg, out, n_sb, n_sh, H, lv, T_len, B * H, gate_q, gate_min, per_bh);
  return check_launch("ta_gate_levels");
}

int ta_gate_append(const void* kc, int dtype, int B, int H, int dh, int64_t c_sb, int64_t c_sh, int64_t c_st,
                   const float* raw, float* lg, float* out, int64_t n_sb, int64_t n_sh, int cap, int L0, int Lm,
                   const int32_t* pos, float gate_q, int gate_min, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_gate_append: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_gate_append: head dim %d (16, 32, 64, 128)", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (L0 > 15) return fail(TA_ERR_ARG, "ta_gate_append: leaf level %d above 15", L0);
  if (B < 0 || H <= 0) return fail(TA_ERR_ARG, "ta_gate_append: bad sizes");
  if (!(gate_q >= 0.f && gate_q <= 1.f)) return fail(TA_ERR_ARG, "ta_gate_append: gate_q outside [0, 1]");
  if (!kc || !raw || !lg || !out || !pos) return fail(TA_ERR_ARG, "ta_gate_append: null pointer");
  const ta::LevelView lv = make_lv(raw, n_sb, n_sh, cap, L0, Lm);
  return by_type_dh<GateAppend>(dtype, dh, kc, B, H, c_sb, c_sh, c_st, raw, lg, out, n_sb, n_sh, lv, pos, gate_q,
                                gate_min, S(stream));
}

int ta_select(const void* q, int q_dtype, int B, int H, int Nq, int dh, int64_t q_sb, int64_t q_sh, int64_t q_st,
              const int64_t* tq, int64_t tq_sb, int64_t tq_st, const float* nodes, int64_t n_sb, int64_t n_sh,
              int cap, int L0, int Lm, int wmax, int wl, int64_t* ids, uint8_t* vld, float* sct, void* stream) {
  g_err.clear();
  if (!valid_dtype(q_dtype)) return fail(TA_ERR_ARG, "ta_select: bad dtype %d", q_dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_select: unsupported head dim %d", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (wmax < 1 || wmax > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_select: wmax=%d outside [1, 64]", wmax);
  if (wl < 1 || wl > wmax) return fail(TA_ERR_ARG, "ta_select: wl=%d outside [1, wmax]", wl);
  if (B < 0 || H <= 0 || Nq < 0) return fail(TA_ERR_ARG, "ta_select: bad sizes");
  if (!q || !tq || !nodes || !ids || !vld) return fail(TA_ERR_ARG, "ta_select: null pointer");
  if (!aligned16(nodes) || (n_sb * 4) % 16 || (n_sh * 4) % 16)
    return fail(TA_ERR_ARG, "ta_select: node rows must be 16-byte aligned");
  ta::SelectParams p{};
  p.q = q;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.q_st = q_st;
  p.tq = tq;
  p.tq_sb = tq_sb;
  p.tq_st = tq_st;
  p.lv = make_lv(nodes, n_sb, n_sh, cap, L0, Lm);
  p.B = B;
  p.H = H;
  p.Nq = Nq;
  p.wmax = wmax;
  p.wl = wl;
  p.ids = ids;
  p.vld = vld;
  p.sct = sct;
  return by_type_dh<Select>(q_dtype, dh, p, S(stream));
}

int ta_finish(const int64_t* ids, const uint8_t* vld, const int64_t* nid, const uint8_t* match, const int64_t* nL,
              const int64_t* lhat, int64_t Q, int wl, int nbw, int leaf, int wmax, int64_t* tree_pos,
              int64_t* nb_pos, int64_t* n_tree, int64_t* nb_leaves, void* stream) {
  g_err.clear();
  if (Q < 0 || wl < 0 || nbw < 0 || leaf < 1) return fail(TA_ERR_ARG, "ta_finish: bad sizes");
  if (!ids || !vld || !lhat || !n_tree || !nb_leaves) return fail(TA_ERR_ARG, "ta_finish: null pointer");
  if (Q == 0) return TA_OK;
  ta::FinishParams p{ids, vld, nid, match, nL, lhat, Q, wl, nbw, leaf, wmax, tree_pos, nb_pos, n_tree, nb_leaves};
  ta::finish_kernel<<<(unsigned)((Q + 127) / 128), 128, 0, S(stream)>>>(p);
  return check_launch("ta_finish");
}

int ta_seg_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int Nq, int dh,
                int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const int64_t* tq, int64_t tq_sb,
                int64_t tq_st, const int64_t* ids, const uint8_t* vld, int wl, const int64_t* n_tree,
                int ntree_const, int leaf, int Lw, float scale, void* o, int64_t o_sb, int64_t o_sh, int64_t o_st,
                float* lse, int32_t* nkeys, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_seg_attn: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_seg_attn: unsupported head dim %d", dh);
  if (wl < 0 || wl > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_seg_attn: wl=%d outside [0, 64]", wl);
  if (leaf < 1 || (leaf & (leaf - 1))) return fail(TA_ERR_ARG, "ta_seg_attn: leaf %d not a power of two", leaf);
  if (Lw < 1) return fail(TA_ERR_ARG, "ta_seg_attn: window %d < 1", Lw);
  if (!q || !k || !v || !tq || (wl > 0 && (!ids || !vld)) || !o) return fail(TA_ERR_ARG, "ta_seg_attn: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(q, es, {q_sb, q_sh, q_st}) || !rows_aligned(k, es, {k_sb, k_sh, k_st}) ||
      !rows_aligned(v, es, {v_sb, v_sh, v_st}) || !rows_aligned(o, es, {o_sb, o_sh, o_st}))
    return fail(TA_ERR_ARG, "ta_seg_attn: q/k/v/o rows must be 16-byte aligned");
  ta::SegAttnParams p{};
  p.q = q; p.k = k; p.v = v;
  p.q_sb = q_sb; p.q_sh = q_sh; p.q_st = q_st;
  p.k_sb = k_sb; p.k_sh = k_sh; p.k_st = k_st;
  p.v_sb = v_sb; p.v_sh = v_sh; p.v_st = v_st;
  p.tq = tq; p.tq_sb = tq_sb; p.tq_st = tq_st;
  p.ids = ids; p.vld = vld; p.n_tree = n_tree; p.ntree_const = ntree_const;
  p.B = B; p.H = H; p.Nq = Nq; p.wl = wl; p.leaf = leaf; p.Lw = Lw; p.T_kv = T_kv;
  p.scale = scale;
  p.o = o; p.o_sb = o_sb; p.o_sh = o_sh; p.o_st = o_st;
  p.lse = lse; p.nkeys = nkeys;
  return by_type_dh<SegAttn>(dtype, dh, p, S(stream));
}

int ta_prefill_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int Nq, int dh,
                    int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                    int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const int64_t* tq, int64_t tq_sb,
                    int64_t tq_st, const int64_t* ids, const uint8_t* vld, int wl, const int64_t* n_tree,
                    int ntree_const, int leaf, int Lw, float scale, void* o, int64_t o_sb, int64_t o_sh,
                    int64_t o_st, float* lse, int32_t* nkeys, void* stream) {
  g_err.clear();
  if (dtype != TA_BF16 && dtype != TA_F16) return fail(TA_ERR_ARG, "ta_prefill_attn: dtype must be bf16 or f16");
  if (dh != 64 && dh != 128) return fail(TA_ERR_ARG, "ta_prefill_attn: head dim %d not 64 or 128", dh);
  if (wl < 0 || wl > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_prefill_attn: wl=%d outside [0, 64]", wl);
  if (leaf < 2 || (leaf & (leaf - 1))) return fail(TA_ERR_ARG, "ta_prefill_attn: leaf %d not a power of two >= 2", leaf);
  if (Lw < 1) return fail(TA_ERR_ARG, "ta_prefill_attn: window %d < 1", Lw);
  if (B < 0 || H < 0 || Nq < 0 || T_kv < 1) return fail(TA_ERR_ARG, "ta_prefill_attn: bad sizes");
  if (!q || !k || !v || !tq || (wl > 0 && (!ids || !vld)) || !o) return fail(TA_ERR_ARG, "ta_prefill_attn: null pointer");
  const int64_t nleaves = ((int64_t)T_kv + leaf - 1) / leaf, ntiles = ((int64_t)T_kv + ta::PF_KT - 1) / ta::PF_KT;
  if (nleaves > 32 * ta::PF_MAX_LEAF_WORDS)
    return fail(TA_ERR_ARG, "ta_prefill_attn: %lld leaf blocks per sequence (at most %d; use ta_seg_attn)",
                (long long)nleaves, 32 * ta::PF_MAX_LEAF_WORDS);
  if (ntiles > 32 * ta::PF_MAX_TILE_WORDS) return fail(TA_ERR_ARG, "ta_prefill_attn: T_kv %d too long", T_kv);
  if (!rows_aligned(q, 2, {q_sb, q_sh, q_st}) || !rows_aligned(k, 2, {k_sb, k_sh, k_st}) ||
      !rows_aligned(v, 2, {v_sb, v_sh, v_st}) || !rows_aligned(o, 2, {o_sb, o_sh, o_st}))
    return fail(TA_ERR_ARG, "ta_prefill_attn: q/k/v/o rows must be 16-byte aligned");
  if ((int64_t)B * H * Nq == 0) return TA_OK;
  if (int r = get_encode_tiled()) return r;
  CUtensorMap mq, mk, mv;
  if (int r = make_rows_map(&mq, q, dtype, dh, Nq, H, B, q_st, q_sh, q_sb, ta::PF_QT, "q")) return r;
  if (int r = make_rows_map(&mk, k, dtype, dh, T_kv, H, B, k_st, k_sh, k_sb, ta::PF_KT, "k")) return r;
  if (int r = make_rows_map(&mv, v, dtype, dh, T_kv, H, B, v_st, v_sh, v_sb, ta::PF_KT, "v")) return r;
  ta::PrefillParams p{};
  p.tq = tq; p.tq_sb = tq_sb; p.tq_st = tq_st;
  p.ids = ids; p.vld = vld; p.n_tree = n_tree; p.ntree_const = ntree_const;
  p.B = B; p.H = H; p.Nq = Nq; p.wl = wl; p.Lw = Lw; p.T_kv = T_kv;
  p.L0 = 0;
  while ((1 << p.L0) < leaf) ++p.L0;
  p.n_qtiles = (Nq + ta::PF_QT - 1) / ta::PF_QT;
  p.leaf_words = (int)((nleaves + 31) / 32);
  p.tile_words = (int)((ntiles + 31) / 32);
  p.scale_log2 = scale * ta::LOG2E;
  p.o = o; p.o_sb = o_sb; p.o_sh = o_sh; p.o_st = o_st;
  p.lse = lse; p.nkeys = nkeys;
  cudaStream_t st = S(stream);
  if (dtype == TA_BF16)
    return dh == 64 ? Prefill<__nv_bfloat16, 64>::run(mq, mk, mv, p, st) : Prefill<__nv_bfloat16, 128>::run(mq, mk, mv, p, st);
  return dh == 64 ? Prefill<__half, 64>::run(mq, mk, mv, p, st) : Prefill<__half, 128>::run(mq, mk, mv, p, st);
}

int ta_sparse_attn(const void* q, const void* k, const void* v, int dtype, int B, int H, int T, int dh,
                   int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_st,
                   int64_t v_sb, int64_t v_sh, int64_t v_st, int T_kv, const void* cand, int cand64, int Kc,
                   float scale, void* o, int64_t o_sb, int64_t o_sh, int64_t o_st, float* lse, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_sparse_attn: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_sparse_attn: unsupported head dim %d", dh);
  if (Kc < 0) return fail(TA_ERR_ARG, "ta_sparse_attn: Kc < 0");
  if (!q || !k || !v || !o || (Kc > 0 && !cand)) return fail(TA_ERR_ARG, "ta_sparse_attn: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(q, es, {q_sb, q_sh, q_st}) || !rows_aligned(k, es, {k_sb, k_sh, k_st}) ||
      !rows_aligned(v, es, {v_sb, v_sh, v_st}) || !rows_aligned(o, es, {o_sb, o_sh, o_st}))
    return fail(TA_ERR_ARG, "ta_sparse_attn: q/k/v/o rows must be 16-byte aligned");
  ta::SparseAttnParams p{};
  p.q = q; p.k = k; p.v = v;
  p.q_sb = q_sb; p.q_sh = q_sh; p.q_st = q_st;
  p.k_sb = k_sb; p.k_sh = k_sh; p.k_st = k_st;
  p.v_sb = v_sb; p.v_sh = v_sh; p.v_st = v_st;
  p.cand = cand; p.cand64 = cand64;
  p.B = B; p.H = H; p.T = T; p.Kc = Kc; p.T_kv = T_kv;
  p.scale = scale;
  p.o = o; p.o_sb = o_sb; p.o_sh = o_sh; p.o_st = o_st;
  p.lse = lse;
  return by_type_dh<SparseAttn>(dtype, dh, p, S(stream));
}

int ta_neighbor_pass(const void* q, int q_dtype, int B, int H, int Nq, int dh, int64_t q_sb, int64_t q_sh,
                     int64_t q_st, const int64_t* tq, int64_t tq_sb, int64_t tq_st, const float* leaf_nodes,
                     int64_t n_sb, int64_t n_sh, int n_leaf, int L0, const int64_t* st_leaf, const float* st_score,
                     const uint8_t* st_ok, int T_st, int nb_window, int nb_store, float nb_rho, int nb_probe,
                     int nb_cap_min, int neighbors, int64_t* nid, uint8_t* match, int64_t* nL, void* stream) {
  g_err.clear();
  if (!valid_dtype(q_dtype)) return fail(TA_ERR_ARG, "ta_neighbor_pass: bad dtype %d", q_dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_neighbor_pass: unsupported head dim %d", dh);
  if (B < 0 || H < 0 || Nq < 0 || n_leaf < 1 || T_st < 1 || L0 < 0 || L0 > 30)
    return fail(TA_ERR_ARG, "ta_neighbor_pass: bad sizes");
  if (nb_window < 1 || nb_store < 1 || nb_window * nb_store > 32)
    return fail(TA_ERR_ARG, "ta_neighbor_pass: nb_window * nb_store = %d outside [1, 32]", nb_window * nb_store);
  if (nb_probe < 0 || nb_cap_min < 0) return fail(TA_ERR_ARG, "ta_neighbor_pass: bad probe / cap");
  if (!q || !tq || !leaf_nodes || !st_leaf || !st_score || !st_ok || !nid || !match || !nL)
    return fail(TA_ERR_ARG, "ta_neighbor_pass: null pointer");
  if (!aligned16(leaf_nodes) || (n_sb * 4) % 16 || (n_sh * 4) % 16)
    return fail(TA_ERR_ARG, "ta_neighbor_pass: node rows must be 16-byte aligned");
  ta::NeighborParams p{};
  p.q = q; p.q_sb = q_sb; p.q_sh = q_sh; p.q_st = q_st;
  p.tq = tq; p.tq_sb = tq_sb; p.tq_st = tq_st;
  p.leaf_nodes = leaf_nodes; p.n_sb = n_sb; p.n_sh = n_sh; p.n_leaf = n_leaf;
  p.scale = ldexpf(1.f, -L0);
  p.st_leaf = st_leaf; p.st_score = st_score; p.st_ok = st_ok; p.T_st = T_st;
  p.B = B; p.H = H; p.Nq = Nq; p.Wn = nb_window; p.NS = nb_store;
  p.probe = std::min(nb_probe * nb_store, nb_window * nb_store);
  p.cap_min = nb_cap_min; p.neighbors = neighbors; p.rho = nb_rho;
  p.nid = nid; p.match = match; p.nL = nL;
  return by_type_dh<NeighborPass>(q_dtype, dh, p, S(stream));
}

int ta_lane_search(const float* q, const float* sums, const int32_t* cnt, int P, int D, int dh, int wmax, int wl,
                   int64_t* ids, uint8_t* vld, float* sct, void* stream) {
  g_err.clear();
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_lane_search: unsupported head dim %d", dh);
  if (P < 0 || D < 1 || D > 24) return fail(TA_ERR_ARG, "ta_lane_search: bad sizes P=%d D=%d", P, D);
  if (wmax < 1 || wmax > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_lane_search: wmax=%d outside [1, 64]", wmax);
  if (wl < 1 || wl > wmax) return fail(TA_ERR_ARG, "ta_lane_search: wl=%d outside [1, wmax]", wl);
  if (!q || !sums || !cnt || !ids || !vld) return fail(TA_ERR_ARG, "ta_lane_search: null pointer");
  if (!aligned16(q) || !aligned16(sums)) return fail(TA_ERR_ARG, "ta_lane_search: q / sums must be 16-byte aligned");
  ta::LaneSearchParams p{q, sums, cnt, P, D, wmax, wl, ids, vld, sct};
  return by_dh<LaneSearch, float>(dh, p, S(stream));
}

static int log2_exact(int64_t x) {
  int l = 0;
  while ((int64_t(1) << l) < x) ++l;
  return (int64_t(1) << l) == x ? l : -1;
}

int ta_lane_order(const float* keys, int64_t key_lane_div, int64_t key_stride, const int64_t* n, int first, int P,
                  int C, int dh, int iters, int levels, int32_t* perm, uint8_t* valid, int32_t* perm_tmp,
                  uint8_t* valid_tmp, void* stream) {
  g_err.clear();
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_lane_order: unsupported head dim %d", dh);
  const int lc = log2_exact(C);
  if (P < 0 || lc < 2 || C > 16384) return fail(TA_ERR_ARG, "ta_lane_order: C=%d is not a power of two in [4, 16384]", C);
  if (levels < 0 || levels > lc - 1) return fail(TA_ERR_ARG, "ta_lane_order: levels=%d outside [0, %d]", levels, lc - 1);
  if (iters < 0 || first < 0 || key_lane_div < 1) return fail(TA_ERR_ARG, "ta_lane_order: bad iters / first / lane divisor");
  if (!keys || !n || !perm || !valid || !perm_tmp || !valid_tmp) return fail(TA_ERR_ARG, "ta_lane_order: null pointer");
  if (!aligned16(keys) || (key_stride * 4) % 16 != 0)
    return fail(TA_ERR_ARG, "ta_lane_order: keys and the key array stride must be 16-byte aligned");
  if (P == 0) return TA_OK;
  cudaStream_t st = S(stream);
  const int64_t total = (int64_t)P * C;
  lane_init_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(n, first, P, C, perm, valid);
  if (int e = check_launch("ta_lane_order")) return e;
  int32_t* pa = perm; uint8_t* va = valid;
  int32_t* pb = perm_tmp; uint8_t* vb = valid_tmp;
  for (int lvl = 0; lvl < levels; ++lvl) {
    ta::LaneSplitParams p{keys, key_lane_div, key_stride, pa, va, pb, vb, P, C, lvl, iters};
    if (int e = by_dh<LaneSplit, float>(dh, p, levels - lvl, st)) return e;
    std::swap(pa, pb);
    std::swap(va, vb);
    if ((C >> lvl) <= ta::SUBTREE_SLOTS) break;  // the subtree kernel did every remaining level
  }
  if (pa != perm) {
    cudaMemcpyAsync(perm, pa, total * sizeof(int32_t), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(valid, va, total, cudaMemcpyDeviceToDevice, st);
    return check_launch("ta_lane_order");
  }
  return TA_OK;
}

// ta_lane_order for callers that may not allocate device memory: the second ping-pong buffer is the library's
// static scratch above instead of a caller buffer, its address looked up for the calling thread's current context.
int ta_lane_order_noalloc(const float* keys, int64_t key_lane_div, int64_t key_stride, const int64_t* n, int first,
                          int P, int C, int dh, int iters, int levels, int32_t* perm, uint8_t* valid, void* stream) {
  g_err.clear();
  if (P < 0 || C < 0 || (int64_t)P * C > kLaneScratchSlots)
    return fail(TA_ERR_ARG, "ta_lane_order_noalloc: P*C=%lld slots exceed the static scratch of %lld",
                (long long)P * C, (long long)kLaneScratchSlots);
  int32_t* pt = nullptr;
  uint8_t* vt = nullptr;
  if (int r = lane_scratch(S(stream), &pt, &vt)) return r;
  return ta_lane_order(keys, key_lane_div, key_stride, n, first, P, C, dh, iters, levels, perm, valid, pt, vt,
                       stream);
}

int ta_lane_sums(const float* keys, int64_t key_lane_div, int64_t key_stride, const int32_t* perm,
                 const uint8_t* valid, int P, int C, int dh, float* sums, int32_t* cnt, int32_t* slot, void* stream) {
  g_err.clear();
  const int lc = log2_exact(C);
  if (dh < 1 || dh > 128 || P < 0 || lc < 1) return fail(TA_ERR_ARG, "ta_lane_sums: bad sizes P=%d C=%d dh=%d", P, C, dh);
  if (key_lane_div < 1) return fail(TA_ERR_ARG, "ta_lane_sums: bad lane divisor");
  if (!keys || !perm || !valid || !sums || !cnt || !slot) return fail(TA_ERR_ARG, "ta_lane_sums: null pointer");
  if (P == 0) return TA_OK;
  ta::LaneSumsParams p{keys, key_lane_div, key_stride, perm, valid, P, C, lc - 1, dh, sums, cnt, slot};
  ta::lane_sums_kernel<<<(unsigned)P, 512, 0, S(stream)>>>(p);
  return check_launch("ta_lane_sums");
}

int ta_lane_insert(const float* kv, const int64_t* kpos, const uint8_t* active, int P, int C, int dh, float* sums,
                   int32_t* cnt, int32_t* slot, void* stream) {
  g_err.clear();
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_lane_insert: unsupported head dim %d", dh);
  const int lc = log2_exact(C);
  if (P < 0 || lc < 2) return fail(TA_ERR_ARG, "ta_lane_insert: C=%d is not a power of two >= 4", C);
  if (!kv || !kpos || !active || !sums || !cnt || !slot) return fail(TA_ERR_ARG, "ta_lane_insert: null pointer");
  ta::LaneInsertParams p{kv, kpos, active, P, lc - 1, C, sums, cnt, slot};
  return by_dh<LaneInsert, float>(dh, p, S(stream));
}

int ta_lane_select(const float* q, const float* k, const int64_t* lhat, int B, int H, int T, int dh, int chunk,
                   int wmax, int nb_window, int nb_store, int nb_probe, int nb_cap_min, float nb_rho, int neighbors,
                   float* sums, int32_t* cnt, int32_t* slot, int64_t* tree_pos, uint8_t* leaf_ok, int64_t* nb_pos,
                   int64_t* n_tree, int64_t* nb_leaves, void* stream) {
  g_err.clear();
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_lane_select: unsupported head dim %d", dh);
  const int lt = log2_exact(T);
  if (B < 0 || H < 0 || lt < 2 || chunk < 1 || T % chunk != 0)
    return fail(TA_ERR_ARG, "ta_lane_select: T=%d must be a power of two >= 4 and a multiple of chunk=%d", T, chunk);
  const int D = lt - 1;
  if (wmax < 1 || wmax > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_lane_select: wmax=%d outside [1, 64]", wmax);
  const int wl = std::min(wmax, 1 << D);
  if (nb_window < 1 || nb_store < 1 || nb_window * nb_store > 32 || nb_store > wl)
    return fail(TA_ERR_ARG, "ta_lane_select: nb_window * nb_store must be <= 32 and nb_store <= %d", wl);
  if (nb_probe < 0 || nb_cap_min < 0) return fail(TA_ERR_ARG, "ta_lane_select: bad neighbour probe / cap");
  if (!q || !k || !lhat || !sums || !cnt || !slot || !tree_pos || !leaf_ok || !nb_pos || !n_tree || !nb_leaves)
    return fail(TA_ERR_ARG, "ta_lane_select: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(sums))
    return fail(TA_ERR_ARG, "ta_lane_select: q / k / sums must be 16-byte aligned");
  ta::LaneSelectParams p{};
  p.q = q; p.k = k; p.lhat = lhat; p.sums = sums; p.cnt = cnt; p.slot = slot;
  p.B = B; p.H = H; p.T = T; p.Y = chunk; p.nl = T / chunk; p.D = D; p.wmax = wmax; p.wl = wl;
  p.Wn = nb_window; p.NS = nb_store; p.probe = std::min(nb_probe * nb_store, 32); p.cap_min = nb_cap_min;
  p.neighbors = neighbors; p.rho = nb_rho;
  p.tree_pos = tree_pos; p.leaf_ok = leaf_ok; p.nb_pos = nb_pos; p.n_tree = n_tree; p.nb_leaves = nb_leaves;
  return by_dh<LaneSelect, float>(dh, p, S(stream));
}

int ta_forest_levels(const void* k, int dtype, int P, int B, int dh, int depth, int nb, int zero_sink,
                     const int32_t* perm, int gate, float gate_q, float gate_temp, void* const* out, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_forest_levels: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_forest_levels: unsupported head dim %d", dh);
  if (P < 0 || nb < 1 || B < 4 || (B & (B - 1)) || (2 << depth) != B || depth + 1 > ta::FOREST_MAX_LEVELS)
    return fail(TA_ERR_ARG, "ta_forest_levels: B=%d must be a power of two in [4, 512] with depth=log2(B/2)", B);
  if (!k || !perm || !out) return fail(TA_ERR_ARG, "ta_forest_levels: null pointer");
  ta::ForestLevelsParams p{};
  p.k = k; p.perm = perm; p.P = P; p.B = B; p.depth = depth; p.nb = nb; p.zero_sink = zero_sink; p.gate = gate;
  p.gate_q = gate_q; p.gate_temp = gate_temp;
  for (int l = 0; l <= depth; ++l) {
    if (!out[l]) return fail(TA_ERR_ARG, "ta_forest_levels: null output level %d", l);
    p.out[l] = out[l];
  }
  return by_type_dh<ForestLevels>(dtype, dh, p, S(stream));
}

int ta_soft_gate(const void* sm, const void* grp, int dtype, int64_t N, int members, int dh, float gate_q,
                 float gate_temp, void* out, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_soft_gate: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_soft_gate: unsupported head dim %d", dh);
  if (N < 0 || members < 1) return fail(TA_ERR_ARG, "ta_soft_gate: bad sizes N=%lld S=%d", (long long)N, members);
  if (!sm || !grp || !out) return fail(TA_ERR_ARG, "ta_soft_gate: null pointer");
  return by_type_dh<SoftGate>(dtype, dh, sm, grp, out, N, members, gate_q, gate_temp, S(stream));
}

int ta_forest_select(const void* q, int dtype, int Bn, int H, int T, int dh, int64_t q_sb, int64_t q_sh,
                     int64_t q_st, const void* const* levels, const int32_t* perm, int B, int depth,
                     const int64_t* bq, int bq_const, int wmax, int64_t* leaf, uint8_t* leafv, int64_t* tkey,
                     uint8_t* tok, int32_t* const* lsel, uint8_t* const* lselv, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_forest_select: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_forest_select: unsupported head dim %d", dh);
  if (Bn < 0 || H < 0 || B < 4 || (B & (B - 1)) || (2 << depth) != B || depth + 1 > ta::FOREST_MAX_LEVELS ||
      T < B || T % B != 0)
    return fail(TA_ERR_ARG, "ta_forest_select: T=%d must be a multiple of the block B=%d (a power of two >= 4)", T, B);
  if (wmax < 1 || wmax > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_forest_select: wmax=%d outside [1, 64]", wmax);
  if (!q || !levels || !perm || !leaf || !leafv || !tkey || !tok) return fail(TA_ERR_ARG, "ta_forest_select: null pointer");
  ta::ForestSelectParams p{};
  p.q = q; p.q_sb = q_sb; p.q_sh = q_sh; p.q_st = q_st;
  for (int l = 0; l <= depth; ++l) {
    if (!levels[l]) return fail(TA_ERR_ARG, "ta_forest_select: null level %d", l);
    p.lv[l] = levels[l];
    p.lsel[l] = lsel ? lsel[l] : nullptr;
    p.lselv[l] = lselv ? lselv[l] : nullptr;
  }
  p.perm = perm; p.bq = bq; p.bq_const = bq_const;
  p.Bn = Bn; p.H = H; p.T = T; p.B = B; p.nb = T / B; p.depth = depth; p.wmax = wmax;
  int w = std::min(wmax, T / B);
  for (int l = 1; l <= depth; ++l) w = std::min(wmax, 2 * w);
  p.wl = w;
  p.leaf = leaf; p.leafv = leafv; p.tkey = tkey; p.tok = tok;
  return by_type_dh<ForestSelect>(dtype, dh, p, S(stream));
}

int ta_sparse_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                       const float* lse, int dtype, int B, int H, int T, int T_kv, int dh, const void* cand,
                       int cand64, int Kc, float scale, void* dq, float* dk, float* dv, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_sparse_attn_bwd: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_sparse_attn_bwd: unsupported head dim %d", dh);
  if (B < 0 || H < 0 || T < 0 || T_kv < 0 || Kc < 0) return fail(TA_ERR_ARG, "ta_sparse_attn_bwd: bad sizes");
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || (Kc > 0 && !cand))
    return fail(TA_ERR_ARG, "ta_sparse_attn_bwd: null pointer");
  for (const void* ptr : {q, k, v, o, dout, (const void*)dq, (const void*)dk, (const void*)dv})
    if (!aligned16(ptr)) return fail(TA_ERR_ARG, "ta_sparse_attn_bwd: tensors must be 16-byte aligned");
  ta::SparseAttnBwdParams p{};
  p.q = q; p.k = k; p.v = v; p.o = o; p.dout = dout; p.lse = lse;
  p.cand = cand; p.cand64 = cand64;
  p.B = B; p.H = H; p.T = T; p.Kc = Kc; p.T_kv = T_kv;
  p.scale = scale;
  p.dq = dq; p.dk = dk; p.dv = dv;
  return by_type_dh<SparseAttnBwd>(dtype, dh, p, S(stream));
}

int ta_gather_dot(const void* q, const void* Sn, int dtype, int B, int H, int N, int M, int C, int dh,
                  int64_t q_sb, int64_t q_sh, int64_t q_st, int64_t s_sb, int64_t s_sh, int64_t s_st,
                  const void* cand, int cand64, float scale, float* out, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_gather_dot: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_gather_dot: unsupported head dim %d", dh);
  if (M < 1 || C < 0) return fail(TA_ERR_ARG, "ta_gather_dot: bad sizes M=%d C=%d", M, C);
  if (!q || !Sn || !out || (C > 0 && !cand)) return fail(TA_ERR_ARG, "ta_gather_dot: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(q, es, {q_sb, q_sh, q_st}) || !rows_aligned(Sn, es, {s_sb, s_sh, s_st}))
    return fail(TA_ERR_ARG, "ta_gather_dot: q/S rows must be 16-byte aligned");
  ta::GatherDotParams p{q, q_sb, q_sh, q_st, Sn, s_sb, s_sh, s_st, cand, cand64, B, H, N, C, M, scale, out};
  return by_type_dh<GatherDot>(dtype, dh, p, S(stream));
}

int ta_gather_dot_blocks(const void* q, const void* k, int dtype, int B, int H, int T, int dh, int64_t q_sb,
                         int64_t q_sh, int64_t k_sb, int64_t k_sh, int64_t k_st, const int32_t* blocks, int nblk,
                         int blk, int nb_cta, float scale, float* out, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_gather_dot_blocks: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_gather_dot_blocks: unsupported head dim %d", dh);
  if (nblk < 0 || blk < 1 || nb_cta < 1 || nb_cta > 64)
    return fail(TA_ERR_ARG, "ta_gather_dot_blocks: bad sizes nblk=%d blk=%d nb_cta=%d", nblk, blk, nb_cta);
  if (!q || !k || !out || (nblk > 0 && !blocks)) return fail(TA_ERR_ARG, "ta_gather_dot_blocks: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(q, es, {q_sb, q_sh}) || !rows_aligned(k, es, {k_sb, k_sh, k_st}))
    return fail(TA_ERR_ARG, "ta_gather_dot_blocks: q/k rows must be 16-byte aligned");
  if (k_st != dh) return fail(TA_ERR_ARG, "ta_gather_dot_blocks: key rows of a block must be contiguous");
  ta::GatherDotBlocksParams p{q, q_sb, q_sh, k, k_sb, k_sh, k_st, blocks, B, H, T, nblk, blk, nb_cta, scale, out};
  return by_type_dh<GatherDotBlocks>(dtype, dh, p, S(stream));
}

int ta_dedupe(const int64_t* cand, const uint8_t* valid, uint8_t* keep, int64_t rows, int Kc, void* stream) {
  g_err.clear();
  if (rows < 0 || Kc < 0 || Kc > 6000) return fail(TA_ERR_ARG, "ta_dedupe: bad sizes rows=%lld Kc=%d", (long long)rows, Kc);
  if (rows == 0 || Kc == 0) return TA_OK;
  if (!cand || !valid || !keep) return fail(TA_ERR_ARG, "ta_dedupe: null pointer");
  ta::dedupe_kernel<<<(unsigned)rows, 128, (size_t)Kc * sizeof(int64_t), S(stream)>>>(cand, valid, keep, rows, Kc);
  return check_launch("ta_dedupe");
}

int ta_append(const void* k, const void* v, int dtype, int B, int H, int dh, int64_t k_sb, int64_t k_sh,
              int64_t v_sb, int64_t v_sh, void* kc, void* vc, int64_t c_sb, int64_t c_sh, int64_t c_st,
              float* nodes, int64_t n_sb, int64_t n_sh, int cap, int L0, int Lm, const int32_t* pos,
              void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_append: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_append: unsupported head dim %d", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if ((1 << L0) > ta::APPEND_SMEM_FLOATS) return fail(TA_ERR_ARG, "ta_append: leaf block too large");
  if (!k || !v || !kc || !vc || !nodes || !pos) return fail(TA_ERR_ARG, "ta_append: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(k, es, {k_sb, k_sh}) || !rows_aligned(v, es, {v_sb, v_sh}) ||
      !rows_aligned(kc, es, {c_sb, c_sh, c_st}) || !rows_aligned(vc, es, {c_sb, c_sh, c_st}))
    return fail(TA_ERR_ARG, "ta_append: rows must be 16-byte aligned");
  ta::AppendParams p{};
  p.k = k; p.v = v; p.k_sb = k_sb; p.k_sh = k_sh; p.v_sb = v_sb; p.v_sh = v_sh;
  p.kc = kc; p.vc = vc; p.c_sb = c_sb; p.c_sh = c_sh; p.c_st = c_st;
  p.nodes = nodes;
  p.lv = make_lv(nodes, n_sb, n_sh, cap, L0, Lm);
  p.pos = pos; p.B = B; p.H = H;
  return by_type_dh<Append>(dtype, dh, p, S(stream));
}

int ta_decode_default_splits(int B, int H, int dh, int dtype) {
  if (!valid_dtype(dtype) || dh < 1) return 1;
  return default_splits(B, H, dh * esize_of(dtype));
}

int ta_embed_ln(const void* wte, const void* wpe, int dtype, const int64_t* tok, const int32_t* pos, int B, int V,
                int P, int C, const float* w, float eps, float* x, void* h, void* stream) {
  g_err.clear();
  if (!wte || !wpe || !tok || !pos || !w || !x || !h) return fail(TA_ERR_ARG, "ta_embed_ln: null pointer");
  if (B < 0 || V < 1 || P < 1 || C < 1) return fail(TA_ERR_ARG, "ta_embed_ln: bad sizes");
  if (B == 0) return TA_OK;
  return rows_dispatch(dtype, 0, wte, wpe, tok, pos, B, V, P, C, w, eps, x, h, S(stream));
}

int ta_add_ln(float* x, const void* y, int dtype, int B, int C, const float* w, float eps, void* h, void* stream) {
  g_err.clear();
  if (!x || !w || !h) return fail(TA_ERR_ARG, "ta_add_ln: null pointer");
  if (B < 0 || C < 1) return fail(TA_ERR_ARG, "ta_add_ln: bad sizes");
  if (B == 0) return TA_OK;
  return rows_dispatch(dtype, 1, nullptr, y, nullptr, nullptr, B, 0, 0, C, w, eps, x, h, S(stream));
}

int ta_gelu(void* x, int dtype, int64_t n, void* stream) {
  g_err.clear();
  if (!x || n < 0 || n % 8 != 0 || !aligned16(x)) return fail(TA_ERR_ARG, "ta_gelu: bad arguments");
  if (n == 0) return TA_OK;
  const unsigned blocks = (unsigned)((n / 8 + 255) / 256);
  switch (dtype) {
    case TA_F32: ta::gelu_kernel<float><<<blocks, 256, 0, S(stream)>>>(reinterpret_cast<float*>(x), n); break;
    case TA_BF16: ta::gelu_kernel<__nv_bfloat16><<<blocks, 256, 0, S(stream)>>>(reinterpret_cast<__nv_bfloat16*>(x), n); break;
    case TA_F16: ta::gelu_kernel<__half><<<blocks, 256, 0, S(stream)>>>(reinterpret_cast<__half*>(x), n); break;
    default: return fail(TA_ERR_ARG, "ta_gelu: bad dtype %d", dtype);
  }
  return check_launch("ta_gelu");
}

int ta_argmax_advance(const void* logits, int dtype, int B, int V, int64_t* tok, int32_t* pos, void* stream) {
  g_err.clear();
  if (!logits || !tok || !pos) return fail(TA_ERR_ARG, "ta_argmax_advance: null pointer");
  if (B < 0 || V < 1) return fail(TA_ERR_ARG, "ta_argmax_advance: bad sizes");
  if (B == 0) return TA_OK;
  switch (dtype) {
    case TA_F32: ta::argmax_advance_kernel<float><<<B, ta::ARG_THREADS, 0, S(stream)>>>(reinterpret_cast<const float*>(logits), V, tok, pos); break;
    case TA_BF16: ta::argmax_advance_kernel<__nv_bfloat16><<<B, ta::ARG_THREADS, 0, S(stream)>>>(reinterpret_cast<const __nv_bfloat16*>(logits), V, tok, pos); break;
    case TA_F16: ta::argmax_advance_kernel<__half><<<B, ta::ARG_THREADS, 0, S(stream)>>>(reinterpret_cast<const __half*>(logits), V, tok, pos); break;
    default: return fail(TA_ERR_ARG, "ta_argmax_advance: bad dtype %d", dtype);
  }
  return check_launch("ta_argmax_advance");
}

int ta_linear_supported(int dtype, int B, int N, int K, int splits) {
  if (dtype != TA_BF16 && dtype != TA_F16) return 0;
  if (B < 1 || B > ta::LIN_MAX_BN || N < 8 || N % 8 != 0 || K < ta::LIN_KB || splits < 1) return 0;
  if (K % (ta::LIN_KB * splits) != 0) return 0;
  return linear_shape((B + 15) / 16 * 16, K / splits).nst > 0 ? 1 : 0;
}

int ta_linear_rows(const void* act, int64_t act_ld, int dtype, int B, int N, int K, const void* w, int splits, int mode,
                   void* out, int64_t out_ld, float* part, unsigned long long* keys, float* ws, int* counters,
                   void* stream) {
  g_err.clear();
  if (dtype != TA_BF16 && dtype != TA_F16) return fail(TA_ERR_ARG, "ta_linear_rows: bf16 or f16 operands only");
  if (B < 1 || B > ta::LIN_MAX_BN || N < 8 || N % 8 != 0 || K < ta::LIN_KB || splits < 1)
    return fail(TA_ERR_ARG, "ta_linear_rows: bad sizes B=%d (1..%d) N=%d (a multiple of 8) K=%d splits=%d", B,
                ta::LIN_MAX_BN, N, K, splits);
  if (K % (ta::LIN_KB * splits) != 0)
    return fail(TA_ERR_ARG, "K=%d is not a multiple of %d x splits (splits=%d)", K, ta::LIN_KB, splits);
  if (mode < ta::LIN_STORE || mode > ta::LIN_ARGMAX) return fail(TA_ERR_ARG, "ta_linear_rows: bad mode %d", mode);
  if (mode != ta::LIN_PARTIAL && splits > 1 && (!ws || !counters || !aligned16(ws)))
    return fail(TA_ERR_ARG, "ta_linear_rows: mode %d with %d K splits needs the workspace and counters", mode, splits);
  if (!act || !w) return fail(TA_ERR_ARG, "ta_linear_rows: null pointer");
  if (!aligned16(act) || act_ld < K || act_ld % 8 != 0 || !aligned16(w))
    return fail(TA_ERR_ARG, "ta_linear_rows: rows and weight must be 16-byte aligned with a row stride of >= K, a "
                "multiple of 8 elements");
  if (mode == ta::LIN_PARTIAL ? (!part || !aligned16(part)) : (!out || out_ld < N || out_ld % 8 != 0 || !aligned16(out)))
    return fail(TA_ERR_ARG, "ta_linear_rows: missing, short or unaligned output for mode %d (16-byte aligned rows)",
                mode);
  if (mode == ta::LIN_ARGMAX && !keys) return fail(TA_ERR_ARG, "ta_linear_rows: ARGMAX needs the key buffer");
  const int BN = (B + 15) / 16 * 16, Ks = K / splits;
  const LinShape sh = linear_shape(BN, Ks);
  if (sh.nst == 0)
    return fail(TA_ERR_ARG, "ta_linear_rows: %d rows x %d of K per CTA do not fit in shared memory (use more splits)",
                B, Ks);
  const size_t smem = ta::linear_smem_bytes(BN, Ks, sh.nst, sh.nb);
  CUtensorMap tw, trows;
  if (int r = make_blocks_map(&tw, w, dtype, N, K, K, ta::LIN_MT, sh.nb, "weight")) return r;
  if (int r = make_blocks_map(&trows, act, dtype, B, K, act_ld, BN, sh.na, "rows")) return r;
  ta::LinearParams p{};
  p.B = B;
  p.BN = BN;
  p.N = N;
  p.K = K;
  p.Ks = Ks;
  p.nb = sh.nb;
  p.na = sh.na;
  p.nst = sh.nst;
  p.out = out;
  p.out_ld = out_ld;
  p.part = part;
  p.keys = keys;
  p.ws = ws;
  p.counters = counters;
  const dim3 grid((unsigned)ta::ceil_div(N, ta::LIN_MT), (unsigned)splits);
  return dtype == TA_BF16 ? launch_linear_mode<__nv_bfloat16>(mode, tw, trows, p, grid, smem, S(stream))
                          : launch_linear_mode<__half>(mode, tw, trows, p, grid, smem, S(stream));
}

int ta_add_splits_ln(float* x, const float* part, int splits, int dtype, int B, int C, const float* w, float eps,
                     void* h, void* stream) {
  g_err.clear();
  if (!x || !part || !w || !h) return fail(TA_ERR_ARG, "ta_add_splits_ln: null pointer");
  if (dtype != TA_BF16 && dtype != TA_F16) return fail(TA_ERR_ARG, "ta_add_splits_ln: bf16 or f16 rows only");
  if (B < 0 || C < 8 || C % 8 != 0 || splits < 1 || !aligned16(x) || !aligned16(part) || !aligned16(h))
    return fail(TA_ERR_ARG, "ta_add_splits_ln: bad sizes or alignment (C a multiple of 8, 16-byte aligned rows)");
  if (B == 0) return TA_OK;
  if (C > 8 * 256) return fail(TA_ERR_ARG, "ta_add_splits_ln: row width %d above 2048", C);
  const dim3 grid((unsigned)B), block((unsigned)(((C / 8) + 31) / 32 * 32));
  cudaStream_t st = S(stream);
  cudaError_t e;
  if (dtype == TA_BF16)
    e = launch_pdl(ta::add_splits_ln_kernel<__nv_bfloat16>, grid, block, 0, st, x, part, splits, B, C, w, eps,
                   reinterpret_cast<__nv_bfloat16*>(h));
  else
    e = launch_pdl(ta::add_splits_ln_kernel<__half>, grid, block, 0, st, x, part, splits, B, C, w, eps,
                   reinterpret_cast<__half*>(h));
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_add_splits_ln: launch failed: %s", cudaGetErrorString(e));
  return check_launch("ta_add_splits_ln");
}

int ta_argmax_finish(const unsigned long long* keys, int n_tiles, int B, int V, int64_t* tok, int32_t* pos,
                     void* stream) {
  g_err.clear();
  if (!keys || !tok || !pos) return fail(TA_ERR_ARG, "ta_argmax_finish: null pointer");
  if (B < 0 || n_tiles < 1 || V < 1) return fail(TA_ERR_ARG, "ta_argmax_finish: bad sizes");
  if (B == 0) return TA_OK;
  const cudaError_t e = launch_pdl(ta::argmax_finish_kernel, dim3((unsigned)((B + 3) / 4)), dim3(128), 0, S(stream),
                                   keys, n_tiles, B, V, tok, pos);
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "ta_argmax_finish: launch failed: %s", cudaGetErrorString(e));
  return check_launch("ta_argmax_finish");
}

#ifdef TA_TAIL_TRACE
// Profiling build only: the block tail's phase timestamps (256 x 32 uint64) to host memory.
int ta_tail_trace_read(void* host) {
  const cudaError_t e = cudaMemcpyFromSymbol(host, ta::g_tail_trace, sizeof(ta::g_tail_trace));
  return e == cudaSuccess ? TA_OK : fail(TA_ERR_CUDA, "ta_tail_trace_read: %s", cudaGetErrorString(e));
}
#endif

int ta_block_tail_plan(int dtype, int B, int C, int with_qkv, int64_t* ws_bytes, int* sync_words) {
  g_err.clear();
  if (dtype != TA_BF16 && dtype != TA_F16) return fail(TA_ERR_ARG, "ta_block_tail: bf16 or f16 weights only");
  TailPlan pl;
  if (!tail_plan(B, C, with_qkv != 0, 2, pl))
    return fail(TA_ERR_ARG, "ta_block_tail: %d rows of width %d not taken (1..%d rows, width a multiple of 128 up to "
                "%d whose weight slices fit one CTA per SM)", B, C, ta::BT_MAX_BN, ta::BT_MAX_C);
  if (ws_bytes) *ws_bytes = (int64_t)pl.ws_bytes;
  if (sync_words) *sync_words = pl.nsync;
  return TA_OK;
}

int ta_block_tail(const void* att, float* x, const void* w_proj, const float* ln2_w, const void* w_fc,
                  const void* w_mlp, const float* ln_next_w, const void* w_qkv, float eps, int dtype, int B, int C,
                  void* h, void* qkv, void* ws, int64_t ws_bytes, int* sync, void* stream) {
  g_err.clear();
  if (dtype != TA_BF16 && dtype != TA_F16) return fail(TA_ERR_ARG, "ta_block_tail: bf16 or f16 weights only");
  if (!att || !x || !w_proj || !ln2_w || !w_fc || !w_mlp || !ln_next_w || !h || !ws || !sync)
    return fail(TA_ERR_ARG, "ta_block_tail: null pointer");
  if ((w_qkv == nullptr) != (qkv == nullptr))
    return fail(TA_ERR_ARG, "ta_block_tail: the next block's c_attn weight and its output go together");
  const bool with_qkv = w_qkv != nullptr;
  TailPlan pl;
  if (!tail_plan(B, C, with_qkv, 2, pl))
    return fail(TA_ERR_ARG, "ta_block_tail: %d rows of width %d not taken (1..%d rows, width a multiple of 128 up to "
                "%d whose weight slices fit one CTA per SM)", B, C, ta::BT_MAX_BN, ta::BT_MAX_C);
  if (ws_bytes < (int64_t)pl.ws_bytes)
    return fail(TA_ERR_ARG, "ta_block_tail: workspace of %lld B, the plan needs %zu B", (long long)ws_bytes,
                pl.ws_bytes);
  for (const void* q : {att, (const void*)x, w_proj, w_fc, w_mlp, (const void*)h, (const void*)ws})
    if (!aligned16(q)) return fail(TA_ERR_ARG, "ta_block_tail: rows, weights and workspace must be 16-byte aligned");
  if (with_qkv && (!aligned16(qkv) || !aligned16(w_qkv)))
    return fail(TA_ERR_ARG, "ta_block_tail: rows, weights and workspace must be 16-byte aligned");
  ta::TailMaps m;
  unsigned char* wsb = reinterpret_cast<unsigned char*>(ws);
  const void* wts[4] = {w_proj, w_fc, w_mlp, with_qkv ? w_qkv : w_proj};
  const void* rows[4] = {att, wsb + pl.o_h2, wsb + pl.o_fc, with_qkv ? h : att};
  const char* names[4] = {"c_proj weight", "c_fc weight", "c_mlp weight", "c_attn weight"};
  const char* rnames[4] = {"attention rows", "ln_2 rows", "GELU rows", "ln_1 rows"};
  for (int i = 0; i < 4; ++i) {
    const ta::TailGemm& g = pl.g[i == 3 && !with_qkv ? 0 : i];
    if (int r = make_blocks_map(&m.w[i], wts[i], dtype, g.N, g.K, g.K, ta::LIN_MT, 1, names[i])) return r;
    if (int r = make_blocks_map(&m.a[i], rows[i], dtype, B, g.K, g.K, pl.BN, 1, rnames[i])) return r;
  }
  ta::BlockTailParams p{};
  p.B = B;
  p.BN = pl.BN;
  p.C = C;
  p.G = num_sms();
  p.nslot = pl.nslot;
  for (int i = 0; i < 4; ++i) p.g[i] = pl.g[i];
  p.off_ln = pl.off_ln;
  p.nsync = pl.nsync;
  p.att = att;
  p.x = x;
  p.ln2 = ln2_w;
  p.ln_next = ln_next_w;
  p.eps = eps;
  p.part_proj = reinterpret_cast<float*>(wsb + pl.o_part_proj);
  p.ws_fc = reinterpret_cast<float*>(wsb + pl.o_ws_fc);
  p.part_mlp = reinterpret_cast<float*>(wsb + pl.o_part_mlp);
  p.ws_qkv = reinterpret_cast<float*>(wsb + pl.o_ws_qkv);
  p.h2 = wsb + pl.o_h2;
  p.fc = wsb + pl.o_fc;
  p.h = h;
  p.qkv = qkv;
  p.sync = sync;
  return dtype == TA_BF16 ? launch_tail_by_c<__nv_bfloat16>(pl.maxc, m, p, pl.smem, S(stream))
                          : launch_tail_by_c<__half>(pl.maxc, m, p, pl.smem, S(stream));
}

int ta_decode_step(const void* qkv, int dtype, int B, int H, int dh, int64_t qkv_sb, int64_t k_ofs, int64_t v_ofs,
                   void* kc, void* vc, int64_t c_sb, int64_t c_sh, int64_t c_st, float* nodes, int64_t n_sb,
                   int64_t n_sh, int cap, int L0, int Lm, const int32_t* pos, int wmax, int n_tree, int Lw,
                   float scale, void* out, int64_t o_sb, float* lse, int32_t* nkeys, int32_t* sel, int splits,
                   float* part, int32_t* part_cnt, void* stream) {
  g_err.clear();
  if (!valid_dtype(dtype)) return fail(TA_ERR_ARG, "ta_decode_step: bad dtype %d", dtype);
  if (!valid_dh(dh)) return fail(TA_ERR_ARG, "ta_decode_step: unsupported head dim %d", dh);
  if (int r = check_levels(cap, L0, Lm)) return r;
  if (wmax < 1 || wmax > ta::WMAX_LIMIT) return fail(TA_ERR_ARG, "ta_decode_step: wmax=%d outside [1, 64]", wmax);
  if (n_tree < 0) return fail(TA_ERR_ARG, "ta_decode_step: n_tree < 0");
  if (Lw < 1) return fail(TA_ERR_ARG, "ta_decode_step: window %d < 1", Lw);
  if (splits == 0) splits = default_splits(B, H, dh * esize_of(dtype));
  if (splits < -1 || splits > 8) return fail(TA_ERR_ARG, "ta_decode_step: splits=%d outside [-1, 8]", splits);
  if (!qkv || !kc || !vc || !nodes || !pos || !out) return fail(TA_ERR_ARG, "ta_decode_step: null pointer");
  const int es = esize_of(dtype);
  if (!rows_aligned(qkv, es, {qkv_sb, k_ofs, v_ofs, (int64_t)dh}) || !rows_aligned(kc, es, {c_sb, c_sh, c_st}) ||
      !rows_aligned(vc, es, {c_sb, c_sh, c_st}) || !rows_aligned(out, es, {o_sb, (int64_t)dh}))
    return fail(TA_ERR_ARG, "ta_decode_step: rows must be 16-byte aligned");
  if (!aligned16(nodes) || (n_sb * 4) % 16 || (n_sh * 4) % 16)
    return fail(TA_ERR_ARG, "ta_decode_step: node rows must be 16-byte aligned");
  if (B * H > 65535) return fail(TA_ERR_ARG, "ta_decode_step: B*H=%d above 65535", B * H);
  ta::DecodeParams p{};
  p.qkv = qkv; p.qkv_sb = qkv_sb; p.k_ofs = k_ofs; p.v_ofs = v_ofs;
  p.kc = kc; p.vc = vc; p.c_sb = c_sb; p.c_sh = c_sh; p.c_st = c_st;
  p.nodes = nodes;
  p.lv = make_lv(nodes, n_sb, n_sh, cap, L0, Lm);
  p.pos = pos; p.B = B; p.H = H; p.wmax = wmax; p.n_tree = n_tree; p.Lw = Lw;
  p.scale = scale;
  p.out = out; p.o_sb = o_sb;
  p.lse = lse; p.nkeys = nkeys; p.sel = sel;
  p.splits = splits;
  p.psplit = 1;
  p.part = part;
  p.part_cnt = part_cnt;
  return by_type_dh<Decode>(dtype, dh, p, S(stream));
}

}  // extern "C"
