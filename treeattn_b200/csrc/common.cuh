// Shared device helpers for the treeattn_b200 kernels (sm_100a only).
//
// Everything in this library is one translation unit (treeattn_b200.cu includes the kernel headers), so
// the device error record below is a single symbol that every kernel writes to and the host reads back.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#ifndef TA_WAIT_LIMIT_NS
// Every spin on an mbarrier or a cluster barrier gives up after this many nanoseconds of wall time
// (read from %globaltimer), records an error and lets the kernel return. No correct launch waits this long.
#define TA_WAIT_LIMIT_NS 2000000000ull
#endif

namespace ta {

// ------------------------------------------------------------------------------------------------ errors
enum DevErrCode : int {
  DEV_OK = 0,
  DEV_WAIT_TIMEOUT = 1,     // an mbarrier / cluster wait ran past TA_WAIT_LIMIT_NS
  DEV_POS_RANGE = 2,        // a query position outside [0, capacity)
  DEV_INDEX_RANGE = 3,      // a candidate / block index outside its extent
};

// code, kernel id, detail a, detail b. The first error wins (atomicCAS on code).
__device__ int g_dev_err[4];

__device__ __forceinline__ void record_error(int code, int kernel, int a, int b) {
  if (atomicCAS(&g_dev_err[0], 0, code) == 0) {
    g_dev_err[1] = kernel;
    g_dev_err[2] = a;
    g_dev_err[3] = b;
    __threadfence();
  }
}

enum KernelId : int {
  K_BUILD_LEVELS = 1,
  K_SELECT = 2,
  K_SEG_ATTN = 3,
  K_SPARSE_ATTN = 4,
  K_GATHER_DOT = 5,
  K_GATHER_DOT_BLOCKS = 6,
  K_DEDUPE = 7,
  K_APPEND = 8,
  K_DECODE = 9,
  K_FINISH = 10,
  K_ROWS = 11,
  K_PREFILL = 12,
  K_WAIT_PROBE = 13,
};

// ------------------------------------------------------------------------------------------------ types
template <typename T> struct TypeInfo;
template <> struct TypeInfo<float> { static constexpr int VEC = 4; };            // 16 B = 4 floats
template <> struct TypeInfo<__nv_bfloat16> { static constexpr int VEC = 8; };    // 16 B = 8 bf16
template <> struct TypeInfo<__half> { static constexpr int VEC = 8; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Load 16 bytes (one VEC-wide chunk of T) and widen to fp32.
template <typename T>
__device__ __forceinline__ void load_vec_f32(const T* p, float* out);

template <>
__device__ __forceinline__ void load_vec_f32<float>(const float* p, float* out) {
  float4 v = *reinterpret_cast<const float4*>(p);
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}
template <>
__device__ __forceinline__ void load_vec_f32<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    out[2 * i] = f.x; out[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec_f32<__half>(const __half* p, float* out) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    out[2 * i] = f.x; out[2 * i + 1] = f.y;
  }
}

// Same, through the read-only / non-coherent path for data this kernel never writes.
template <typename T>
__device__ __forceinline__ void ldg_vec_f32(const T* p, float* out) {
  uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  load_vec_f32<T>(reinterpret_cast<const T*>(&v), out);
}

// Store VEC fp32 values as one 16-byte chunk of T.
template <typename T>
__device__ __forceinline__ void store_vec_from_f32(T* p, const float* in);

template <>
__device__ __forceinline__ void store_vec_from_f32<float>(float* p, const float* in) {
  *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
}
template <>
__device__ __forceinline__ void store_vec_from_f32<__nv_bfloat16>(__nv_bfloat16* p, const float* in) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = v;
}
template <>
__device__ __forceinline__ void store_vec_from_f32<__half>(__half* p, const float* in) {
  uint4 v;
  __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = v;
}

// ------------------------------------------------------------------------------------------------ warp
__device__ __forceinline__ float warp_sum_sub(float v, int width) {
  // butterfly sum over aligned groups of `width` lanes (width a power of two <= 32)
  for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------ mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Invalidates an mbarrier so its shared memory can be reused for something else; no thread may be waiting on it or
// arrive at it afterwards.
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread is parked by the hardware until the phase completes (or
// the hint, in ns, runs out) instead of spinning and taking issue slots from the warps doing the work.
constexpr uint32_t TA_SUSPEND_HINT_NS = 0x989680u;  // 10 ms

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(TA_SUSPEND_HINT_NS)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (after recording DEV_WAIT_TIMEOUT) if the phase does not complete within limit_ns.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int kernel, int where,
                                                  uint64_t limit_ns = TA_WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 3u) == 0 && global_timer_ns() - t0 > limit_ns) {
      record_error(DEV_WAIT_TIMEOUT, kernel, where, (int)parity);
      return false;
    }
  }
}

// The same bounded wait by polling (mbarrier.test_wait: the thread never suspends), for a wait on the critical path
// whose phase completes within microseconds.
__device__ __forceinline__ bool mbar_poll_bounded(uint64_t* bar, uint32_t parity, int kernel, int where,
                                                  uint64_t limit_ns = TA_WAIT_LIMIT_NS) {
  uint32_t ok;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t spins = 0;; ++spins) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((spins & 63u) == 63u && global_timer_ns() - t0 > limit_ns) {
      record_error(DEV_WAIT_TIMEOUT, kernel, where, (int)parity);
      return false;
    }
  }
}

// The bounded wait's failure path, on purpose: thread 0 waits on an mbarrier that no thread arrives at, gives up
// after limit_ns and records DEV_WAIT_TIMEOUT (kernel K_WAIT_PROBE, where = 7). Once no thread waits any more the
// abandoned barrier is invalidated (what a give-up path must do before its shared memory is reused), and the
// kernel ends normally.
__global__ void wait_probe_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, K_WAIT_PROBE, 7, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) mbar_inval(&bar);
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on `bar` (bytes multiple of 16,
// both addresses 16-byte aligned), one destination CTA.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same with an L2 eviction-priority hint (streamed data that is not re-read this step).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ------------------------------------------------------------------------------------------------ dependent launch
// Programmatic dependent launch: wait until the grid this one depends on has completed and its memory is visible
// (a no-op when the kernel was launched without the attribute) / let the grids that depend on this one start
// launching (they still wait for its completion before reading what it writes).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------ cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier (all threads of all CTAs, warp-convergent), release/acquire so that shared-memory writes
// made before it are visible to remote readers after it. barrier.cluster has no try form; every thread of every
// CTA in this library reaches each cluster barrier unconditionally (error paths included), so no arrival is
// ever skipped.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Named CTA barriers (ids 1..15), executed warp-convergently.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Address of the same shared-memory variable in CTA `rank` of this cluster (generic address usable by ld).
template <typename T>
__device__ __forceinline__ const T* cluster_map(const T* p, uint32_t rank) {
  uint64_t out;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<const T*>(out);
}

// ------------------------------------------------------------------------------------------------ misc
__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Total order used by every top-k in this library: higher score first, ties broken by the smaller node id.
// NaN scores rank as -inf so that ranks stay distinct.
__device__ __forceinline__ float rank_key(float s) { return (s != s) ? -INFINITY : s; }
__device__ __forceinline__ bool better(float sa, int ia, float sb, int ib) {
  return sa > sb || (sa == sb && ia < ib);
}

}  // namespace ta
