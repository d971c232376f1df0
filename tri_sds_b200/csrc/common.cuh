// Shared device helpers for libtsds (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "../../include/tsds.h"

typedef __nv_bfloat16 bf16;

#define TSDS_RETURN_IF(cond, code) \
  do {                             \
    if (cond) return (code);       \
  } while (0)

void tsds_count_launch();

// Map the launch's own error (not a sticky earlier one) to a status code;
// every kernel launch in the library is followed by exactly one call.
static inline int tsds_launch_status() {
  tsds_count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TSDS_OK : TSDS_E_LAUNCH;
}

static inline bool tsds_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Host-side state of the library is safe under calls from several host
// threads at once (the ABI allows concurrent calls on different streams):
// per-device "done" records are atomics, and the small lookup caches of
// occupancy results take this process-wide lock.
std::mutex& tsds_host_cache_lock();

// Raise a kernel's dynamic shared-memory limit on the current device, once per
// device (the attribute is per device): `done` is the caller's per-kernel record.
// Two threads may both set it the first time; the attribute is the same.
constexpr int TSDS_MAX_DEVICES = 64;
typedef std::atomic<bool> tsds_device_flags[TSDS_MAX_DEVICES];
template <typename Kernel>
static inline int tsds_smem_limit_once(Kernel kernel, int bytes, tsds_device_flags& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= TSDS_MAX_DEVICES) {
    cudaGetLastError();
    return TSDS_E_DEVICE;
  }
  if (!done[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
      cudaGetLastError();
      return TSDS_E_LAUNCH;
    }
    done[dev].store(true, std::memory_order_release);
  }
  return TSDS_OK;
}

// Programmatic dependent launch: every kernel of the library is launched so
// that it may start while the previous kernel in the stream drains; each
// kernel executes griddepcontrol.wait before touching memory the previous
// kernels write.  Each executes griddepcontrol.launch_dependents first (the
// GEMM after its setup), so the next kernel is launched as soon as all of
// this one's CTAs run and its CTAs take SMs as they free up: a GEMM after a
// small kernel streams its first weight tiles while that kernel runs.  This
// is safe because every kernel waits before it reads or writes anything an
// earlier kernel touches (the GEMM reads only its weights before the wait),
// and no kernel completes before its own wait has returned, so a wait covers
// every earlier kernel of the stream, not only the previous one.
// tsds_set_pdl(0) turns the attribute off.
int tsds_pdl_enabled();

template <typename... KArgs, typename... Args>
static inline void tsds_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = tsds_pdl_enabled() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with a thread-block cluster of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
static inline void tsds_launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                       cudaStream_t stream, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = tsds_pdl_enabled() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

namespace tsds {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// bf16 pairs packed in a 32-bit word -> fp32 (exact).
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf2f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ bf16 f2bf(float x) { return __float2bfloat16_rn(x); }
// Round an fp32 value to the nearest bf16 and back (the reference's bf16 tensor ops).
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed fp32 FMA (sm_100): (a.x*b.x + c.x, a.y*b.y + c.y).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t ra, rb, rc;
  asm("mov.b64 %0, {%1,%2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1,%2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1,%2};" : "=l"(rc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(rc) : "l"(ra), "l"(rb));
  float2 r;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(rc));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Read-only 16-byte global load through the non-coherent path.
__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Streaming 16-byte load: weights are read once per launch, keep them out of L1.
__device__ __forceinline__ uint4 ldg16_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ----------------------------------------------------------------------------
// mbarrier / TMA helpers (PTX).  Every wait is bounded: after `limit` polls
// it returns false and the caller records TSDS_E_TIMEOUT and bails out.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after `limit_ns` of wall time
// (default 2 s, far above any legitimate wait in these kernels).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, phase)) {
    if (global_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// Abort paths only: a CTA that gave up on a wait still lets the TMA copies it
// has in flight land before it frees TMEM or exits.  `full` is a ring of
// `stages` barriers with one expect_tx per issued stage (ring index j uses
// barrier j % stages, phase j / stages); only the last min(issued, stages)
// issues can still be pending.  Bounded by `limit_ns` in total: a stage whose
// bytes never arrive (its barrier never completes) costs at most that.
__device__ __forceinline__ void drain_tma_ring(uint64_t* full, int stages, int issued,
                                               uint64_t limit_ns = 20000000ull) {
  const uint64_t t0 = global_ns();
  for (int j = issued > stages ? issued - stages : 0; j < issued; ++j) {
    while (!mbar_try_wait(&full[j % stages], (uint32_t)(j / stages) & 1u)) {
      if (global_ns() - t0 > limit_ns) return;
    }
  }
}

// 2-D TMA tile load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

}  // namespace tsds

// ----------------------------------------------------------------------------
// Host: tensor-map encoding through the runtime's driver entry point (no
// direct libcuda link).
// ----------------------------------------------------------------------------
int tsds_make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                           int swizzle_128b);
