// tcgen05 building blocks shared by the skinny GEMM (gemm_tc.cu) and the
// fused-layer kernel (fused_layer.cu): tile constants, shared-memory
// descriptors, MMA issue / commit, TMEM loads and the stream-K bookkeeping.
#pragma once

#include "common.cuh"

namespace tsds {
namespace tc {

constexpr int BK = 64;                     // k per stage: one 128-byte swizzle row
constexpr int TILE_J = 128;                // MMA M
constexpr int A_STAGE = TILE_J * BK * 2;   // 16 KB
constexpr int MAX_STAGES = 16;

// ---- tcgen05 / descriptor helpers ------------------------------------------
// Shared-memory matrix descriptor: K-major operand in 128-byte-swizzled
// rows, 8-row core groups 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// ---- stream-K bookkeeping ---------------------------------------------------
// 32-bit arithmetic: W * P < 2^32 is checked on the host.
__device__ __forceinline__ int it_begin(int p, int P, uint32_t W) { return (int)(((uint32_t)p * W) / (uint32_t)P); }

// CTA whose range holds iteration x
__device__ __forceinline__ int owner_of(int x, int P, uint32_t W) {
  int q = (int)(((uint32_t)x * (uint32_t)P) / W);
  if (q > P - 1) q = P - 1;
  while (q + 1 < P && it_begin(q + 1, P, W) <= x) ++q;
  while (q > 0 && it_begin(q, P, W) > x) --q;
  return q;
}

// Whether unit q's range holds two split tiles (its first and its last tile
// are both cut by a range boundary).
__device__ __forceinline__ bool two_split(int q, int P, uint32_t W, int KT) {
  const int qb = it_begin(q, P, W), qe = it_begin(q + 1, P, W);
  if (qe <= qb) return false;
  const int f = qb / KT, l = (qe - 1) / KT;
  return f != l && owner_of(f * KT, P, W) != owner_of(f * KT + KT - 1, P, W) &&
         owner_of(l * KT, P, W) != owner_of(l * KT + KT - 1, P, W);
}

// Units that sum the partials of the split tile starting at iteration tb,
// whose contributors are q_lo..q_hi: all of them except q_hi when q_hi holds
// two split tiles (it sums a slice of its last tile only, so no unit reduces
// twice).  The reducers are q_lo .. q_lo + result - 1.
__device__ __forceinline__ int split_reducers(int q_lo, int q_hi, int P, uint32_t W, int KT) {
  return q_hi - q_lo + 1 - ((q_hi != q_lo && two_split(q_hi, P, W, KT)) ? 1 : 0);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---- CTA pair (cta_group::2) ---------------------------------------------
// A pair of CTAs on two SMs computes one 256-row tile: each CTA stages its
// own 128 weight rows and half of the token rows, the leader (cluster rank 0)
// issues the MMA for both, and each CTA's TMEM holds its 128 rows x N.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

// completion of the pair's MMAs, arriving on the barrier at this offset in both CTAs
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// TMA tile load into this CTA's shared memory, its bytes counted on the pair
// leader's barrier (bar: shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// arrive on an mbarrier of another CTA of the cluster (bar: shared::cluster address)
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Abort paths only: the MMA-issuing thread commits every tcgen05 operation
// it has issued to `bar` (count 1, used for nothing else, phase 0) and
// waits, bounded, until the tensor cores are done with TMEM and shared
// memory.  CG = 2: the pair's MMAs, the commit arriving in both CTAs.
template <int CG>
__device__ __forceinline__ void drain_mma(uint64_t* bar, uint64_t limit_ns = 20000000ull) {
  if constexpr (CG == 2)
    umma_commit_pair(bar);
  else
    umma_commit(bar);
  mbar_wait(bar, 0, limit_ns);
}

}  // namespace tc
}  // namespace tsds
