// Layout of a peer buffer and the device side of the cross-rank flag
// protocol, shared by the standalone all-reduce (peer.cu) and the all-reduce
// phase of the fused-layer kernel (fused_layer.cu).
//
//   [0, 2 KB)       counters[PEER_MAX_CTAS]         u32  this rank's per-CTA call count
//   [2 KB, 18 KB)   flags[PEER_MAX_CTAS][8]         u32  flags[b][p] written by rank p
//   [32 KB, ...)    slot 0, slot 1: max_elems fp32 each
//   then            published: max_elems bf16 - the two-shot all-reduce's
//                   final values of this rank's chunk
//   then            exchange: exchange_bytes - a vocab-parallel LM head's
//                   argmax candidates and logits shard (tsds_peer_lm_gather)
#pragma once

#include "common.cuh"

namespace tsds {
namespace peer {

constexpr int PEER_MAX_CTAS = 512;
constexpr int PEER_MAX_RANKS = 8;
constexpr size_t PEER_FLAGS_OFF = 2048;
constexpr size_t PEER_HEADER_BYTES = 32768;
constexpr uint64_t PEER_WAIT_NS = 1000000000ull;

static_assert(PEER_MAX_CTAS * 4 <= PEER_FLAGS_OFF, "counters overlap the flags");
static_assert(PEER_FLAGS_OFF + PEER_MAX_CTAS * PEER_MAX_RANKS * 4 <= PEER_HEADER_BYTES, "flags overlap slot 0");

__host__ __device__ inline size_t slot_bytes(int max_elems) { return ((size_t)max_elems * 4 + 255) / 256 * 256; }
__host__ __device__ inline size_t slot_offset(int max_elems, int slot) {
  return PEER_HEADER_BYTES + (size_t)(slot & 1) * slot_bytes(max_elems);
}
__host__ __device__ inline size_t published_offset(int max_elems) {
  return PEER_HEADER_BYTES + 2 * slot_bytes(max_elems);
}
__host__ __device__ inline size_t exchange_offset(int max_elems) {
  return published_offset(max_elems) + ((size_t)max_elems * 2 + 255) / 256 * 256;
}
__host__ __device__ inline size_t buffer_bytes(int max_elems, size_t exchange_bytes) {
  return exchange_offset(max_elems) + (exchange_bytes + 255) / 256 * 256;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Peer data is read with volatile loads: never served from a stale cached line.
__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Wait (bounded) until the flag at f has reached epoch e; a rank can be at
// most one call ahead of another, hence the wrap-safe `>=`.
__device__ __forceinline__ bool wait_flag(const uint32_t* f, uint32_t e) {
  if ((int)(ld_acquire_sys(f) - e) >= 0) return true;
  const uint64_t t0 = global_ns();
  while ((int)(ld_acquire_sys(f) - e) < 0) {
    if (global_ns() - t0 > PEER_WAIT_NS) return false;
  }
  return true;
}

}  // namespace peer
}  // namespace tsds
