// One-shot all-reduce of row-parallel partials over NVLink peer memory, fused
// with the residual add.
//
// Every rank owns one peer buffer (cudaMalloc'd here, shared with the other
// ranks of the node through CUDA IPC; layout in peer.cuh).
//
// A row-parallel projection writes its fp32 partial [M][N] into this rank's
// slot (calls alternate slots 0 / 1); tsds_peer_allreduce_residual then
//   1. per CTA b: counter c = ++counters[b]; store c into flags[b][rank] of
//      every rank (system-scope release, after a system fence);
//   2. waits (bounded, 1 s) until flags[b][p] >= c for every rank p - every
//      rank's CTA b has started this call, so every rank's partial is
//      complete (each rank's previous kernel finished before its CTA b
//      passed griddepcontrol.wait);
//   3. x = bf16(x + bf16(sum_p partial_p)), the sum in rank order 0..tp-1, so
//      every rank computes bit-identical x.
// Why two slots suffice: a rank overwrites slot s two calls later, after the
// barrier of the call in between, which no rank passes before every rank has
// finished the kernel that read slot s.  A rank can be at most one call ahead
// of another (it needs the other's flag for the next call), hence the `>=`.
// Calls must be issued in the same order with the same (M, N) on every rank.
// No TMA, no multicast: plain loads of peer memory.
#include "common.cuh"
#include "peer.cuh"

#include <string.h>

using namespace tsds;
using namespace tsds::peer;

namespace {

constexpr int PEER_THREADS = 256;

struct PeerArgs {
  const float* slot[PEER_MAX_RANKS];  // this call's slot in every rank's buffer
  uint32_t* flags[PEER_MAX_RANKS];    // every rank's flags[PEER_MAX_CTAS][PEER_MAX_RANKS]
  uint32_t* counters;                 // this rank's counters
  int rank, tp;
};

__global__ void __launch_bounds__(PEER_THREADS) peer_allreduce_residual_kernel(PeerArgs a, bf16* __restrict__ x,
                                                                               int64_t n4, int* __restrict__ status) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int b = blockIdx.x;
  pdl_wait();  // this rank's partial (previous kernel) is complete
  if (threadIdx.x == 0) {
    const uint32_t e = a.counters[b] + 1;
    a.counters[b] = e;
    s_epoch = e;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  if (threadIdx.x < a.tp) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + b * PEER_MAX_RANKS + a.rank, e);
    if (!wait_flag(a.flags[a.rank] + b * PEER_MAX_RANKS + threadIdx.x, e)) {
      s_ok = 0;
      atomicExch(status, TSDS_E_TIMEOUT);
    }
  }
  __syncthreads();
  pdl_trigger();
  if (!s_ok) return;
  for (int64_t i = (int64_t)b * PEER_THREADS + threadIdx.x; i < n4; i += (int64_t)gridDim.x * PEER_THREADS) {
    float4 v[PEER_MAX_RANKS];
#pragma unroll
    for (int p = 0; p < PEER_MAX_RANKS; ++p)
      if (p < a.tp) v[p] = ld_volatile_f4(a.slot[p] + 4 * i);
    float4 s = v[0];
#pragma unroll
    for (int p = 1; p < PEER_MAX_RANKS; ++p)
      if (p < a.tp) {
        s.x += v[p].x;
        s.y += v[p].y;
        s.z += v[p].z;
        s.w += v[p].w;
      }
    uint2* xp = reinterpret_cast<uint2*>(x) + i;
    const uint2 xv = *xp;
    uint2 o;
    o.x = pack_bf2(bf_lo(xv.x) + rbf(s.x), bf_hi(xv.x) + rbf(s.y));
    o.y = pack_bf2(bf_lo(xv.y) + rbf(s.z), bf_hi(xv.y) + rbf(s.w));
    *xp = o;
  }
}

}  // namespace

extern "C" size_t tsds_peer_buffer_bytes(int max_elems) { return max_elems <= 0 ? 0 : buffer_bytes(max_elems); }

extern "C" size_t tsds_peer_slot_offset(int max_elems, int slot) { return slot_offset(max_elems, slot); }

extern "C" size_t tsds_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int tsds_peer_alloc(size_t bytes, void** buf) {
  TSDS_RETURN_IF(!buf || bytes < PEER_HEADER_BYTES, TSDS_E_INVALID);
  *buf = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_RUNTIME;
  }
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return TSDS_E_RUNTIME;
  }
  *buf = p;
  return TSDS_OK;
}

extern "C" int tsds_peer_free(void* buf) {
  TSDS_RETURN_IF(!buf, TSDS_E_INVALID);
  if (cudaFree(buf) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_RUNTIME;
  }
  return TSDS_OK;
}

extern "C" int tsds_peer_export(const void* buf, void* handle) {
  TSDS_RETURN_IF(!buf || !handle, TSDS_E_INVALID);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(buf)) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_RUNTIME;
  }
  memcpy(handle, &h, sizeof(h));
  return TSDS_OK;
}

extern "C" int tsds_peer_import(const void* handle, void** buf) {
  TSDS_RETURN_IF(!handle || !buf, TSDS_E_INVALID);
  *buf = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    *buf = nullptr;
    return TSDS_E_RUNTIME;
  }
  return TSDS_OK;
}

extern "C" int tsds_peer_close(void* buf) {
  TSDS_RETURN_IF(!buf, TSDS_E_INVALID);
  if (cudaIpcCloseMemHandle(buf) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_RUNTIME;
  }
  return TSDS_OK;
}

extern "C" int tsds_peer_allreduce_residual(void* x, void* const* bufs, int rank, int tp, int slot, int M, int N,
                                            int max_elems, int* status, tsds_stream_t stream) {
  TSDS_RETURN_IF(!x || !bufs || !status || tp < 1 || tp > PEER_MAX_RANKS || rank < 0 || rank >= tp, TSDS_E_INVALID);
  TSDS_RETURN_IF((slot & ~1) != 0 || M <= 0 || N <= 0 || (N % 4) != 0 || max_elems <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF((int64_t)M * N > max_elems, TSDS_E_INVALID);
  TSDS_RETURN_IF((reinterpret_cast<uintptr_t>(x) & 7u) != 0, TSDS_E_ALIGN);
  PeerArgs a = {};
  for (int p = 0; p < tp; ++p) {
    TSDS_RETURN_IF(!bufs[p], TSDS_E_INVALID);
    TSDS_RETURN_IF(!tsds_aligned16(bufs[p]), TSDS_E_ALIGN);
    char* base = static_cast<char*>(bufs[p]);
    a.slot[p] = reinterpret_cast<const float*>(base + tsds_peer_slot_offset(max_elems, slot));
    a.flags[p] = reinterpret_cast<uint32_t*>(base + PEER_FLAGS_OFF);
  }
  a.counters = static_cast<uint32_t*>(bufs[rank]);
  a.rank = rank;
  a.tp = tp;
  const int64_t n4 = (int64_t)M * N / 4;
  const int64_t want = (n4 + PEER_THREADS - 1) / PEER_THREADS;
  const int grid = (int)(want < PEER_MAX_CTAS ? want : PEER_MAX_CTAS);
  tsds_launch(peer_allreduce_residual_kernel, dim3(grid), dim3(PEER_THREADS), 0, stream, a, (bf16*)x, n4, status);
  return tsds_launch_status();
}
