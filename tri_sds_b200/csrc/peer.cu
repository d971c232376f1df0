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

// ---- vocab-parallel LM head over peer memory ---------------------------------
// Each rank's LM head wrote, into the exchange region of its peer buffer, its
// shard's argmax candidates (rows int64 local indices at 0, rows fp32 values
// at val_off) and, when full logits are wanted, its logits shard ([rows][vl]
// bf16 at log_off).  CTA b meets CTA b of every rank, merges the candidates
// of its rows (the highest value, ties to the lowest global index - the rule
// of tsds_argmax_merge) and copies its share of every rank's shard into the
// full logits rows; then it meets them again, so no rank leaves the kernel -
// and overwrites its region with the next call's data - while another rank
// still reads it.
struct LmArgs {
  const char* ex[PEER_MAX_RANKS];     // every rank's exchange region
  uint32_t* flags[PEER_MAX_RANKS];
  uint32_t* counters;
  int rank, tp;
};

__device__ __forceinline__ bool lm_meet(const LmArgs& a, int b, uint32_t* s_epoch, int* s_ok, int* status) {
  if (threadIdx.x == 0) {
    const uint32_t e = a.counters[b] + 1;
    a.counters[b] = e;
    *s_epoch = e;
    *s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = *s_epoch;
  if (threadIdx.x < a.tp) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + b * PEER_MAX_RANKS + a.rank, e);
    if (!wait_flag(a.flags[a.rank] + b * PEER_MAX_RANKS + threadIdx.x, e)) {
      *s_ok = 0;
      atomicExch(status, TSDS_E_TIMEOUT);
    }
  }
  __syncthreads();
  return *s_ok != 0;
}

__global__ void __launch_bounds__(PEER_THREADS) peer_lm_gather_kernel(const __grid_constant__ LmArgs a, int rows,
                                                                      int vl, int64_t val_off,
                                                                      int64_t log_off, int64_t* __restrict__ argmax_out,
                                                                      int stride, bf16* __restrict__ logits_out,
                                                                      int* __restrict__ status) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int b = blockIdx.x;
  pdl_wait();  // this rank's LM head (previous kernel) is complete
  if (!lm_meet(a, b, &s_epoch, &s_ok, status)) return;
  pdl_trigger();
  // argmax merge: one thread per row
  for (int m = b * PEER_THREADS + threadIdx.x; m < rows; m += gridDim.x * PEER_THREADS) {
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int q = 0; q < a.tp; ++q) {
      const int64_t li = *reinterpret_cast<const volatile int64_t*>(a.ex[q] + (int64_t)m * 8);
      const float v = *reinterpret_cast<const volatile float*>(a.ex[q] + val_off + (int64_t)m * 4);
      const int64_t gi = li + (int64_t)q * vl;
      if (v > bv || (v == bv && gi < bi)) {
        bv = v;
        bi = gi;
      }
    }
    argmax_out[(int64_t)m * stride] = bi == INT64_MAX ? 0 : bi;
  }
  // full logits: every rank's shard into its columns
  if (logits_out) {
    if ((vl & 7) == 0) {
      const int64_t per = (int64_t)rows * (vl / 8);  // 16-byte chunks of one shard
      for (int64_t i = (int64_t)b * PEER_THREADS + threadIdx.x; i < per * a.tp; i += (int64_t)gridDim.x * PEER_THREADS) {
        const int q = (int)(i / per);
        const int64_t j = i - (int64_t)q * per;
        const int m = (int)(j / (vl / 8)), c = (int)(j - (int64_t)m * (vl / 8));
        uint4 v;
        asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(a.ex[q] + log_off + ((int64_t)m * vl + 8 * c) * 2)
                     : "memory");
        *reinterpret_cast<uint4*>(logits_out + (int64_t)m * a.tp * vl + (int64_t)q * vl + 8 * c) = v;
      }
    } else {
      const int64_t per = (int64_t)rows * vl;
      for (int64_t i = (int64_t)b * PEER_THREADS + threadIdx.x; i < per * a.tp; i += (int64_t)gridDim.x * PEER_THREADS) {
        const int q = (int)(i / per);
        const int64_t j = i - (int64_t)q * per;
        const int m = (int)(j / vl), v = (int)(j - (int64_t)m * vl);
        const unsigned short u = *reinterpret_cast<const volatile unsigned short*>(a.ex[q] + log_off + j * 2);
        reinterpret_cast<unsigned short*>(logits_out)[(int64_t)m * a.tp * vl + (int64_t)q * vl + v] = u;
      }
    }
  }
  lm_meet(a, b, &s_epoch, &s_ok, status);  // every rank is done reading every region
}

}  // namespace

extern "C" size_t tsds_peer_buffer_bytes(int max_elems, size_t exchange_bytes) {
  return max_elems <= 0 ? 0 : buffer_bytes(max_elems, exchange_bytes);
}

extern "C" size_t tsds_peer_exchange_offset(int max_elems) { return max_elems <= 0 ? 0 : exchange_offset(max_elems); }

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

extern "C" int tsds_peer_lm_gather(void* const* bufs, int rank, int tp, int max_elems, size_t exchange_bytes, int rows,
                                   int vocab_shard, int64_t val_off, int64_t log_off, int64_t* argmax_out,
                                   int argmax_stride, void* logits_out, int* status, tsds_stream_t stream) {
  TSDS_RETURN_IF(!bufs || !argmax_out || !status || tp < 1 || tp > PEER_MAX_RANKS || rank < 0 || rank >= tp,
                 TSDS_E_INVALID);
  TSDS_RETURN_IF(rows <= 0 || vocab_shard <= 0 || argmax_stride <= 0 || max_elems <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(val_off < (int64_t)rows * 8 || (val_off % 8) != 0 || (log_off % 16) != 0, TSDS_E_ALIGN);
  const int64_t need = logits_out ? log_off + (int64_t)rows * vocab_shard * 2 : val_off + (int64_t)rows * 4;
  TSDS_RETURN_IF(logits_out && log_off < val_off + (int64_t)rows * 4, TSDS_E_INVALID);
  TSDS_RETURN_IF(need > (int64_t)exchange_bytes, TSDS_E_INVALID);
  TSDS_RETURN_IF(logits_out && (vocab_shard % 8) == 0 && !tsds_aligned16(logits_out), TSDS_E_ALIGN);
  LmArgs a = {};
  for (int q = 0; q < tp; ++q) {
    TSDS_RETURN_IF(!bufs[q], TSDS_E_INVALID);
    TSDS_RETURN_IF(!tsds_aligned16(bufs[q]), TSDS_E_ALIGN);
    char* base = static_cast<char*>(bufs[q]);
    a.ex[q] = base + exchange_offset(max_elems);
    a.flags[q] = reinterpret_cast<uint32_t*>(base + PEER_FLAGS_OFF);
  }
  a.counters = static_cast<uint32_t*>(bufs[rank]);
  a.rank = rank;
  a.tp = tp;
  // a grid that depends only on (rows, vocab_shard, tp): the same on every rank
  const int64_t work = logits_out ? (int64_t)rows * tp * ((vocab_shard + 7) / 8) : rows;
  const int64_t want = (work + PEER_THREADS - 1) / PEER_THREADS;
  const int grid = (int)(want < 1 ? 1 : (want < 128 ? want : 128));
  tsds_launch(peer_lm_gather_kernel, dim3(grid), dim3(PEER_THREADS), 0, stream, a, rows, vocab_shard, val_off,
              log_off, argmax_out, argmax_stride, (bf16*)logits_out, status);
  return tsds_launch_status();
}
