// Fused-layer kernel: one persistent tcgen05 launch runs a sequence
// of dependent phases over the same M token rows, e.g. for a decoder layer
//
//   O-proj (+residual) -> RMSNorm -> gate/up (+SwiGLU) -> down (+residual)
//   -> RMSNorm (next layer) -> q/k/v (+QK-norm, RoPE, K/V cache write)
//
// Each GEMM phase is the skinny GEMM of gemm_tc.cu (swap-AB, TMA weight and
// X tiles, tcgen05.mma into double-buffered TMEM accumulators, stream-K over
// all CTAs, deterministic split-tile reduction); an RMSNorm phase normalises
// M rows on the epilogue warps.  Phases are separated by a grid barrier (an
// arrival counter; every CTA of the one resident wave arrives after its share
// of a phase is written).  What a single kernel buys over one launch per
// phase: the TMA warp requests the next GEMM phase's weight tiles as soon as
// ring slots free up - weights never depend on the previous phase - and only
// the activation tiles wait for the barrier, so HBM keeps streaming across
// phase boundaries instead of draining at every kernel edge.
//
// Under tensor parallelism the row-parallel projections store fp32 partials
// into this rank's peer slot and a PEER phase all-reduces them across the
// ranks over NVLink (plain peer loads, the flag protocol of peer.cuh run per
// CTA index) and adds them to the residual: GEMM and all-reduce in one
// kernel, no NCCL between them.
//
// Data produced inside the launch is read with L2-coherent loads (ld.cg) or
// by TMA after a proxy fence, never through the non-coherent path.  Every
// wait is bounded (2 s; 1 s across ranks): a timeout records TSDS_E_TIMEOUT
// in the status word and the CTA unwinds.  No TMA multicast.
#include "common.cuh"
#include "linear.cuh"
#include "peer.cuh"
#include "rowops.cuh"
#include "tc_core.cuh"

#include <string.h>

using namespace tsds;
using namespace tsds::tc;
using tsds::peer::PEER_MAX_RANKS;

static_assert((int)TSDS_EPI_STORE == (int)EPI_STORE && (int)TSDS_EPI_RESIDUAL == (int)EPI_RESIDUAL &&
                  (int)TSDS_EPI_SWIGLU == (int)EPI_SWIGLU && (int)TSDS_EPI_STORE_F32 == (int)EPI_STORE_F32 &&
                  (int)TSDS_EPI_QKROPE == (int)EPI_QKROPE,
              "ABI epilogue codes");

namespace {

constexpr int CH_THREADS = 192;
constexpr int CH_MAX_PHASES = 8;
constexpr int CH_MAX_COUNTERS = 8192;  // arrival + departure counters of all GEMM phases
constexpr int CH_SMEM_BUDGET = 220 * 1024;
constexpr int SMEM_PER_SM = 233472;
constexpr int SMEM_RESERVE = 8192;
constexpr uint64_t CH_WAIT_NS = 2000000000ull;
enum { CH_GEMM = 0, CH_NORM = 1, CH_PEER = 2 };

struct ChPhase {
  int kind, epi;
  // GEMM: out[m][j] (ldo) from weights [n_out (x2 for SwiGLU)][K] and X [M][K]
  int n_out, K, KT, tiles;
  uint32_t W;                  // tiles x KT (host: W * P < 2^32)
  int up_off, ldo, res_ld, ctr;  // ctr: arrival counters at counters[ctr], departures at + tiles
  int Pf;                        // units sharing this phase's iterations: min(W, units), so each owns one or more
  int dp;                        // 1: data-parallel (whole tiles per unit, Pf = min(tiles, units)), 0: stream-K
  const bf16* res;
  bf16* out;
  // NORM: out[m][0:n] (ldo) = RMSNorm(x[m][0:n]) * w
  // PEER: out[m][0:n] (ldo) += sum over ranks of slot `slot` (fp32 [M][n])
  const bf16* x;
  const bf16* w;
  int n, ldx, slot, two_shot;
  float eps;
};

struct ChPeer {  // the ranks' peer buffers (see peer.cuh)
  const float* slot[2][PEER_MAX_RANKS];
  bf16* published[PEER_MAX_RANKS];  // two-shot: each rank's final values of its chunk
  uint32_t* flags[PEER_MAX_RANKS];
  uint32_t* counters;
  int rank, tp;
};

struct ChRope {  // EPI_QKROPE: tile t = head slot t of [q heads | k heads | v heads]
  const bf16* qn;
  const bf16* kn;
  const bf16* cos_t;
  const bf16* sin_t;
  const int32_t* pos;
  const int32_t* starts;
  bf16* q_out;
  bf16* k_cache;
  bf16* v_cache;
  int T, Hq, Hkv, S, rope_len;
  float eps;
};

struct ChParams {
  int M, Npad, P, nph, stages, b_stage_bytes, tmem_cols;
  uint32_t idesc;
  float* ws;
  int* counters;
  int* gbar;  // [0] phase arrivals, [1] departures
  int32_t* status;
  ChPhase ph[CH_MAX_PHASES];
  ChRope qr;
  ChPeer pr;
};

struct ChMaps {
  CUtensorMap a[CH_MAX_PHASES];
  CUtensorMap b[CH_MAX_PHASES];
};

struct ChSmem {
  uint64_t full_bar[MAX_STAGES];
  uint64_t empty_bar[MAX_STAGES];
  uint64_t tfull_bar[2];
  uint64_t tempty_bar[2];
  uint64_t drain_bar;  // abort path: completion of the MMAs issued so far
  uint32_t tmem_base;
  int abort;
  int go;
  int last;
  float xch[64][17];  // SwiGLU: up rows; QKROPE: a [128][8] exchange of 8 columns
  float red[8];
  uint32_t epoch;
  int peer_ok;
};

__device__ __forceinline__ bool wait_count(const int* c, int target) {
  if (ld_acquire(c) >= target) return true;
  const uint64_t t0 = global_ns();
  while (ld_acquire(c) < target) {
    if (global_ns() - t0 > CH_WAIT_NS) return false;
  }
  return true;
}

// generic-proxy writes of this thread (and those it observed) before later
// async-proxy (TMA) reads of the same global memory
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// A unit's range of a GEMM phase (a unit is a CTA, or a CTA pair when
// CG = 2): units 0..Pf-1 split its W iterations, every one of them owning at
// least one (so the contributors of a split tile are consecutive units);
// units from Pf on sit the phase out.  Data-parallel phases (the schedule of
// gemm_tc.cu's tsds_set_gemm_dp_rows) hand out whole tiles instead.
__device__ __forceinline__ void phase_range(const ChPhase& ph, int unit, int& b, int& e) {
  if (ph.dp) {
    b = unit < ph.Pf ? (int)(((uint32_t)unit * (uint32_t)ph.tiles) / (uint32_t)ph.Pf) * ph.KT : 0;
    e = unit < ph.Pf ? (int)(((uint32_t)(unit + 1) * (uint32_t)ph.tiles) / (uint32_t)ph.Pf) * ph.KT : 0;
    return;
  }
  b = unit < ph.Pf ? it_begin(unit, ph.Pf, ph.W) : 0;
  e = unit < ph.Pf ? it_begin(unit + 1, ph.Pf, ph.W) : 0;
}

__device__ __forceinline__ float ldcg_bf(const bf16* p) {
  return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p)) << 16);
}

// ---- epilogue of 16 accumulator columns m0..m0+15 of tile row r -------------
template <int EPI>
__device__ __forceinline__ void ch_finish(const ChParams& p, const ChPhase& ph, ChSmem& sh, int t, int r, int m0,
                                          const float (&v)[16]) {
  if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_STORE_F32) {
    const int j = t * TILE_J + r;
    if (j < ph.n_out) {
      float rv[16];
      if constexpr (EPI == EPI_RESIDUAL) {  // read before any store: out may alias res
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
          rv[jj] = m0 + jj < p.M ? ldcg_bf(ph.res + (int64_t)(m0 + jj) * ph.res_ld + j) : 0.f;
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int m = m0 + jj;
        if (m < p.M) {
          const int64_t o = (int64_t)m * ph.ldo + j;
          if constexpr (EPI == EPI_STORE_F32)
            reinterpret_cast<float*>(ph.out)[o] = v[jj];
          else if constexpr (EPI == EPI_STORE)
            ph.out[o] = f2bf(v[jj]);
          else
            ph.out[o] = f2bf(rv[jj] + rbf(v[jj]));
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    if (r >= 64) {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) sh.xch[r - 64][jj] = rbf(v[jj]);
    }
    epi_bar();
    const int j = t * 64 + r;
    if (r < 64 && j < ph.n_out) {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int m = m0 + jj;
        if (m < p.M) {
          const float g = rbf(v[jj]);
          const float s = rbf(g / (1.0f + expf(-g)));
          ph.out[(int64_t)m * ph.ldo + j] = f2bf(s * sh.xch[r][jj]);
        }
      }
    }
    epi_bar();
  } else {  // EPI_QKROPE: the arithmetic of qk_norm_rope_kv_kernel, lane for lane
    const ChRope& q = p.qr;
    constexpr int D = 128;
    if (t >= q.Hq + 2 * q.Hkv) return;  // the second half of a CTA pair past the last head (uniform)
    float(*xq)[8] = reinterpret_cast<float(*)[8]>(&sh.xch[0][0]);
    const int w = r >> 5, lane = r & 31;
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) xq[r][jj] = rbf(v[half * 8 + jj]);  // the bf16 q/k/v projection
      epi_bar();
      for (int cc = 0; cc < 2; ++cc) {
        const int col = w * 2 + cc;
        const int m = m0 + half * 8 + col;
        if (m >= p.M) continue;  // uniform over the warp
        const int b = m / q.T, tt = m - b * q.T;
        const int row_in_seq = q.starts[b] + tt;
        const int pos = q.pos[m];
        if (row_in_seq < 0 || row_in_seq >= q.S || pos < 0 || pos >= q.rope_len) continue;
        float e[4] = {xq[2 * lane][col], xq[2 * lane + 1][col], xq[64 + 2 * lane][col], xq[65 + 2 * lane][col]};
        if (t >= q.Hq + q.Hkv) {  // v head: into the cache as is
          const int kvh = t - q.Hq - q.Hkv;
          bf16* dst = q.v_cache + (((int64_t)b * q.Hkv + kvh) * q.S + row_in_seq) * D;
          *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack_bf2(e[0], e[1]);
          *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack_bf2(e[2], e[3]);
          continue;
        }
        const bool is_q = t < q.Hq;
        const bf16* nw = is_q ? q.qn : q.kn;
        if (nw) qk_norm_pair(e, nw, lane, q.eps);
        bf16* dst = is_q ? q.q_out + ((int64_t)m * q.Hq + t) * D
                         : q.k_cache + (((int64_t)b * q.Hkv + (t - q.Hq)) * q.S + row_in_seq) * D;
        rope_store(e, q.cos_t, q.sin_t, pos, lane, dst);
      }
      epi_bar();
    }
  }
}

// ---- RMSNorm phase (epilogue warps): rows pc, pc + P, ... ----------------------
// The arithmetic of rms_norm_kernel (256 threads) with 128 threads: thread r
// plays virtual threads r and r + 128, so every partial sum and the order of
// the block reduction are the same.
__device__ void ch_norm(const ChParams& p, const ChPhase& ph, ChSmem& sh, int pc, int r) {
  const int eq = r >> 5, lane = r & 31;
  const int n8 = ph.n / 8;
  for (int m = pc; m < p.M; m += p.P) {
    const bf16* xr = ph.x + (int64_t)m * ph.ldx;
    bf16* orow = ph.out + (int64_t)m * ph.ldo;
    float ssa = 0.f, ssb = 0.f;
    for (int c = r; c < n8; c += 256) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xr + c * 8));
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf_lo(u[i]), b = bf_hi(u[i]);
        ssa = fmaf(a, a, ssa);
        ssa = fmaf(b, b, ssa);
      }
    }
    for (int c = r + 128; c < n8; c += 256) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xr + c * 8));
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf_lo(u[i]), b = bf_hi(u[i]);
        ssb = fmaf(a, a, ssb);
        ssb = fmaf(b, b, ssb);
      }
    }
    ssa = warp_sum(ssa);
    ssb = warp_sum(ssb);
    if (lane == 0) {
      sh.red[eq] = ssa;
      sh.red[eq + 4] = ssb;
    }
    epi_bar();
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += sh.red[i];
    epi_bar();
    const float rstd = 1.0f / sqrtf(ss / (float)ph.n + ph.eps);
    for (int c = r; c < n8; c += 128) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xr + c * 8));
      const uint4 g = ldg16(ph.w + c * 8);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = pack_bf2(bf_lo(u[i]) * rstd * bf_lo(gw[i]), bf_hi(u[i]) * rstd * bf_hi(gw[i]));
      *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ---- all-reduce phase (epilogue warps): x += sum of the ranks' partials ------
// CTA pc meets CTA pc of every other rank (flags of peer.cuh).  Each rank's
// CTA pc reaches a meeting only after its own grid barrier, i.e. after all
// of that rank's partial tiles are stored.
//  one-shot: every CTA then sums its slice of all elements over the ranks in
//    rank order and updates x - every rank reads every rank's whole partial;
//  two-shot: rank r sums only its chunk (elements [r*n/tp, (r+1)*n/tp)) in
//    rank order, updates x there and publishes the bf16 result in its peer
//    buffer; after a second meeting every rank copies the other chunks - a
//    1/tp of the remote reads, the same bits.
__device__ bool ch_meet(const ChParams& p, ChSmem& sh, int pc, int r) {
  using namespace tsds::peer;
  const ChPeer& g = p.pr;
  if (r == 0) {
    const uint32_t e = g.counters[pc] + 1;
    g.counters[pc] = e;
    sh.epoch = e;
    sh.peer_ok = 1;
  }
  epi_bar();
  const uint32_t e = sh.epoch;
  if (r < g.tp) {
    __threadfence_system();
    st_release_sys(g.flags[r] + pc * PEER_MAX_RANKS + g.rank, e);
    if (!wait_flag(g.flags[g.rank] + pc * PEER_MAX_RANKS + r, e)) {
      sh.peer_ok = 0;
      atomicExch(p.status, TSDS_E_TIMEOUT);
    }
  }
  epi_bar();
  return sh.peer_ok != 0;
}

// x[i] (float4 index i of the [M][n] residual, stride ldo) += bf16(sum over ranks)
__device__ __forceinline__ uint2 ch_reduce4(const ChPeer& g, const ChPhase& ph, int64_t i, uint2* xp) {
  using namespace tsds::peer;
  const int n4 = ph.n / 4;
  const int m = (int)(i / n4), c4 = (int)(i - (int64_t)m * n4);
  float4 v[PEER_MAX_RANKS];
#pragma unroll
  for (int q = 0; q < PEER_MAX_RANKS; ++q)
    if (q < g.tp) v[q] = ld_volatile_f4(g.slot[ph.slot][q] + (int64_t)m * ph.n + 4 * c4);
  float4 s = v[0];
#pragma unroll
  for (int q = 1; q < PEER_MAX_RANKS; ++q)
    if (q < g.tp) {
      s.x += v[q].x;
      s.y += v[q].y;
      s.z += v[q].z;
      s.w += v[q].w;
    }
  const uint2 xv = __ldcg(xp);
  uint2 o;
  o.x = pack_bf2(bf_lo(xv.x) + rbf(s.x), bf_hi(xv.x) + rbf(s.y));
  o.y = pack_bf2(bf_lo(xv.y) + rbf(s.z), bf_hi(xv.y) + rbf(s.w));
  return o;
}

__device__ bool ch_peer(const ChParams& p, const ChPhase& ph, ChSmem& sh, int pc, int r) {
  using namespace tsds::peer;
  const ChPeer& g = p.pr;
  if (!ch_meet(p, sh, pc, r)) return false;
  const int n4 = ph.n / 4;
  const int64_t total = (int64_t)p.M * n4;
  auto x_at = [&](int64_t i) {
    const int m = (int)(i / n4), c4 = (int)(i - (int64_t)m * n4);
    return reinterpret_cast<uint2*>(ph.out + (int64_t)m * ph.ldo) + c4;
  };
  if (!ph.two_shot) {
    for (int64_t i = (int64_t)pc * 128 + r; i < total; i += (int64_t)p.P * 128) {
      uint2* xp = x_at(i);
      *xp = ch_reduce4(g, ph, i, xp);
    }
    return true;
  }
  // two-shot: this rank's chunk, then publish
  const int64_t c0 = total * g.rank / g.tp, c1 = total * (g.rank + 1) / g.tp;
  uint2* mine = reinterpret_cast<uint2*>(g.published[g.rank]);
  for (int64_t i = c0 + (int64_t)pc * 128 + r; i < c1; i += (int64_t)p.P * 128) {
    uint2* xp = x_at(i);
    const uint2 o = ch_reduce4(g, ph, i, xp);
    *xp = o;
    mine[i] = o;
  }
  if (!ch_meet(p, sh, pc, r)) return false;  // every rank's chunk is published
  for (int q = 0; q < g.tp; ++q) {
    if (q == g.rank) continue;
    const int64_t q0 = total * q / g.tp, q1 = total * (q + 1) / g.tp;
    const uint2* theirs = reinterpret_cast<const uint2*>(g.published[q]);
    for (int64_t i = q0 + (int64_t)pc * 128 + r; i < q1; i += (int64_t)p.P * 128) {
      uint2 v;
      asm volatile("ld.volatile.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(theirs + i) : "memory");
      *x_at(i) = v;
    }
  }
  return true;
}

// ---- one GEMM phase on the epilogue warps --------------------------------------
template <int EPI, int CG>
__device__ void ch_gemm_epilogue(const ChParams& p, const ChPhase& ph, ChSmem& sh, uint32_t tmem, int pc, int crank,
                                 int r, int& seg, bool& alive) {
  const int eq = r >> 5, lane = r & 31;
  const int nchunk = p.Npad / 16;
  const int KT = ph.KT;
  const int unit = pc / CG;
  int b, e;
  phase_range(ph, unit, b, e);
  int* arr = p.counters + ph.ctr;  // per 128-row (virtual) tile
  int* dep = arr + ph.tiles * CG;
  // STORE / RESIDUAL / STORE_F32: split tiles reduced by all contributors;
  // SWIGLU / QKROPE need whole tiles: the last arriver finishes them
  constexpr bool DIST = EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_STORE_F32;
  int pend0 = -1, pend1 = -1, npend = 0;
  if (b < e) {
    for (int t = b / KT; alive && t <= (e - 1) / KT; ++t, ++seg) {
      const int tb = t * KT;
      const int vt = t * CG + crank;  // this CTA's 128-row tile
      const int k0 = (b > tb ? b : tb) - tb;
      const int k1 = (e < tb + KT ? e : tb + KT) - tb;
      const int buf = seg & 1, use = seg >> 1;
      if (!mbar_wait(&sh.tfull_bar[buf], use & 1)) {
        atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
      epi_bar();
      if (r == 0) sh.go = !*(volatile int*)&sh.abort;
      epi_bar();
      if (!sh.go) {
        alive = false;
        break;
      }
      tc_fence_after();
      const bool full = (k0 == 0 && k1 == KT);
      const uint32_t taddr = tmem + buf * p.tmem_cols + ((uint32_t)(eq * 32) << 16);
      const int slot = (t == b / KT) ? 0 : 1;
      float4* part = reinterpret_cast<float4*>(p.ws + ((size_t)(pc * 2 + slot) * p.Npad) * TILE_J) + r;
      for (int c = 0; c < nchunk; ++c) {
        float v[16];
        tmem_ld16(taddr + c * 16, v);
        if (full) {
          ch_finish<EPI>(p, ph, sh, vt, r, c * 16, v);
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            part[(size_t)(c * 4 + q4) * TILE_J] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_remote(mapa_shared(smem_u32(&sh.tempty_bar[buf]), 0));  // the leader's MMA reuses it
        else
          mbar_arrive(&sh.tempty_bar[buf]);
      }
      if (!full && DIST) {
        __threadfence();
        epi_bar();
        if (r == 0) atomicAdd(&arr[vt], 1);
        if (npend++ == 0)
          pend0 = t;
        else
          pend1 = t;
      } else if (!full) {
        const int q_lo = owner_of(tb, ph.Pf, ph.W), q_hi = owner_of(tb + KT - 1, ph.Pf, ph.W);
        __threadfence();
        epi_bar();
        if (r == 0) sh.last = (atomicAdd(&arr[vt], 1) == q_hi - q_lo);
        epi_bar();
        if (sh.last) {
          __threadfence();
          const int nq = q_hi - q_lo + 1;
          const int lo_slot = it_begin(q_lo, ph.Pf, ph.W) < tb ? 1 : 0;
          for (int c = 0; c < nchunk; ++c) {
            float v[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v[jj] = 0.f;
            for (int qi = 0; qi < nq; ++qi) {  // unit order: deterministic
              const int q = (q_lo + qi) * CG + crank;  // the contributor's CTA for this half
              const int qs = qi == 0 ? lo_slot : 0;
              const float4* src = reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                                  (size_t)c * 4 * TILE_J + r;
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                const float4 f = __ldcg(src + (size_t)q4 * TILE_J);
                v[4 * q4] += f.x;
                v[4 * q4 + 1] += f.y;
                v[4 * q4 + 2] += f.z;
                v[4 * q4 + 3] += f.w;
              }
            }
            ch_finish<EPI>(p, ph, sh, vt, r, c * 16, v);
          }
          if (r == 0) arr[vt] = 0;  // ready for the next launch
        }
      }
    }
  }
  if constexpr (DIST) {
    for (int pi = 0; alive && pi < npend; ++pi) {
      const int t = pi == 0 ? pend0 : pend1, tb = t * KT;
      const int vt = t * CG + crank;
      const int q_lo = owner_of(tb, ph.Pf, ph.W), q_hi = owner_of(tb + KT - 1, ph.Pf, ph.W);
      const int nq = q_hi - q_lo + 1, c = unit - q_lo;
      const int lo_slot = it_begin(q_lo, ph.Pf, ph.W) < tb ? 1 : 0;
      const int rlo = c * TILE_J / nq, R = (c + 1) * TILE_J / nq - rlo;
      const int nel = R * (p.Npad / 4);
      if (r == 0) {
        const bool ok = wait_count(&arr[vt], nq);
        if (!ok) atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.go = ok;
      }
      epi_bar();
      const bool go = sh.go;
      epi_bar();
      if (!go) {
        alive = false;
        break;
      }
      for (int e0 = r; e0 < nel; e0 += 128) {
        const int rr = rlo + e0 % R, g = e0 / R;
        const int j = vt * TILE_J + rr;
        float rv[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (j < ph.n_out && 4 * g + i < p.M) rv[i] = ldcg_bf(ph.res + (int64_t)(4 * g + i) * ph.res_ld + j);
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int qi = 0; qi < nq; ++qi) {
          const int q = (q_lo + qi) * CG + crank;
          const int qs = qi == 0 ? lo_slot : 0;
          const float4 f = __ldcg(reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                                  (size_t)g * TILE_J + rr);
          acc.x += f.x;
          acc.y += f.y;
          acc.z += f.z;
          acc.w += f.w;
        }
        if (j < ph.n_out) {
          const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = 4 * g + i;
            if (m < p.M) {
              const int64_t o = (int64_t)m * ph.ldo + j;
              if constexpr (EPI == EPI_STORE_F32)
                reinterpret_cast<float*>(ph.out)[o] = a4[i];
              else if constexpr (EPI == EPI_STORE)
                ph.out[o] = f2bf(a4[i]);
              else
                ph.out[o] = f2bf(rv[i] + rbf(a4[i]));
            }
          }
        }
      }
      epi_bar();
      if (r == 0 && atomicAdd(&dep[vt], 1) == nq - 1) {
        arr[vt] = 0;  // every contributor has left
        dep[vt] = 0;
      }
    }
  }
}

// CG = 2: CTA pairs (clusters of 2) for the GEMM phases - each CTA stages
// its 128 weight rows of a 256-row tile and half of the token rows, the
// leader issues the pair's MMAs (see gemm_tc.cu); row phases stay per CTA.
template <int CG>
__global__ void __launch_bounds__(CH_THREADS, 2)
    fused_layer_kernel(const __grid_constant__ ChMaps maps, const __grid_constant__ ChParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ ChSmem sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pc = blockIdx.x;
  const int crank = CG == 2 ? (int)cluster_ctarank() : 0;
  const int unit = pc / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&sh.full_bar[s], 1);
      mbar_init(&sh.empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.tfull_bar[i], 1);
      mbar_init(&sh.tempty_bar[i], 4 * CG);  // every epilogue warp of the pair
    }
    mbar_init(&sh.drain_bar, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                   "r"(2 * p.tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                   "r"(2 * p.tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync_all();  // both CTAs' barriers and TMEM exist before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + p.stages * A_STAGE;
  pdl_trigger();
  int issued = 0;  // producer lane: ring stages requested; MMA lane: stages consumed

  if (warp == 0) {
    // ---------------- TMA producer: every GEMM phase's tiles, in order -------
    if (lane == 0) {
      bool ok = true, waited = false;
      int i = 0;  // ring position (stages issued so far, over all phases)
      for (int f = 0; ok && f < p.nph; ++f) {
        const ChPhase& ph = p.ph[f];
        if (ph.kind != CH_GEMM) continue;
        int b, e;
        phase_range(ph, unit, b, e);
        if (b >= e) continue;
        const CUtensorMap* am = &maps.a[f];
        const CUtensorMap* bm = &maps.b[f];
        prefetch_tmap(am);
        prefetch_tmap(bm);
        const int KT = ph.KT;
        const bool swiglu = ph.epi == EPI_SWIGLU;
        auto load_a = [&](int it, int s) {
          const int t = it / KT, kt = it % KT;
          if constexpr (CG == 2) {  // this CTA's 128 rows of the pair's 256, counted on the leader's barrier
            const int row0 = swiglu ? t * 128 + crank * 64 : t * 256 + crank * 128;
            const int row1 = swiglu ? ph.up_off + t * 128 + crank * 64 : row0 + 64;
            const uint32_t bar = mapa_shared(smem_u32(&sh.full_bar[s]), 0);
            tma_load_2d_pair(a_smem + s * A_STAGE, am, bar, kt * BK, row0);
            tma_load_2d_pair(a_smem + s * A_STAGE + A_STAGE / 2, am, bar, kt * BK, row1);
          } else {
            const int row0 = swiglu ? t * 64 : t * TILE_J;
            const int row1 = swiglu ? ph.up_off + t * 64 : t * TILE_J + 64;
            tma_load_2d(a_smem + s * A_STAGE, am, &sh.full_bar[s], kt * BK, row0);
            tma_load_2d(a_smem + s * A_STAGE + A_STAGE / 2, am, &sh.full_bar[s], kt * BK, row1);
          }
        };
        auto load_b = [&](int it, int s) {
          if constexpr (CG == 2)  // this CTA's half of the token rows
            tma_load_2d_pair(b_smem + s * p.b_stage_bytes, bm, mapa_shared(smem_u32(&sh.full_bar[s]), 0),
                             (it % KT) * BK, crank * (p.Npad / 2));
          else
            tma_load_2d(b_smem + s * p.b_stage_bytes, bm, &sh.full_bar[s], (it % KT) * BK, 0);
        };
        auto expect = [&](int s) {  // the leader's full barrier counts both CTAs' bytes
          if (crank == 0) mbar_arrive_expect_tx(&sh.full_bar[s], CG * (A_STAGE + p.b_stage_bytes));
        };
        // weight tiles first: they do not depend on the earlier phases
        const int npre = (e - b) < p.stages ? (e - b) : p.stages;
        for (int k = 0; k < npre; ++k) {
          const int s = (i + k) % p.stages, rnd = (i + k) / p.stages;
          if ((rnd > 0 && !mbar_wait(&sh.empty_bar[s], (rnd - 1) & 1)) || *(volatile int*)&sh.abort) {
            ok = false;
            break;
          }
          expect(s);
          load_a(b + k, s);
          issued = i + k + 1;
        }
        if (!ok) break;
        // activations: written by the previous kernel (f == 0) or by phase f-1
        if (!waited) {
          pdl_wait();
          waited = true;
        }
        if (f > 0) {
          if (!wait_count(&p.gbar[0], p.P * f)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        for (int k = 0; k < npre; ++k) load_b(b + k, (i + k) % p.stages);
        for (int k = npre; k < e - b; ++k) {
          const int s = (i + k) % p.stages, rnd = (i + k) / p.stages;
          if (!mbar_wait(&sh.empty_bar[s], (rnd - 1) & 1) || *(volatile int*)&sh.abort) {
            ok = false;
            break;
          }
          expect(s);
          load_a(b + k, s);
          load_b(b + k, s);
          issued = i + k + 1;
        }
        i += e - b;
      }
      if (!ok) {
        atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
      if (!waited) pdl_wait();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && crank == 0) {
      int i = 0, seg = 0;
      bool ok = true;
      for (int f = 0; ok && f < p.nph; ++f) {
        const ChPhase& ph = p.ph[f];
        if (ph.kind != CH_GEMM) continue;
        int b, e;
        phase_range(ph, unit, b, e);
        if (b >= e) continue;
        const int KT = ph.KT;
        for (int t = b / KT; ok && t <= (e - 1) / KT; ++t, ++seg) {
          const int tb = t * KT;
          const int k0 = (b > tb ? b : tb) - tb;
          const int k1 = (e < tb + KT ? e : tb + KT) - tb;
          const int buf = seg & 1, use = seg >> 1;
          if (use > 0 && !mbar_wait(&sh.tempty_bar[buf], (use - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + buf * p.tmem_cols;
          for (int kt = k0; kt < k1; ++kt, ++i) {
            const int s = i % p.stages, rnd = i / p.stages;
            if (!mbar_wait(&sh.full_bar[s], rnd & 1) || *(volatile int*)&sh.abort) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_smem + s * A_STAGE);
            const uint32_t b_base = smem_u32(b_smem + s * p.b_stage_bytes);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              if constexpr (CG == 2)
                umma_bf16_pair(d, sdesc_sw128(a_base + kk * 32), sdesc_sw128(b_base + kk * 32), p.idesc,
                               (kt > k0 || kk > 0) ? 1u : 0u);
              else
                umma_bf16(d, sdesc_sw128(a_base + kk * 32), sdesc_sw128(b_base + kk * 32), p.idesc,
                          (kt > k0 || kk > 0) ? 1u : 0u);
            }
            if constexpr (CG == 2)
              umma_commit_pair(&sh.empty_bar[s]);  // frees stage s in both CTAs
            else
              umma_commit(&sh.empty_bar[s]);
          }
          if (!ok) break;
          if constexpr (CG == 2)
            umma_commit_pair(&sh.tfull_bar[buf]);
          else
            umma_commit(&sh.tfull_bar[buf]);
        }
      }
      issued = i;
      if (!ok) {
        atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
    }
  } else {
    // ---------------- epilogue warps (2-5): GEMM epilogues and row phases ----
    pdl_wait();
    const int r = (warp & 3) * 32 + lane;
    int seg = 0;
    bool alive = true;
    for (int f = 0; alive && f < p.nph; ++f) {
      const ChPhase& ph = p.ph[f];
      if (f > 0) {  // phase f-1 complete on every CTA: its outputs are this phase's inputs
        if (r == 0) {
          const bool ok = wait_count(&p.gbar[0], p.P * f);
          if (!ok) atomicExch(p.status, TSDS_E_TIMEOUT);
          sh.go = ok && !*(volatile int*)&sh.abort;
        }
        epi_bar();
        alive = sh.go;
        epi_bar();
        if (!alive) break;
      }
      if (ph.kind == CH_NORM) {
        ch_norm(p, ph, sh, pc, r);
      } else if (ph.kind == CH_PEER) {
        alive = ch_peer(p, ph, sh, pc, r);
      } else {
        switch (ph.epi) {
          case EPI_STORE: ch_gemm_epilogue<EPI_STORE, CG>(p, ph, sh, tmem, pc, crank, r, seg, alive); break;
          case EPI_RESIDUAL: ch_gemm_epilogue<EPI_RESIDUAL, CG>(p, ph, sh, tmem, pc, crank, r, seg, alive); break;
          case EPI_SWIGLU: ch_gemm_epilogue<EPI_SWIGLU, CG>(p, ph, sh, tmem, pc, crank, r, seg, alive); break;
          case EPI_STORE_F32: ch_gemm_epilogue<EPI_STORE_F32, CG>(p, ph, sh, tmem, pc, crank, r, seg, alive); break;
          default: ch_gemm_epilogue<EPI_QKROPE, CG>(p, ph, sh, tmem, pc, crank, r, seg, alive); break;
        }
      }
      if (!alive) break;
      // publish this phase: its global writes before the arrival, for both
      // plain loads and TMA reads of the next phases
      fence_proxy_async_global();
      __threadfence();
      epi_bar();
      if (r == 0) atomicAdd(&p.gbar[0], 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (sh.abort) {  // uniform: read after the barrier
    // a CTA that gave up still lets its copies and MMAs in flight finish
    // (bounded) before TMEM is freed and it exits.  A pair's copies complete
    // on the leader's barriers, which the leader drains; the other CTA
    // leaves only after the leader (the cluster barrier below).
    if (warp == 0 && lane == 0 && crank == 0 && issued > 0) drain_tma_ring(sh.full_bar, p.stages, issued);
    if (warp == 1 && lane == 0 && crank == 0 && issued > 0) drain_mma<CG>(&sh.drain_bar);
    __syncthreads();
  }
  if constexpr (CG == 2) cluster_sync_all();  // the pair is done with both TMEM halves
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * p.tmem_cols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * p.tmem_cols));
  }
  // the last CTA out resets the phase counter for the next launch (every CTA
  // has finished waiting on it by then)
  if (threadIdx.x == 0 && atomicAdd(&p.gbar[1], 1) == p.P - 1) {
    p.gbar[0] = 0;
    p.gbar[1] = 0;
    __threadfence();
  }
}

int pow2_at_least(int x) {
  int v = 32;
  while (v < x) v <<= 1;
  return v;
}

// CTAs that can be resident at once with `smem` dynamic bytes each (CG = 2:
// as 2-CTA clusters, which need two SMs of one GPC): the grid barrier needs
// the whole grid resident.  Cached per (CG, size); the devices of one
// process are assumed alike.
int resident_ctas(int CG, size_t smem) {
  static size_t keys[16];
  static int vals[16];
  static int n = 0;
  const size_t key = smem * 2 + (CG == 2);
  std::lock_guard<std::mutex> hold(tsds_host_cache_lock());
  for (int i = 0; i < n; ++i)
    if (keys[i] == key) return vals[i];
  int ctas = 0;
  if (CG == 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(CH_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = 2;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    cfg.attrs = ca;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, fused_layer_kernel<2>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    ctas = 2 * clusters;
  } else {
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fused_layer_kernel<1>, CH_THREADS, smem) !=
        cudaSuccess) {
      cudaGetLastError();
      blocks = 0;
    }
    ctas = blocks * tsds_tc_num_sms();
  }
  if (n < 16) {
    keys[n] = key;
    vals[n] = ctas;
    ++n;
  }
  return ctas;
}

size_t partial_bytes(int M) {
  const int npad = M <= 0 ? 0 : (M + 15) / 16 * 16;
  return (size_t)tsds_tc_num_sms() * 4 * 2 * npad * TILE_J * sizeof(float);
}

}  // namespace

extern "C" size_t tsds_fused_layer_workspace_bytes(int M) {
  if (M <= 0 || M > 256) return 0;
  return 64 + (size_t)CH_MAX_COUNTERS * sizeof(int) + partial_bytes(M);
}

// The status word and the counters (see tsds_linear_workspace_header_bytes).
extern "C" size_t tsds_fused_layer_workspace_header_bytes(void) { return 64 + (size_t)CH_MAX_COUNTERS * sizeof(int); }

// The grid the fused kernel takes for M token rows under the current tuning
// switches: out[0] CTAs, out[1] CTAs per weight tile (1, or 2 for pairs),
// out[2] pipeline stages, out[3] CTAs per SM requested.  The same arithmetic
// as tsds_fused_layer below (a test and tuning aid).
extern "C" int tsds_fused_layer_grid(int M, int32_t* out) {
  TSDS_RETURN_IF(!out || M <= 0 || M > 256, TSDS_E_INVALID);
  const int npad = (M + 15) / 16 * 16;
  const int tmem_cols = pow2_at_least(npad);
  int ctas = tsds_tc_ctas_setting();
  while (ctas > 1 && 2 * tmem_cols * ctas > 512) --ctas;
  const int pr = tsds_tc_pair_rows();
  const int CG = (pr > 0 && M >= pr) ? 2 : 1;
  const int b_stage_bytes = npad / CG * BK * 2;
  int budget = SMEM_PER_SM / ctas - SMEM_RESERVE;
  if (budget > CH_SMEM_BUDGET) budget = CH_SMEM_BUDGET;
  int stages = (budget - 1024) / (A_STAGE + b_stage_bytes);
  if (stages > MAX_STAGES) stages = MAX_STAGES;
  TSDS_RETURN_IF(stages < 2, TSDS_E_UNSUPPORTED);
  const size_t smem = (size_t)stages * (A_STAGE + b_stage_bytes) + 1024;
  static tsds_device_flags attr1, attr2;
  const int st = CG == 2 ? tsds_smem_limit_once(fused_layer_kernel<2>, CH_SMEM_BUDGET, attr2)
                         : tsds_smem_limit_once(fused_layer_kernel<1>, CH_SMEM_BUDGET, attr1);
  if (st != TSDS_OK) return st;
  int P = tsds_tc_num_sms() * ctas;
  const int resident = resident_ctas(CG, smem) / CG * CG;
  TSDS_RETURN_IF(resident < CG, TSDS_E_UNSUPPORTED);
  if (resident < P) P = resident;
  out[0] = P;
  out[1] = CG;
  out[2] = stages;
  out[3] = ctas;
  return TSDS_OK;
}

extern "C" int tsds_fused_layer(const tsds_fused_phase* phases, int n_phases, int M, const tsds_qk_rope* qr,
                                const tsds_peer_group* peers, void* workspace, size_t workspace_bytes,
                                tsds_stream_t stream) {
  TSDS_RETURN_IF(!phases || n_phases < 1 || n_phases > CH_MAX_PHASES || M <= 0 || M > 256, TSDS_E_INVALID);
  TSDS_RETURN_IF(!workspace || workspace_bytes < tsds_fused_layer_workspace_bytes(M), TSDS_E_WORKSPACE);
  TSDS_RETURN_IF(!tsds_aligned16(workspace), TSDS_E_ALIGN);
  ChParams p = {};
  ChMaps maps;
  memset(&maps, 0, sizeof(maps));
  p.M = M;
  p.Npad = (M + 15) / 16 * 16;
  p.tmem_cols = pow2_at_least(p.Npad);
  int ctas = tsds_tc_ctas_setting();
  while (ctas > 1 && 2 * p.tmem_cols * ctas > 512) --ctas;
  // CTA pairs for the GEMM phases from the tcgen05 GEMM's pair threshold on
  const int pr = tsds_tc_pair_rows();
  const int CG = (pr > 0 && M >= pr) ? 2 : 1;
  p.nph = n_phases;
  p.status = (int32_t*)workspace;
  p.gbar = (int*)((char*)workspace + 4);
  p.counters = (int*)((char*)workspace + 64);
  p.ws = (float*)((char*)workspace + 64 + (size_t)CH_MAX_COUNTERS * sizeof(int));
  p.b_stage_bytes = p.Npad / CG * BK * 2;  // this CTA's token rows
  int budget = SMEM_PER_SM / ctas - SMEM_RESERVE;
  if (budget > CH_SMEM_BUDGET) budget = CH_SMEM_BUDGET;
  p.stages = (budget - 1024) / (A_STAGE + p.b_stage_bytes);
  if (p.stages > MAX_STAGES) p.stages = MAX_STAGES;
  TSDS_RETURN_IF(p.stages < 2, TSDS_E_UNSUPPORTED);
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.Npad >> 3) << 17) |
            ((uint32_t)((TILE_J * CG) >> 4) << 24);
  const size_t smem = (size_t)p.stages * (A_STAGE + p.b_stage_bytes) + 1024;
  // an upper bound while the phases are checked; lowered below to what can
  // be resident at once (a smaller grid keeps every check valid)
  p.P = tsds_tc_num_sms() * ctas;
  int ctr = 0;
  bool rope = false;
  for (int f = 0; f < n_phases; ++f) {
    const tsds_fused_phase& in = phases[f];
    ChPhase& ph = p.ph[f];
    ph.kind = in.kind;
    ph.epi = in.epi;
    if (in.kind == TSDS_PHASE_PEER) {
      using namespace tsds::peer;
      TSDS_RETURN_IF(!peers || !peers->bufs || peers->tp < 1 || peers->tp > PEER_MAX_RANKS || peers->rank < 0 ||
                         peers->rank >= peers->tp || p.P > PEER_MAX_CTAS,
                     TSDS_E_INVALID);
      TSDS_RETURN_IF(!in.out || in.K <= 0 || (in.K % 4) != 0 || in.ldo < in.K || (in.n_out & ~1) != 0 ||
                         (in.epi & ~1) != 0 || (int64_t)M * in.K > peers->max_elems,
                     TSDS_E_INVALID);
      TSDS_RETURN_IF((reinterpret_cast<uintptr_t>(in.out) & 7u) != 0 || (in.ldo % 4) != 0, TSDS_E_ALIGN);
      for (int q = 0; q < peers->tp; ++q) {
        TSDS_RETURN_IF(!peers->bufs[q], TSDS_E_INVALID);
        TSDS_RETURN_IF(!tsds_aligned16(peers->bufs[q]), TSDS_E_ALIGN);
        char* base = static_cast<char*>(peers->bufs[q]);
        p.pr.slot[0][q] = reinterpret_cast<const float*>(base + slot_offset(peers->max_elems, 0));
        p.pr.slot[1][q] = reinterpret_cast<const float*>(base + slot_offset(peers->max_elems, 1));
        p.pr.published[q] = reinterpret_cast<bf16*>(base + published_offset(peers->max_elems));
        p.pr.flags[q] = reinterpret_cast<uint32_t*>(base + PEER_FLAGS_OFF);
      }
      p.pr.counters = static_cast<uint32_t*>(peers->bufs[peers->rank]);
      p.pr.rank = peers->rank;
      p.pr.tp = peers->tp;
      ph.out = (bf16*)in.out;
      ph.n = in.K;
      ph.ldo = in.ldo;
      ph.slot = in.n_out;
      ph.two_shot = in.epi;
      continue;
    }
    if (in.kind == TSDS_PHASE_NORM) {
      TSDS_RETURN_IF(!in.x || !in.w || !in.out || in.K <= 0 || (in.K % 8) != 0, TSDS_E_INVALID);
      TSDS_RETURN_IF(in.ldx < in.K || in.ldo < in.K, TSDS_E_INVALID);
      TSDS_RETURN_IF(!tsds_aligned16(in.x) || !tsds_aligned16(in.w) || !tsds_aligned16(in.out) || (in.ldx % 8) ||
                         (in.ldo % 8),
                     TSDS_E_ALIGN);
      ph.x = (const bf16*)in.x;
      ph.w = (const bf16*)in.w;
      ph.out = (bf16*)in.out;
      ph.n = in.K;
      ph.ldx = in.ldx;
      ph.ldo = in.ldo;
      ph.eps = in.eps;
      continue;
    }
    TSDS_RETURN_IF(in.kind != TSDS_PHASE_GEMM, TSDS_E_INVALID);
    TSDS_RETURN_IF(in.epi != EPI_STORE && in.epi != EPI_RESIDUAL && in.epi != EPI_SWIGLU && in.epi != EPI_STORE_F32 &&
                       in.epi != EPI_QKROPE,
                   TSDS_E_INVALID);
    TSDS_RETURN_IF(!in.x || !in.w || in.n_out <= 0 || in.K <= 0 || in.ldx < in.K, TSDS_E_INVALID);
    TSDS_RETURN_IF(in.epi != EPI_QKROPE && !in.out, TSDS_E_INVALID);
    TSDS_RETURN_IF(in.epi == EPI_RESIDUAL && (!in.res || in.res_ld < in.n_out), TSDS_E_INVALID);
    TSDS_RETURN_IF(in.epi != EPI_QKROPE && in.ldo < in.n_out, TSDS_E_INVALID);
    TSDS_RETURN_IF(!tsds_aligned16(in.x) || !tsds_aligned16(in.w) || (in.ldx % 8) || (in.K % 8), TSDS_E_ALIGN);
    ph.n_out = in.n_out;
    ph.K = in.K;
    ph.KT = (in.K + BK - 1) / BK;
    ph.tiles = in.epi == EPI_SWIGLU ? (in.n_out + 64 * CG - 1) / (64 * CG)
                                    : (in.n_out + TILE_J * CG - 1) / (TILE_J * CG);
    const long long W64 = (long long)ph.tiles * ph.KT;
    const int units = p.P / CG;
    TSDS_RETURN_IF(W64 * units >= (1ll << 32), TSDS_E_UNSUPPORTED);
    ph.W = (uint32_t)W64;
    ph.Pf = (int)(W64 < units ? W64 : units);  // lowered with P below
    ph.up_off = in.n_out;
    ph.ldo = in.ldo;
    ph.res = (const bf16*)in.res;
    ph.res_ld = in.res_ld;
    ph.out = (bf16*)in.out;
    ph.ctr = ctr;
    ctr += 2 * ph.tiles * CG;  // arrival and departure counters per 128-row tile
    TSDS_RETURN_IF(ctr > CH_MAX_COUNTERS, TSDS_E_UNSUPPORTED);
    if (in.epi == EPI_QKROPE) {
      TSDS_RETURN_IF(!qr || rope, TSDS_E_INVALID);  // one rope phase per launch (one parameter set)
      rope = true;
      TSDS_RETURN_IF(qr->T <= 0 || (M % qr->T) != 0 || qr->Hq <= 0 || qr->Hkv <= 0 || qr->S <= 0 ||
                         qr->rope_len <= 0 || (qr->Hq % qr->Hkv) != 0,
                     TSDS_E_INVALID);
      TSDS_RETURN_IF(in.n_out != (qr->Hq + 2 * qr->Hkv) * 128, TSDS_E_INVALID);
      TSDS_RETURN_IF(!qr->cos || !qr->sin || !qr->positions || !qr->starts || !qr->q_out || !qr->k_cache ||
                         !qr->v_cache,
                     TSDS_E_INVALID);
      p.qr.qn = (const bf16*)qr->q_norm_w;
      p.qr.kn = (const bf16*)qr->k_norm_w;
      p.qr.cos_t = (const bf16*)qr->cos;
      p.qr.sin_t = (const bf16*)qr->sin;
      p.qr.pos = qr->positions;
      p.qr.starts = qr->starts;
      p.qr.q_out = (bf16*)qr->q_out;
      p.qr.k_cache = (bf16*)qr->k_cache;
      p.qr.v_cache = (bf16*)qr->v_cache;
      p.qr.T = qr->T;
      p.qr.Hq = qr->Hq;
      p.qr.Hkv = qr->Hkv;
      p.qr.S = qr->S;
      p.qr.rope_len = qr->rope_len;
      p.qr.eps = qr->eps;
    }
    const int w_rows = in.epi == EPI_SWIGLU ? 2 * in.n_out : in.n_out;
    int st = tsds_make_tmap_2d_bf16(&maps.a[f], in.w, in.K, w_rows, (uint64_t)in.K * 2, BK, 64, 1);
    if (st != TSDS_OK) return st;
    st = tsds_make_tmap_2d_bf16(&maps.b[f], in.x, in.K, M, (uint64_t)in.ldx * 2, BK, p.Npad / CG, 1);
    if (st != TSDS_OK) return st;
  }
  {
    static tsds_device_flags attr1, attr2;
    const int st = CG == 2 ? tsds_smem_limit_once(fused_layer_kernel<2>, CH_SMEM_BUDGET, attr2)
                           : tsds_smem_limit_once(fused_layer_kernel<1>, CH_SMEM_BUDGET, attr1);
    if (st != TSDS_OK) return st;
    const int resident = resident_ctas(CG, smem) / CG * CG;
    TSDS_RETURN_IF(resident < CG, TSDS_E_UNSUPPORTED);
    if (resident < p.P) p.P = resident;
  }
  for (int f = 0; f < n_phases; ++f) {
    ChPhase& ph = p.ph[f];
    if (ph.kind != CH_GEMM) continue;
    const int units = p.P / CG;
    if (ph.Pf > units) ph.Pf = units;
    // the data-parallel choice of tsds_tc_gemm, on the resident units
    const int dp_units = tsds_tc_dp_units(M, ph.tiles, units);
    ph.dp = dp_units > 0 ? 1 : 0;
    if (ph.dp) ph.Pf = dp_units;
  }
  if (CG == 2)
    tsds_launch_cluster(fused_layer_kernel<2>, dim3(p.P), dim3(CH_THREADS), smem, stream, 2, maps, p);
  else
    tsds_launch(fused_layer_kernel<1>, dim3(p.P), dim3(CH_THREADS), smem, stream, maps, p);
  return tsds_launch_status();
}
