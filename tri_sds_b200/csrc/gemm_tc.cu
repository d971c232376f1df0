// Persistent tcgen05 skinny GEMM for the linear layers and the LM head (sm_100a).
//
//   D[j][m] = sum_k W[j][k] * X[m][k]      (swap-AB: weight rows j fill the MMA's
//                                            M = 128, token rows m are its N)
//
// * Persistent CTAs (two per SM by default).  The work (tiles of 128 weight rows x k-tiles of 64) is
//   split stream-K style: CTA p owns the contiguous iteration range
//   [W*p/P, W*(p+1)/P) of the flattened (tile, k-tile) space, so every SM
//   streams the same number of weight bytes whatever the layer shape.
// * Warp 0 (one lane) issues TMA loads of the weight tile (two 64x64 boxes,
//   128-byte swizzle) and of the X tile (64 x Npad box; rows past M are
//   zero-filled by TMA) into a STAGES-deep ring (mbarrier full/empty).
// * Warp 1 (one lane) issues tcgen05.mma kind::f16 (bf16 in, fp32 out,
//   M=128, N=Npad, K=16 per instruction) into one of two TMEM accumulators
//   and commits completion to the ring's empty barriers / the accumulator's
//   full barrier.
// * Warps 2-5 drain TMEM with tcgen05.ld (lane quarter = warp % 4) and run
//   the epilogue: bf16 store, residual add, SwiGLU (gate rows 0-63 and up
//   rows 64-127 of the same tile), or LM-head argmax candidates.
// * A tile split across CTAs is finished from its contributors' fp32
//   partials, summed in CTA order, so the result is deterministic and -
//   since the split depends only on (n_out, K, P) - a row's result never
//   depends on M or on the other rows.  The LM head's argmax tile is summed
//   by its last contributor (atomic counter); the other epilogues spread a
//   tile's rows over its reducers, at most one tile per CTA, so the
//   kernel's tail is one slice of one tile long.
// Every mbarrier wait is bounded; on a timeout the CTA records
// TSDS_E_TIMEOUT in the status word and unwinds.
#include "common.cuh"
#include "linear.cuh"
#include "tc_core.cuh"

using namespace tsds;
using namespace tsds::tc;

namespace {

constexpr int NUM_THREADS = 192;
constexpr int SMEM_BUDGET = 220 * 1024;

struct TcParams {
  int M, Npad, n_out, K, KT, tiles, P;
  uint32_t W;  // tiles x KT; the host guarantees W * P < 2^32
  int up_off, ldo, res_ld;
  const bf16* res;
  bf16* out;
  float* ws;
  int* counters;
  int32_t* status;
  float* cand_val;
  int* cand_idx;
  int ldc;
  int stages, b_stage_bytes;
  uint32_t idesc;
  int tmem_cols;
  int dp;  // 1: data-parallel schedule (whole tiles per unit), 0: stream-K
  uint64_t wait_ns;  // limit of every bounded wait (tsds_set_wait_limit_ns)
  // residual epilogue only (tsds_linear_residual_norm): RMSNorm of the
  // finished output rows into norm_out, or none (norm_out null)
  const bf16* norm_w;
  bf16* norm_out;
  int norm_ld;
  float norm_eps;
};

// Workspace header words of the RMSNorm tail (status is word 0 of the
// 64-byte header): CTAs done, counted on HDR_NDONE words (CTA p on word
// HDR_DONE + p % HDR_NDONE, so the P arrivals do not queue on one address),
// and norm workers done.
constexpr int HDR_DONE = 4, HDR_NDONE = 8, HDR_LEFT = HDR_DONE + HDR_NDONE;
static_assert(HDR_LEFT < 16, "the tail's words within the 64-byte header");

constexpr int MAX_TILES = 2048;   // tile counters; departure counters follow them

struct Smem {
  uint64_t full_bar[MAX_STAGES];
  uint64_t empty_bar[MAX_STAGES];
  uint64_t tfull_bar[2];
  uint64_t tempty_bar[2];
  uint64_t drain_bar;  // abort path: completion of the MMAs issued so far
  uint32_t tmem_base;
  int abort;
  int go;
  int last;
  float xch[64][17];
  float red_v[4][16];
  int red_i[4][16];
};

// Final epilogue for 16 accumulator columns m0..m0+15 of tile row r.
template <int EPI>
__device__ __forceinline__ void finish_chunk(const TcParams& p, Smem& sh, int t, int r, int m0, const float (&v)[16]) {
  const int eq = r >> 5, lane = r & 31;
  if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_STORE_F32) {
    const int j = t * TILE_J + r;
    if (j < p.n_out) {
      // The residual may be the output buffer itself (in-place x += ...):
      // read all of it before the first store so the loads are not
      // serialised behind the stores.
      float rv[16];
      if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) rv[jj] = m0 + jj < p.M ? bf2f(p.res[(int64_t)(m0 + jj) * p.res_ld + j]) : 0.f;
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int m = m0 + jj;
        if (m < p.M) {
          const int64_t o = (int64_t)m * p.ldo + j;
          if constexpr (EPI == EPI_STORE_F32)
            reinterpret_cast<float*>(p.out)[o] = v[jj];  // unrounded partial (tensor-parallel shards)
          else if constexpr (EPI == EPI_STORE)
            p.out[o] = f2bf(v[jj]);
          else
            p.out[o] = f2bf(rv[jj] + rbf(v[jj]));
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
    if (r < 64 && j < p.n_out) {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int m = m0 + jj;
        if (m < p.M) {
          const float g = rbf(v[jj]);
          const float s = rbf(g / (1.0f + expf(-g)));
          p.out[(int64_t)m * p.ldo + j] = f2bf(s * sh.xch[r][jj]);
        }
      }
    }
    epi_bar();
  } else {  // EPI_ARGMAX (LM head): bf16 logits, per-tile candidates
    const int j = t * TILE_J + r;
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int m = m0 + jj;
      float lv = j < p.n_out ? rbf(v[jj]) : -INFINITY;
      if (p.out && j < p.n_out && m < p.M) p.out[(int64_t)m * p.ldo + j] = f2bf(lv);
      int li = j;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, lv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, li, o);
        if (better(ov, oi, lv, li)) {
          lv = ov;
          li = oi;
        }
      }
      if (lane == 0) {
        sh.red_v[eq][jj] = lv;
        sh.red_i[eq][jj] = li;
      }
    }
    epi_bar();
    if (r < 16 && m0 + r < p.M) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = 0; q < 4; ++q)
        if (better(sh.red_v[q][r], sh.red_i[q][r], bv, bi)) {
          bv = sh.red_v[q][r];
          bi = sh.red_i[q][r];
        }
      p.cand_val[(int64_t)(m0 + r) * p.ldc + t] = bv;
      p.cand_idx[(int64_t)(m0 + r) * p.ldc + t] = bi;
    }
    epi_bar();
  }
}

// RMSNorm of output rows m = row0, row0 + step, ... < M into norm_out
// (tsds_linear_residual_norm): the arithmetic of rms_norm_kernel (256
// threads) on the 128 epilogue threads, thread r playing threads r and
// r + 128, so every partial sum and the block reduction's order are the
// same and the result is bit for bit the separate kernel's.  The rows were
// written by other CTAs of this launch: read through L2.
// Rows of n <= NORM_V * 1024 (n / 8 vectors over 128 threads) stay in
// registers: vector c = r + 128 i is thread r's i-th, which belongs to
// virtual thread r (i even) or r + 128 (i odd), and each virtual thread's
// vectors are summed in ascending order as in the separate kernel.  gw
// holds the thread's norm-weight vectors, read by the caller.
constexpr int NORM_V = 8;
__device__ void norm_rows(const TcParams& p, Smem& sh, int r, int row0, int step, const uint4 (&gw)[NORM_V]) {
  float* red = &sh.red_v[0][0];
  const int n = p.n_out, nv = n / 8;
  const int w = r >> 5, lane = r & 31;
  for (int m = row0; m < p.M; m += step) {
    const bf16* xr = p.out + (int64_t)m * p.ldo;
    bf16* orow = p.norm_out + (int64_t)m * p.norm_ld;
    uint4 v[NORM_V];
#pragma unroll
    for (int i = 0; i < NORM_V; ++i)
      if (r + 128 * i < nv) v[i] = __ldcg(reinterpret_cast<const uint4*>(xr + (r + 128 * i) * 8));
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NORM_V; ++i) {
      if (r + 128 * i < nv) {
        const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a = bf_lo(u[k]), b = bf_hi(u[k]);
          ss[i & 1] = fmaf(a, a, ss[i & 1]);
          ss[i & 1] = fmaf(b, b, ss[i & 1]);
        }
      }
    }
    const float s0 = warp_sum(ss[0]), s1 = warp_sum(ss[1]);
    if (lane == 0) {
      red[w] = s0;
      red[w + 4] = s1;
    }
    epi_bar();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    epi_bar();
    const float rstd = 1.0f / sqrtf(t / (float)n + p.norm_eps);
#pragma unroll
    for (int i = 0; i < NORM_V; ++i) {
      const int c = r + 128 * i;
      if (c < nv) {
        const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const uint32_t g4[4] = {gw[i].x, gw[i].y, gw[i].z, gw[i].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = pack_bf2(bf_lo(u[k]) * rstd * bf_lo(g4[k]), bf_hi(u[k]) * rstd * bf_hi(g4[k]));
        *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CG = 1: one CTA per tile of 128 weight rows.  CG = 2: a CTA pair on two
// SMs (cluster of 2) per tile of 256 rows - each CTA stages its 128 weight
// rows and half of the token rows, the leader (cluster rank 0) issues the
// pair's MMAs (tcgen05 cta_group::2) and every CTA finishes its own half as
// "virtual tile" vt = t * 2 + rank, so counters, partials and epilogues keep
// their one-CTA meaning.  The pair halves the activation bytes each SM stages
// per weight byte, which leaves room for more weight stages in flight when
// the token count is large.
template <int EPI, int CG>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Smem sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pc = blockIdx.x;
  const int crank = CG == 2 ? (int)cluster_ctarank() : 0;
  const int unit = pc / CG, PU = p.P / CG;  // stream-K units: CTAs or CTA pairs
  const int KT = p.KT;
  // stream-K: contiguous ranges of the (tile, k-block) iterations; data-parallel:
  // whole tiles per unit (PU = min(tiles, units) units), so no tile is split and
  // no partials are exchanged
  const int b = p.dp ? (int)(((uint32_t)unit * (uint32_t)p.tiles) / (uint32_t)PU) * KT : it_begin(unit, PU, p.W);
  const int e = p.dp ? (int)(((uint32_t)(unit + 1) * (uint32_t)p.tiles) / (uint32_t)PU) * KT
                     : it_begin(unit + 1, PU, p.W);

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
    // ---------------- TMA producer ----------------
    // The weights do not depend on earlier kernels: the first `stages` weight
    // tiles are requested before the dependency wait, so they stream in
    // while the previous kernel drains; X (its output) only after the wait.
    if (lane == 0 && b < e) {
      prefetch_tmap(&amap);
      prefetch_tmap(&bmap);
      const int npre = (e - b) < p.stages ? (e - b) : p.stages;
      auto load_a = [&](int it, int s) {
        const int t = it / KT, kt = it % KT;
        if constexpr (CG == 2) {
          // this CTA's 128 rows of the pair's 256; bytes counted on the leader's barrier
          const int row0 = EPI == EPI_SWIGLU ? t * 128 + crank * 64 : t * 256 + crank * 128;
          const int row1 = EPI == EPI_SWIGLU ? p.up_off + t * 128 + crank * 64 : row0 + 64;
          const uint32_t bar = mapa_shared(smem_u32(&sh.full_bar[s]), 0);
          tma_load_2d_pair(a_smem + s * A_STAGE, &amap, bar, kt * BK, row0);
          tma_load_2d_pair(a_smem + s * A_STAGE + A_STAGE / 2, &amap, bar, kt * BK, row1);
        } else {
          const int row0 = EPI == EPI_SWIGLU ? t * 64 : t * TILE_J;
          const int row1 = EPI == EPI_SWIGLU ? p.up_off + t * 64 : t * TILE_J + 64;
          tma_load_2d(a_smem + s * A_STAGE, &amap, &sh.full_bar[s], kt * BK, row0);
          tma_load_2d(a_smem + s * A_STAGE + A_STAGE / 2, &amap, &sh.full_bar[s], kt * BK, row1);
        }
      };
      auto load_b = [&](int it, int s) {
        if constexpr (CG == 2)  // this CTA's half of the token rows
          tma_load_2d_pair(b_smem + s * p.b_stage_bytes, &bmap, mapa_shared(smem_u32(&sh.full_bar[s]), 0),
                           (it % KT) * BK, crank * (p.Npad / 2));
        else
          tma_load_2d(b_smem + s * p.b_stage_bytes, &bmap, &sh.full_bar[s], (it % KT) * BK, 0);
      };
      // the leader's full barrier counts both CTAs' bytes of a stage
      auto expect = [&](int s) {
        if (crank == 0) mbar_arrive_expect_tx(&sh.full_bar[s], CG * (A_STAGE + p.b_stage_bytes));
      };
      for (int i = 0; i < npre; ++i) {
        expect(i);
        load_a(b + i, i);
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i) load_b(b + i, i);
      int i = npre;
      for (int it = b + npre; it < e; ++it, ++i) {
        const int s = i % p.stages, r = i / p.stages;
        if (!mbar_wait(&sh.empty_bar[s], (r - 1) & 1, p.wait_ns)) {
          atomicExch(p.status, TSDS_E_TIMEOUT);
          sh.abort = 1;
          break;
        }
        if (*(volatile int*)&sh.abort) break;
        expect(s);
        load_a(it, s);
        load_b(it, s);
      }
      issued = i;
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the pair's leader for CG = 2) ----------------
    if (lane == 0 && b < e && crank == 0) {
      int i = 0, seg = 0;
      bool ok = true;
      for (int t = (int)(b / KT); ok && t <= (int)((e - 1) / KT); ++t, ++seg) {
        const int tb = t * KT;
        const int k0 = (int)((b > tb ? b : tb) - tb);
        const int k1 = (int)((e < tb + KT ? e : tb + KT) - tb);
        const int buf = seg & 1, use = seg >> 1;
        if (use > 0 && !mbar_wait(&sh.tempty_bar[buf], (use - 1) & 1, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * p.tmem_cols;
        for (int kt = k0; kt < k1; ++kt, ++i) {
          const int s = i % p.stages, r = i / p.stages;
          if (!mbar_wait(&sh.full_bar[s], r & 1, p.wait_ns) || *(volatile int*)&sh.abort) {
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
      issued = i;
      if (!ok) {
        atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5) ----------------
    pdl_wait();  // reads the residual, writes outputs and the shared workspace
    const int eq = warp & 3;
    const int r = eq * 32 + lane;  // tile row == TMEM lane
    const int nchunk = p.Npad / 16;
    // STORE / RESIDUAL / STORE_F32 / SWIGLU: split tiles are reduced by all
    // their contributors (each sums a slice of rows - for SwiGLU a slice of
    // gate rows together with their up rows) once every partial is stored;
    // ARGMAX needs whole tiles and keeps the last-arriver reduction.
    constexpr bool DIST = EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_STORE_F32 || EPI == EPI_SWIGLU;
    int pend0 = -1, pend1 = -1;  // split tiles of this CTA (registers, not an indexed array)
    int npend = 0;
    int seg = 0;
    bool alive = b < e;
    for (int t = (int)(b / KT); alive && t <= (int)((e - 1) / KT); ++t, ++seg) {
      const int tb = t * KT;
      const int vt = t * CG + crank;  // this CTA's 128-row tile
      const int k0 = (int)((b > tb ? b : tb) - tb);
      const int k1 = (int)((e < tb + KT ? e : tb + KT) - tb);
      const int buf = seg & 1, use = seg >> 1;
      const int ok = mbar_wait(&sh.tfull_bar[buf], use & 1, p.wait_ns) ? 1 : 0;
      if (!ok) {
        atomicExch(p.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
      // the four epilogue warps take one decision from one snapshot
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
      // partial of a split tile: slot 0 = this CTA's first segment, 1 = its
      // last; layout [Npad/4][TILE_J][4] - a thread moves 4 columns of its row
      // per access and a warp's access covers 512 contiguous bytes
      const int slot = (t == b / KT) ? 0 : 1;
      float4* part = reinterpret_cast<float4*>(p.ws + ((size_t)(pc * 2 + slot) * p.Npad) * TILE_J) + r;
      for (int c = 0; c < nchunk; ++c) {
        float v[16];
        tmem_ld16(taddr + c * 16, v);
        if (full) {
          finish_chunk<EPI>(p, sh, vt, r, c * 16, v);
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
        // arrive without waiting: a split tile is only a first or a last
        // segment, so there are at most two
        __threadfence();
        epi_bar();
        if (r == 0) atomicAdd(&p.counters[vt], 1);
        if (npend++ == 0)
          pend0 = t;
        else
          pend1 = t;
      } else if (!full) {
        // contributors of tile t: units q_lo..q_hi, in order
        const int q_lo = owner_of(tb, PU, p.W), q_hi = owner_of(tb + KT - 1, PU, p.W);
        __threadfence();
        epi_bar();
        if (r == 0) sh.last = (atomicAdd(&p.counters[vt], 1) == q_hi - q_lo);
        epi_bar();
        if (sh.last) {
          __threadfence();
          // Partials are summed in CTA order (deterministic); the loads of up
          // to FIX_Q contributors are issued together so the tail costs one
          // L2 round trip per FIX_Q partials instead of one per partial.
          // Contributors after q_lo start inside tile t (their slot 0); q_lo
          // holds it in slot 1 unless its range starts exactly at the tile.
          constexpr int FIX_Q = EPI == EPI_RESIDUAL ? 5 : 6;
          const int nq = q_hi - q_lo + 1;
          const int lo_slot = it_begin(q_lo, PU, p.W) < tb ? 1 : 0;
          for (int c = 0; c < nchunk; ++c) {
            float v[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v[jj] = 0.f;
            for (int q0 = 0; q0 < nq; q0 += FIX_Q) {
              float tmp[FIX_Q][16];
#pragma unroll
              for (int i = 0; i < FIX_Q; ++i) {
                if (q0 + i < nq) {
                  const int q = (q_lo + q0 + i) * CG + crank;  // the contributor's CTA for this half
                  const int qs = q0 + i == 0 ? lo_slot : 0;
                  const float4* src =
                      reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                      (size_t)c * 4 * TILE_J + r;
#pragma unroll
                  for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 f = __ldcg(src + (size_t)q4 * TILE_J);
                    tmp[i][4 * q4] = f.x;
                    tmp[i][4 * q4 + 1] = f.y;
                    tmp[i][4 * q4 + 2] = f.z;
                    tmp[i][4 * q4 + 3] = f.w;
                  }
                }
              }
#pragma unroll
              for (int i = 0; i < FIX_Q; ++i) {
                if (q0 + i < nq) {
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) v[jj] += tmp[i][jj];
                }
              }
            }
            finish_chunk<EPI>(p, sh, vt, r, c * 16, v);
          }
          if (r == 0) p.counters[vt] = 0;  // ready for the next launch
        }
      }
    }
    if constexpr (DIST) {
      // Every arrival of this CTA is done, so no wait below can block
      // another CTA's arrival (the grid is one resident wave).  The tile's
      // nr reducers (split_reducers: its contributors, less the last one
      // when that one holds two split tiles) each sum a slice of rows:
      // reducer c takes rows [c*128/nr, (c+1)*128/nr) (SwiGLU: gate rows
      // [c*64/nr, (c+1)*64/nr) and the up rows 64 below them) over all nq
      // partials in CTA order; the last reducer to leave resets the
      // counters.  A CTA with two split tiles reduces its last one only, so
      // every CTA's tail is at most one slice long.
      constexpr bool SW = EPI == EPI_SWIGLU;
      constexpr int ROWS = SW ? 64 : TILE_J;  // rows (SwiGLU: gate rows) split among reducers
      for (int pi = npend == 2 ? 1 : 0; alive && pi < npend; ++pi) {
        const int t = pi == 0 ? pend0 : pend1, tb = t * KT;
        const int vt = t * CG + crank;
        const int q_lo = owner_of(tb, PU, p.W), q_hi = owner_of(tb + KT - 1, PU, p.W);
        const int nq = q_hi - q_lo + 1, c = unit - q_lo;
        const int nr = split_reducers(q_lo, q_hi, PU, p.W, KT);
        const int lo_slot = it_begin(q_lo, PU, p.W) < tb ? 1 : 0;
        const int rlo = c * ROWS / nr, R = (c + 1) * ROWS / nr - rlo;
        const int nel = R * (p.Npad / 4);
        if (r == 0) {
          int ok = 1;
          if (ld_acquire(&p.counters[vt]) < nq) {
            const uint64_t t0 = global_ns();
            while (ld_acquire(&p.counters[vt]) < nq) {
              if (global_ns() - t0 > p.wait_ns) {
                ok = 0;
                break;
              }
            }
          }
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
        if constexpr (SW) {
          // element e = (gate row rr of the slice, 4-column group g): its gate
          // row and its up row 64 below are summed over the partials in CTA
          // order from zero.  A thread takes EU elements per pass and issues
          // the loads of all their partials (QB per batch) before summing, so
          // a pass costs one L2 round trip instead of one per element.
          constexpr int EU = 4, QB = 3;
          for (int e0 = r; e0 < nel; e0 += 128 * EU) {
            float4 acc[EU][2];
#pragma unroll
            for (int u = 0; u < EU; ++u) acc[u][0] = acc[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q0 = 0; q0 < nq; q0 += QB) {
              float4 f[EU][QB][2];
#pragma unroll
              for (int u = 0; u < EU; ++u) {
                const int e = e0 + u * 128;
                if (e < nel) {
                  const int rr = rlo + e % R, g = e / R;
#pragma unroll
                  for (int i = 0; i < QB; ++i)
                    if (q0 + i < nq) {
                      const int q = (q_lo + q0 + i) * CG + crank;
                      const int qs = q0 + i == 0 ? lo_slot : 0;
                      const float4* src =
                          reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                          (size_t)g * TILE_J + rr;
                      f[u][i][0] = __ldcg(src);
                      f[u][i][1] = __ldcg(src + 64);
                    }
                }
              }
#pragma unroll
              for (int u = 0; u < EU; ++u)
                if (e0 + u * 128 < nel) {
#pragma unroll
                  for (int i = 0; i < QB; ++i)
                    if (q0 + i < nq) {
#pragma unroll
                      for (int h = 0; h < 2; ++h) {
                        acc[u][h].x += f[u][i][h].x;
                        acc[u][h].y += f[u][i][h].y;
                        acc[u][h].z += f[u][i][h].z;
                        acc[u][h].w += f[u][i][h].w;
                      }
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < EU; ++u) {
              const int e = e0 + u * 128;
              if (e >= nel) continue;
              const int rr = rlo + e % R, g = e / R;
              const int j = vt * 64 + rr;
              if (j >= p.n_out) continue;
              // the SwiGLU of the whole-tile epilogue: gate and up rounded to
              // bf16, silu(gate) rounded, the product rounded
              const float a4[4] = {acc[u][0].x, acc[u][0].y, acc[u][0].z, acc[u][0].w};
              const float b4[4] = {acc[u][1].x, acc[u][1].y, acc[u][1].z, acc[u][1].w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int m = 4 * g + i;
                if (m < p.M) {
                  const float gv = rbf(a4[i]);
                  const float sv = rbf(gv / (1.0f + expf(-gv)));
                  p.out[(int64_t)m * p.ldo + j] = f2bf(sv * rbf(b4[i]));
                }
              }
            }
          }
        } else if constexpr (EPI == EPI_STORE || EPI == EPI_STORE_F32) {
          // plain stores: EU elements per pass with all their partials'
          // loads in flight (measured faster at many token rows: q/k/v at
          // M=208 55 us instead of 64 us with two); each element sums its
          // partials in CTA order from zero, as below
          constexpr int EU = 3, QB = 6;
          for (int e0 = r; e0 < nel; e0 += 128 * EU) {
            float4 acc[EU];
#pragma unroll
            for (int u = 0; u < EU; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q0 = 0; q0 < nq; q0 += QB) {
              float4 f[EU][QB];
#pragma unroll
              for (int u = 0; u < EU; ++u) {
                const int e = e0 + u * 128;
                if (e < nel) {
                  const int rr = rlo + e % R, g = e / R;
#pragma unroll
                  for (int i = 0; i < QB; ++i)
                    if (q0 + i < nq) {
                      const int q = (q_lo + q0 + i) * CG + crank;
                      const int qs = q0 + i == 0 ? lo_slot : 0;
                      f[u][i] = __ldcg(reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                                       (size_t)g * TILE_J + rr);
                    }
                }
              }
#pragma unroll
              for (int u = 0; u < EU; ++u)
                if (e0 + u * 128 < nel) {
#pragma unroll
                  for (int i = 0; i < QB; ++i)
                    if (q0 + i < nq) {
                      acc[u].x += f[u][i].x;
                      acc[u].y += f[u][i].y;
                      acc[u].z += f[u][i].z;
                      acc[u].w += f[u][i].w;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < EU; ++u) {
              const int e = e0 + u * 128;
              if (e >= nel) continue;
              const int rr = rlo + e % R, g = e / R;
              const int j = vt * TILE_J + rr;
              if (j >= p.n_out) continue;
              const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int m = 4 * g + i;
                if (m < p.M) {
                  const int64_t o = (int64_t)m * p.ldo + j;
                  if constexpr (EPI == EPI_STORE_F32)
                    reinterpret_cast<float*>(p.out)[o] = a4[i];
                  else
                    p.out[o] = f2bf(a4[i]);
                }
              }
            }
          }
        } else {
          for (int e0 = r; e0 < nel; e0 += 128) {
            const int rr = rlo + e0 % R, g = e0 / R;
            const int j = vt * TILE_J + rr;
            float rv[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (j < p.n_out && 4 * g + i < p.M) rv[i] = bf2f(p.res[(int64_t)(4 * g + i) * p.res_ld + j]);
            }
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            constexpr int QB = 10;
            for (int q0 = 0; q0 < nq; q0 += QB) {
              float4 f[QB];
#pragma unroll
              for (int i = 0; i < QB; ++i)
                if (q0 + i < nq) {
                  const int q = (q_lo + q0 + i) * CG + crank;
                  const int qs = q0 + i == 0 ? lo_slot : 0;
                  f[i] = __ldcg(reinterpret_cast<const float4*>(p.ws + ((size_t)(q * 2 + qs) * p.Npad) * TILE_J) +
                                (size_t)g * TILE_J + rr);
                }
#pragma unroll
              for (int i = 0; i < QB; ++i)
                if (q0 + i < nq) {
                  acc.x += f[i].x;
                  acc.y += f[i].y;
                  acc.z += f[i].z;
                  acc.w += f[i].w;
                }
            }
            if (j < p.n_out) {
              const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int m = 4 * g + i;
                if (m < p.M) {
                  const int64_t o = (int64_t)m * p.ldo + j;
                  if constexpr (EPI == EPI_STORE_F32)
                    reinterpret_cast<float*>(p.out)[o] = a4[i];
                  else if constexpr (EPI == EPI_STORE)
                    p.out[o] = f2bf(a4[i]);
                  else
                    p.out[o] = f2bf(rv[i] + rbf(a4[i]));
                }
              }
            }
          }
        }
        epi_bar();
        if (r == 0 && atomicAdd(&p.counters[MAX_TILES + vt], 1) == nr - 1) {
          p.counters[vt] = 0;  // every reducer has left: ready for the next launch
          p.counters[MAX_TILES + vt] = 0;
        }
      }
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
  if constexpr (EPI == EPI_RESIDUAL) {
    // RMSNorm tail (tsds_linear_residual_norm): every CTA reports itself
    // done; CTAs 0..NW-1 (NW = min(M, P)) wait (bounded) until all P have,
    // then normalise rows blockIdx.x, + NW, ...; the last of them to finish
    // resets the two header words.  The grid is one resident wave, so the
    // wait always ends.  A CTA that gave up still reports itself done.
    if (p.norm_out != nullptr) {
      int* done = p.status + HDR_DONE;
      int* left = p.status + HDR_LEFT;
      // the barrier above orders this CTA's stores before thread 0's fence
      // and release (the grid-barrier pattern)
      if (threadIdx.x == 0) {
        __threadfence();
        red_release_add(done + blockIdx.x % HDR_NDONE, 1);
      }
      const int NW = p.M < p.P ? p.M : p.P;
      if ((int)blockIdx.x < NW) {
        const int nr = (warp & 3) * 32 + lane;
        uint4 gw[NORM_V];  // the norm weights are constant: read before the wait
        if (warp >= 2 && p.n_out / 8 <= NORM_V * 128) {
#pragma unroll
          for (int i = 0; i < NORM_V; ++i)
            if (nr + 128 * i < p.n_out / 8) gw[i] = ldg16(p.norm_w + (nr + 128 * i) * 8);
        }
        if (threadIdx.x == 0) {
          int ok = 1;
          const uint64_t t0 = global_ns();
          for (;;) {
            int c[HDR_NDONE];  // every word's load in flight at once
#pragma unroll
            for (int k = 0; k < HDR_NDONE; ++k) c[k] = *(volatile int*)(done + k);
            bool all = true;
#pragma unroll
            for (int k = 0; k < HDR_NDONE; ++k) all &= c[k] >= (p.P - k + HDR_NDONE - 1) / HDR_NDONE;
            if (all) break;
            if (global_ns() - t0 > p.wait_ns) {
              ok = 0;
              break;
            }
          }
          __threadfence();  // acquire: the other CTAs' rows are read after this
          if (!ok) atomicExch(p.status, TSDS_E_TIMEOUT);
          sh.go = ok;
        }
        __syncthreads();
        if (sh.go && warp >= 2 && p.n_out / 8 <= NORM_V * 128) norm_rows(p, sh, nr, (int)blockIdx.x, NW, gw);
        __syncthreads();
        if (threadIdx.x == 0 && atomicAdd(left, 1) == NW - 1) {
          // every worker has seen all P: ready for the next launch
#pragma unroll
          for (int k = 0; k < HDR_NDONE; ++k) atomicExch(done + k, 0);
          atomicExch(left, 0);
        }
      }
    }
  }
}

std::atomic<int> g_num_sms{0};
// CTAs per SM: two CTAs with half the pipeline each keep more weight bytes in
// flight per SM than one CTA with a deep pipeline (measured on B200: 6.3 vs
// 5.5 TB/s for the bare TMA stream).  Capped so both fit in TMEM (512
// columns) and shared memory.
std::atomic<int> g_ctas_per_sm{2};
// Token rows from which a projection runs on CTA pairs (CG = 2); 0: never.
std::atomic<int> g_pair_min_rows{0};
// Token rows from which a projection may run data-parallel instead of
// stream-K (when within the slack below); 0: never.  Default 128: the B=8
// tree verify's 208 rows run gate/up in 139 us instead of 161 us; below 128
// rows stream-K stays.
std::atomic<int> g_dp_min_rows{128};
// Largest makespan increase (percent over the ideal tiles / units) the
// data-parallel schedule may cost.  Default 100: at 208 rows q/k/v (80 tiles)
// runs on 80 CTAs in 46.5 us instead of stream-K's 58 us over 148; O and down
// (40 tiles, 3.7x over ideal) stay stream-K.
std::atomic<int> g_dp_slack_pct{100};
// Limit of every bounded wait of the kernel, in ns of %globaltimer: far above
// any legitimate wait; lowered only to test the recovery from a timeout.
std::atomic<unsigned long long> g_wait_ns{2000000000ull};
constexpr int SMEM_PER_SM = 233472;    // 228 KB
constexpr int SMEM_RESERVE = 8192;     // static shared memory + per-CTA system reserve

int num_sms() {
  int n = g_num_sms.load(std::memory_order_relaxed);
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      n = 148;
    }
    g_num_sms.store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace

extern "C" void tsds_set_gemm_ctas_per_sm(int n) { g_ctas_per_sm = n < 1 ? 1 : (n > 4 ? 4 : n); }
extern "C" void tsds_set_gemm_pair_rows(int rows) { g_pair_min_rows = rows < 0 ? 0 : rows; }
extern "C" int tsds_get_gemm_pair_rows(void) { return g_pair_min_rows; }
extern "C" void tsds_set_gemm_dp_rows(int rows) { g_dp_min_rows = rows < 0 ? 0 : rows; }
extern "C" int tsds_get_gemm_dp_rows(void) { return g_dp_min_rows; }
extern "C" void tsds_set_gemm_dp_slack(int percent) {
  g_dp_slack_pct = percent < 0 ? 0 : (percent > 1000 ? 1000 : percent);
}
extern "C" int tsds_get_gemm_dp_slack(void) { return g_dp_slack_pct; }
extern "C" void tsds_set_wait_limit_ns(unsigned long long ns) {
  g_wait_ns = ns < 1 ? 1 : (ns > 10000000000ull ? 10000000000ull : ns);
}
extern "C" unsigned long long tsds_get_wait_limit_ns(void) { return g_wait_ns; }
int tsds_tc_num_sms() { return num_sms(); }

// Data-parallel: min(tiles, units) units take whole tiles, so no split
// tile's fp32 partials are written, waited for and summed at the end of the
// kernel.  Its makespan is ceil(tiles / used units) tiles against the ideal
// tiles / units; it is chosen when that costs at most g_dp_slack_pct percent
// more (with fewer tiles than units: when tiles / units >= 1 / (1 + slack)).
// Returns the units to use data-parallel, or 0 for stream-K.
int tsds_tc_dp_units(int M, int tiles, int units) {
  const int rows = g_dp_min_rows.load(std::memory_order_relaxed);
  if (rows <= 0 || M < rows || tiles <= 0 || units <= 0) return 0;
  const long long pu = tiles < units ? tiles : units;
  const long long per_unit = (tiles + pu - 1) / pu;
  return per_unit * units * 100 <= (long long)tiles * (100 + g_dp_slack_pct.load(std::memory_order_relaxed))
             ? (int)pu
             : 0;
}
int tsds_tc_ctas_setting() { return g_ctas_per_sm; }
int tsds_tc_pair_rows() { return g_pair_min_rows; }

namespace {

template <int EPI, int CG>
int launch_tc(const CUtensorMap& amap, const CUtensorMap& bmap, const TcParams& p, size_t smem, cudaStream_t stream) {
  static tsds_device_flags attr;
  const int st = tsds_smem_limit_once(tc_gemm_kernel<EPI, CG>, SMEM_BUDGET, attr);
  if (st != TSDS_OK) return st;
  if constexpr (CG == 2)
    tsds_launch_cluster(tc_gemm_kernel<EPI, CG>, dim3(p.P), dim3(NUM_THREADS), smem, stream, 2, amap, bmap, p);
  else
    tsds_launch(tc_gemm_kernel<EPI, CG>, dim3(p.P), dim3(NUM_THREADS), smem, stream, amap, bmap, p);
  return tsds_launch_status();
}

int pow2_at_least(int x) {
  int v = 32;
  while (v < x) v <<= 1;
  return v;
}

// Clusters of two CTAs that can be resident at once with `smem` bytes each.
// The split-tile reduction needs the whole grid resident, and a 2-CTA
// cluster needs two SMs of one GPC, so the pair grid is sized from this
// rather than from the SM count.  Cached per shared-memory size (the
// devices of one process are assumed alike).
template <int EPI>
int max_pair_clusters(size_t smem) {
  static size_t keys[16];
  static int vals[16];
  static int n = 0;
  std::lock_guard<std::mutex> hold(tsds_host_cache_lock());
  for (int i = 0; i < n; ++i)
    if (keys[i] == smem) return vals[i];
  static tsds_device_flags attr;
  if (tsds_smem_limit_once(tc_gemm_kernel<EPI, 2>, SMEM_BUDGET, attr) != TSDS_OK) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute ca[1];
  ca[0].id = cudaLaunchAttributeClusterDimension;
  ca[0].val.clusterDim.x = 2;
  ca[0].val.clusterDim.y = 1;
  ca[0].val.clusterDim.z = 1;
  cfg.attrs = ca;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_kernel<EPI, 2>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    clusters = 0;
  }
  if (n < 16) {
    keys[n] = smem;
    vals[n] = clusters;
    ++n;
  }
  return clusters;
}

int pair_clusters(int epi, size_t smem) {
  switch (epi) {
    case EPI_STORE: return max_pair_clusters<EPI_STORE>(smem);
    case EPI_RESIDUAL: return max_pair_clusters<EPI_RESIDUAL>(smem);
    case EPI_SWIGLU: return max_pair_clusters<EPI_SWIGLU>(smem);
    case EPI_STORE_F32: return max_pair_clusters<EPI_STORE_F32>(smem);
    default: return 0;
  }
}

}  // namespace

// Workspace layout: [status int32, the RMSNorm tail's words 4-12 (HDR_DONE..HDR_LEFT), padding to 64 B]
// [arrival counters: 2048 ints][departure counters: 2048 ints][partials: P x 2 x Npad x 128 fp32].
// The counters must be zero before the first use; every launch leaves them zero.
size_t tsds_tc_workspace_bytes(int M) {
  const int npad = M <= 0 ? 0 : (M + 15) / 16 * 16;
  return 64 + 2 * MAX_TILES * sizeof(int) + (size_t)num_sms() * 4 * 2 * npad * TILE_J * sizeof(float);
}

// The status word and the counters: what must be zero before the next
// launch after a launch that gave up on a wait (an aborted CTA leaves its
// arrivals counted and departs without resetting them).
extern "C" size_t tsds_linear_workspace_header_bytes(void) { return 64 + 2 * MAX_TILES * sizeof(int); }

namespace {

// The launch shape of one projection: tile counts, CTA pair or single CTA,
// pipeline stages and shared memory, stream-K or data-parallel units and the
// grid.  Shared by tsds_tc_gemm and the tsds_tc_gemm_plan query so the two
// cannot disagree.  CUDA is queried only for SM count and, with pairs, the
// resident clusters.
int plan_tc(int epi, int M, int n_out, int K, TcParams& p, int& CG, size_t& smem) {
  TSDS_RETURN_IF(M <= 0 || M > 256 || n_out <= 0 || K <= 0, TSDS_E_INVALID);
  p = TcParams{};
  p.M = M;
  p.Npad = (M + 15) / 16 * 16;
  p.n_out = n_out;
  p.K = K;
  p.KT = (K + BK - 1) / BK;
  // CTA pairs (256-row tiles, half the token rows per CTA) from g_pair_min_rows
  // rows on; not for the LM head's argmax epilogue (its candidates are per
  // 128-row tile of a vocabulary that need not fill whole pairs)
  CG = (g_pair_min_rows > 0 && M >= g_pair_min_rows && epi != EPI_ARGMAX) ? 2 : 1;
  p.tiles = epi == EPI_SWIGLU ? (n_out + 64 * CG - 1) / (64 * CG) : (n_out + TILE_J * CG - 1) / (TILE_J * CG);
  TSDS_RETURN_IF(p.tiles * CG > MAX_TILES, TSDS_E_UNSUPPORTED);
  const long long W64 = (long long)p.tiles * p.KT;
  p.tmem_cols = pow2_at_least(p.Npad);
  p.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  int ctas = g_ctas_per_sm;
  while (ctas > 1 && 2 * p.tmem_cols * ctas > 512) --ctas;
  p.b_stage_bytes = p.Npad / CG * BK * 2;  // this CTA's token rows
  int budget = SMEM_PER_SM / ctas - SMEM_RESERVE;
  if (budget > SMEM_BUDGET) budget = SMEM_BUDGET;
  p.stages = (budget - 1024) / (A_STAGE + p.b_stage_bytes);
  if (p.stages > MAX_STAGES) p.stages = MAX_STAGES;
  TSDS_RETURN_IF(p.stages < 2, TSDS_E_UNSUPPORTED);
  smem = (size_t)p.stages * (A_STAGE + p.b_stage_bytes) + 1024;
  long long units = (long long)num_sms() * ctas / CG;
  if (CG == 2) {
    const int resident = pair_clusters(epi, smem);
    TSDS_RETURN_IF(resident < 1, TSDS_E_UNSUPPORTED);
    if (resident < units) units = resident;
  }
  long long PU = W64 < units ? W64 : units;
  // stream-K over PU units, or data-parallel where tsds_tc_dp_units says so
  const int dp_units = tsds_tc_dp_units(M, p.tiles, (int)units);
  p.dp = dp_units > 0 ? 1 : 0;
  if (p.dp) PU = dp_units;
  p.P = (int)(PU * CG);
  // the kernel's stream-K bookkeeping is 32-bit
  TSDS_RETURN_IF(W64 * PU >= (1ll << 32), TSDS_E_UNSUPPORTED);
  p.W = (uint32_t)W64;
  // instruction descriptor: bf16 x bf16 -> fp32, K-major A and B, N = Npad,
  // M = 128 rows per CTA (256 for a pair)
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.Npad >> 3) << 17) |
            ((uint32_t)((TILE_J * CG) >> 4) << 24);
  return TSDS_OK;
}

}  // namespace

extern "C" int tsds_tc_gemm_plan(int epi, int M, int n_out, int K, int32_t* out) {
  TSDS_RETURN_IF(!out || (epi != EPI_STORE && epi != EPI_RESIDUAL && epi != EPI_SWIGLU && epi != EPI_ARGMAX &&
                           epi != EPI_STORE_F32),
                 TSDS_E_INVALID);
  TcParams p;
  int CG = 1;
  size_t smem = 0;
  const int st = plan_tc(epi, M, n_out, K, p, CG, smem);
  if (st != TSDS_OK) return st;
  out[0] = p.tiles;
  out[1] = p.KT;
  out[2] = p.P;
  out[3] = p.dp;
  out[4] = p.stages;
  out[5] = CG;
  return TSDS_OK;
}

namespace {
int tc_gemm_impl(int epi, const bf16* x, int ldx, const bf16* W, int w_rows, const bf16* res, int res_ld, bf16* out,
                 int ldo, int M, int n_out, int K, void* workspace, size_t workspace_bytes, float* cand_val,
                 int* cand_idx, int ldc, const bf16* norm_w, bf16* norm_out, int norm_ld, float norm_eps,
                 cudaStream_t stream) {
  TSDS_RETURN_IF(M <= 0 || M > 256, TSDS_E_INVALID);
  TSDS_RETURN_IF(workspace == nullptr || workspace_bytes < tsds_tc_workspace_bytes(M), TSDS_E_WORKSPACE);
  TSDS_RETURN_IF(!tsds_aligned16(workspace), TSDS_E_ALIGN);
  int32_t* status = (int32_t*)workspace;
  TcParams p;
  int CG = 1;
  size_t smem = 0;
  const int pst = plan_tc(epi, M, n_out, K, p, CG, smem);
  if (pst != TSDS_OK) return pst;
  p.up_off = n_out;
  p.ldo = ldo;
  p.res_ld = res_ld;
  p.res = res;
  p.out = out;
  p.counters = (int*)((char*)workspace + 64);
  p.ws = (float*)((char*)workspace + 64 + 2 * MAX_TILES * sizeof(int));
  p.status = status;
  p.cand_val = cand_val;
  p.cand_idx = cand_idx;
  p.ldc = ldc;
  p.norm_w = norm_w;
  p.norm_out = norm_out;
  p.norm_ld = norm_ld;
  p.norm_eps = norm_eps;

  CUtensorMap amap, bmap;
  int st = tsds_make_tmap_2d_bf16(&amap, W, K, w_rows, (uint64_t)K * 2, BK, 64, 1);
  if (st != TSDS_OK) return st;
  st = tsds_make_tmap_2d_bf16(&bmap, x, K, M, (uint64_t)ldx * 2, BK, p.Npad / CG, 1);
  if (st != TSDS_OK) return st;
  if (CG == 2) {
    switch (epi) {
      case EPI_STORE: return launch_tc<EPI_STORE, 2>(amap, bmap, p, smem, stream);
      case EPI_RESIDUAL: return launch_tc<EPI_RESIDUAL, 2>(amap, bmap, p, smem, stream);
      case EPI_SWIGLU: return launch_tc<EPI_SWIGLU, 2>(amap, bmap, p, smem, stream);
      case EPI_STORE_F32: return launch_tc<EPI_STORE_F32, 2>(amap, bmap, p, smem, stream);
      default: return TSDS_E_INVALID;
    }
  }
  switch (epi) {
    case EPI_STORE: return launch_tc<EPI_STORE, 1>(amap, bmap, p, smem, stream);
    case EPI_RESIDUAL: return launch_tc<EPI_RESIDUAL, 1>(amap, bmap, p, smem, stream);
    case EPI_SWIGLU: return launch_tc<EPI_SWIGLU, 1>(amap, bmap, p, smem, stream);
    case EPI_STORE_F32: return launch_tc<EPI_STORE_F32, 1>(amap, bmap, p, smem, stream);
    case EPI_ARGMAX: return launch_tc<EPI_ARGMAX, 1>(amap, bmap, p, smem, stream);
    default: return TSDS_E_INVALID;
  }
}
}  // namespace

int tsds_tc_gemm(int epi, const bf16* x, int ldx, const bf16* W, int w_rows, const bf16* res, int res_ld, bf16* out,
                 int ldo, int M, int n_out, int K, void* workspace, size_t workspace_bytes, float* cand_val,
                 int* cand_idx, int ldc, cudaStream_t stream) {
  return tc_gemm_impl(epi, x, ldx, W, w_rows, res, res_ld, out, ldo, M, n_out, K, workspace, workspace_bytes, cand_val,
                      cand_idx, ldc, nullptr, nullptr, 0, 0.f, stream);
}

int tsds_tc_gemm_residual_norm(const bf16* x, int ldx, const bf16* W, const bf16* res, int res_ld, bf16* out, int ldo,
                               int M, int n_out, int K, const bf16* norm_w, bf16* norm_out, int norm_ld, float eps,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  TSDS_RETURN_IF(!norm_w || !norm_out || (n_out % 8) != 0 || (ldo % 8) != 0 || (norm_ld % 8) != 0 ||
                     norm_ld < n_out || n_out > NORM_V * 1024,
                 TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(out) || !tsds_aligned16(norm_w) || !tsds_aligned16(norm_out), TSDS_E_ALIGN);
  return tc_gemm_impl(EPI_RESIDUAL, x, ldx, W, n_out, res, res_ld, out, ldo, M, n_out, K, workspace, workspace_bytes,
                      nullptr, nullptr, 0, norm_w, norm_out, norm_ld, eps, stream);
}
