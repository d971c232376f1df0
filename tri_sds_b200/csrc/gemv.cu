// Skinny linear layers, out[m][j] = epilogue(sum_k W[j][k] * x[m][k]).
//
// Small-M path: a CUDA-core GEMV.  A warp owns R weight rows; each lane
// streams 16-byte chunks of those rows (ld.global.nc, no L1 allocation),
// keeps its M x-rows' matching chunk in registers (L1-resident: every warp
// of the SM reads the same x), and accumulates with packed fp32 FMAs
// (fma.rn.f32x2).  One warp reduction per output at the end.
//
// Large-M path (tcgen05, TMEM accumulators) lives in gemm_tc.cu and is
// selected by tsds_linear_* when M exceeds the GEMV's row budget.  A
// split-K variant (tsds_set_gemv_splitk) spreads every projection over the
// whole GPU.
#include "common.cuh"
#include "linear.cuh"

using namespace tsds;

namespace {

__device__ __forceinline__ void fma_chunk(float2 (&acc), const uint4& w, const float2 (&xv)[4]) {
  acc = ffma2(make_float2(bf_lo(w.x), bf_hi(w.x)), xv[0], acc);
  acc = ffma2(make_float2(bf_lo(w.y), bf_hi(w.y)), xv[1], acc);
  acc = ffma2(make_float2(bf_lo(w.z), bf_hi(w.z)), xv[2], acc);
  acc = ffma2(make_float2(bf_lo(w.w), bf_hi(w.w)), xv[3], acc);
}

// Rows per warp: enough to reuse each x chunk, few enough to keep the
// R x MT accumulators in registers.
template <int MT>
struct GemvCfg {
  static constexpr int R = MT <= 2 ? 8 : (MT <= 4 ? 4 : 2);
};

template <int MT, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(const bf16* __restrict__ x, int ldx, const bf16* __restrict__ W,
                                                   const bf16* res, int res_ld, bf16* out, int ldo, int n_out,
                                                   int K) {
  constexpr int R = GemvCfg<MT>::R;
  constexpr int OUT_PER_WARP = EPI == EPI_SWIGLU ? R / 2 : R;
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = (blockIdx.x * 8 + warp) * OUT_PER_WARP;
  if (j0 >= n_out) return;
  int64_t row_off[R];
  bool valid[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int j, row;
    if (EPI == EPI_SWIGLU) {
      j = j0 + (r % OUT_PER_WARP);
      row = r < OUT_PER_WARP ? j : n_out + j;  // gate rows, then up rows
    } else {
      j = j0 + r;
      row = j;
    }
    valid[r] = j < n_out;
    row_off[r] = (int64_t)(valid[r] ? row : 0) * K;
  }
  float2 acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = make_float2(0.f, 0.f);

  const int nchunk = K >> 3;
#pragma unroll 2
  for (int c = lane; c < nchunk; c += 32) {
    uint4 w[R];
#pragma unroll
    for (int r = 0; r < R; ++r) w[r] = ldg16_stream(W + row_off[r] + (int64_t)c * 8);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4 xv = ldg16(x + (int64_t)m * ldx + c * 8);
      const float2 xf[4] = {make_float2(bf_lo(xv.x), bf_hi(xv.x)), make_float2(bf_lo(xv.y), bf_hi(xv.y)),
                            make_float2(bf_lo(xv.z), bf_hi(xv.z)), make_float2(bf_lo(xv.w), bf_hi(xv.w))};
#pragma unroll
      for (int r = 0; r < R; ++r) fma_chunk(acc[r][m], w[r], xf);
    }
  }
  // Warp reduction; afterwards every lane holds every sum.
  float sum[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) sum[r][m] = warp_sum(acc[r][m].x + acc[r][m].y);

  // Epilogue: lane i handles output (r, m) = (i / MT, i % MT).
#pragma unroll
  for (int r = 0; r < OUT_PER_WARP; ++r) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (lane != ((r * MT + m) & 31)) continue;
      const int j = j0 + r;
      if (j >= n_out) continue;
      const int64_t o = (int64_t)m * ldo + j;
      if (EPI == EPI_STORE) {
        out[o] = f2bf(sum[r][m]);
      } else if (EPI == EPI_STORE_F32) {
        reinterpret_cast<float*>(out)[o] = sum[r][m];
      } else if (EPI == EPI_RESIDUAL) {
        out[o] = f2bf(bf2f(res[(int64_t)m * res_ld + j]) + rbf(sum[r][m]));
      } else {  // SWIGLU: silu on the bf16 gate, product of bf16 values (qwen_model.py:139-142)
        const float g = rbf(sum[r][m]);
        const float u = rbf(sum[r + OUT_PER_WARP][m]);
        const float s = rbf(g / (1.0f + expf(-g)));
        out[o] = f2bf(s * u);
      }
    }
  }
}

// ---- split-K variant ---------------------------------------------------------
// A CTA owns R weight rows (for SwiGLU R/2 outputs: their gate rows, then
// their up rows) and its 256 threads sweep K together: thread t takes the
// 16-byte chunks t, t + 256, ... of every row, so each pass reads 4 KB of a
// row contiguously, and a grid of n_out / R CTAs covers every SM even for
// the 2560- and 5120-output projections (where one warp per R rows leaves
// most SMs idle).  Per-thread partials are summed by warp shuffles, then
// over the 8 warps in warp order through shared memory: the same order on
// every launch.  The epilogues are those of gemv_kernel.
template <int MT>
struct SplitCfg {
  static constexpr int R = MT <= 2 ? 8 : (MT <= 4 ? 4 : 2);
};

template <int MT, int EPI>
__global__ void __launch_bounds__(256) gemv_splitk_kernel(const bf16* __restrict__ x, int ldx,
                                                          const bf16* __restrict__ W, const bf16* res, int res_ld,
                                                          bf16* out, int ldo, int n_out, int K) {
  constexpr int R = SplitCfg<MT>::R;
  constexpr int OUT = EPI == EPI_SWIGLU ? R / 2 : R;
  __shared__ float part[8][R * MT];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = blockIdx.x * OUT;
  int64_t row_off[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int j, row;
    if (EPI == EPI_SWIGLU) {
      j = j0 + (r % OUT);
      row = r < OUT ? j : n_out + j;  // gate rows, then up rows
    } else {
      j = j0 + r;
      row = j;
    }
    row_off[r] = (int64_t)(j < n_out ? row : 0) * K;  // rows past the end read row 0, unused
  }
  float2 acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = make_float2(0.f, 0.f);

  const int nchunk = K >> 3;
#pragma unroll 2
  for (int c = threadIdx.x; c < nchunk; c += 256) {
    uint4 w[R];
#pragma unroll
    for (int r = 0; r < R; ++r) w[r] = ldg16_stream(W + row_off[r] + (int64_t)c * 8);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4 xv = ldg16(x + (int64_t)m * ldx + c * 8);
      const float2 xf[4] = {make_float2(bf_lo(xv.x), bf_hi(xv.x)), make_float2(bf_lo(xv.y), bf_hi(xv.y)),
                            make_float2(bf_lo(xv.z), bf_hi(xv.z)), make_float2(bf_lo(xv.w), bf_hi(xv.w))};
#pragma unroll
      for (int r = 0; r < R; ++r) fma_chunk(acc[r][m], w[r], xf);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float v = warp_sum(acc[r][m].x + acc[r][m].y);
      if (lane == 0) part[warp][r * MT + m] = v;
    }
  __syncthreads();
  if (threadIdx.x >= OUT * MT) return;
  const int r = threadIdx.x / MT, m = threadIdx.x % MT;
  const int j = j0 + r;
  if (j >= n_out) return;
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) sum += part[q][r * MT + m];
  const int64_t o = (int64_t)m * ldo + j;
  if (EPI == EPI_STORE) {
    out[o] = f2bf(sum);
  } else if (EPI == EPI_STORE_F32) {
    reinterpret_cast<float*>(out)[o] = sum;
  } else if (EPI == EPI_RESIDUAL) {
    out[o] = f2bf(bf2f(res[(int64_t)m * res_ld + j]) + rbf(sum));
  } else {  // SWIGLU: silu on the bf16 gate, product of bf16 values (qwen_model.py:139-142)
    float up = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) up += part[q][(r + OUT) * MT + m];
    const float g = rbf(sum);
    const float u = rbf(up);
    const float s = rbf(g / (1.0f + expf(-g)));
    out[o] = f2bf(s * u);
  }
}

// 1: tsds_linear* rows up to the GEMV limit run gemv_splitk_kernel.
std::atomic<int> g_gemv_splitk{0};

template <int EPI>
int launch_gemv_rows(const bf16* x, int ldx, const bf16* W, const bf16* res, int res_ld, bf16* out, int ldo, int M,
                     int n_out, int K, cudaStream_t stream) {
  const bool splitk = g_gemv_splitk.load(std::memory_order_relaxed) != 0;
  // process up to 8 rows per launch
  for (int m0 = 0; m0 < M; m0 += 8) {
    const int mt = M - m0 < 8 ? M - m0 : 8;
    const bf16* xs = x + (int64_t)m0 * ldx;
    const bf16* rs = res ? res + (int64_t)m0 * res_ld : nullptr;
    bf16* os = EPI == EPI_STORE_F32 ? reinterpret_cast<bf16*>(reinterpret_cast<float*>(out) + (int64_t)m0 * ldo)
                                    : out + (int64_t)m0 * ldo;
#define TSDS_GEMV_CASE(MTV)                                                                          \
  case MTV: {                                                                                        \
    if (splitk) {                                                                                    \
      constexpr int OUT = EPI == EPI_SWIGLU ? SplitCfg<MTV>::R / 2 : SplitCfg<MTV>::R;               \
      tsds_launch(gemv_splitk_kernel<MTV, EPI>, dim3((n_out + OUT - 1) / OUT), dim3(256), 0, stream, xs, ldx, W, \
                  rs, res_ld, os, ldo, n_out, K);                                                    \
      break;                                                                                         \
    }                                                                                                \
    constexpr int R = GemvCfg<MTV>::R;                                                               \
    constexpr int OPW = EPI == EPI_SWIGLU ? R / 2 : R;                                               \
    const int warps = (n_out + OPW - 1) / OPW;                                                       \
    tsds_launch(gemv_kernel<MTV, EPI>, dim3((warps + 7) / 8), dim3(256), 0, stream, xs, ldx, W, rs, res_ld, os, ldo, \
                n_out, K);                                                                            \
    break;                                                                                           \
  }
    switch (mt) {
      TSDS_GEMV_CASE(1)
      TSDS_GEMV_CASE(2)
      TSDS_GEMV_CASE(3)
      TSDS_GEMV_CASE(4)
      TSDS_GEMV_CASE(5)
      TSDS_GEMV_CASE(6)
      TSDS_GEMV_CASE(7)
      TSDS_GEMV_CASE(8)
    }
#undef TSDS_GEMV_CASE
    int st = tsds_launch_status();
    if (st != TSDS_OK) return st;
  }
  return TSDS_OK;
}

}  // namespace

extern "C" void tsds_set_gemv_splitk(int on) { g_gemv_splitk.store(on ? 1 : 0, std::memory_order_relaxed); }
extern "C" int tsds_get_gemv_splitk(void) { return g_gemv_splitk.load(std::memory_order_relaxed); }

int tsds_gemv_dispatch(int epi, const bf16* x, int ldx, const bf16* W, const bf16* res, int res_ld, bf16* out, int ldo,
                       int M, int n_out, int K, cudaStream_t stream) {
  switch (epi) {
    case EPI_STORE: return launch_gemv_rows<EPI_STORE>(x, ldx, W, res, res_ld, out, ldo, M, n_out, K, stream);
    case EPI_RESIDUAL: return launch_gemv_rows<EPI_RESIDUAL>(x, ldx, W, res, res_ld, out, ldo, M, n_out, K, stream);
    case EPI_SWIGLU: return launch_gemv_rows<EPI_SWIGLU>(x, ldx, W, res, res_ld, out, ldo, M, n_out, K, stream);
    case EPI_STORE_F32:
      return launch_gemv_rows<EPI_STORE_F32>(x, ldx, W, res, res_ld, out, ldo, M, n_out, K, stream);
  }
  return TSDS_E_INVALID;
}
