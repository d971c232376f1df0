// LM head + greedy pick (qwen_model.py:191-193,205; eagle_head.py:119-121).
//
// logits[m][v] = bf16(sum_k x[m][k] * W[v][k]); argmax over v with
// torch.argmax semantics on the bf16-rounded logits (largest value, lowest
// index on ties).  Pass 1 streams the vocab rows (the GEMV inner loop of
// gemv.cu) and leaves one (value, index) candidate per CTA and token row;
// pass 2 reduces the candidates per row in CTA order.
#include "common.cuh"
#include "linear.cuh"

using namespace tsds;

namespace {

template <int MT>
struct LmCfg {
  static constexpr int R = MT <= 2 ? 8 : (MT <= 4 ? 4 : 2);
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <int MT>
__global__ void __launch_bounds__(256) lm_head_pass1(const bf16* __restrict__ x, int ldx, const bf16* __restrict__ W,
                                                     bf16* __restrict__ logits, int vocab, int K,
                                                     float* __restrict__ cand_val, int* __restrict__ cand_idx,
                                                     int ldc) {
  constexpr int R = LmCfg<MT>::R;
  __shared__ float s_val[8][MT];
  __shared__ int s_idx[8][MT];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v0 = (blockIdx.x * 8 + warp) * R;
  float2 acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = make_float2(0.f, 0.f);
  if (v0 < vocab) {
    int64_t off[R];
#pragma unroll
    for (int r = 0; r < R; ++r) off[r] = (int64_t)(v0 + r < vocab ? v0 + r : v0) * K;
    const int nchunk = K >> 3;
#pragma unroll 2
    for (int c = lane; c < nchunk; c += 32) {
      uint4 w[R];
#pragma unroll
      for (int r = 0; r < R; ++r) w[r] = ldg16_stream(W + off[r] + (int64_t)c * 8);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const uint4 xv = ldg16(x + (int64_t)m * ldx + c * 8);
        const float2 xf[4] = {make_float2(bf_lo(xv.x), bf_hi(xv.x)), make_float2(bf_lo(xv.y), bf_hi(xv.y)),
                              make_float2(bf_lo(xv.z), bf_hi(xv.z)), make_float2(bf_lo(xv.w), bf_hi(xv.w))};
#pragma unroll
        for (int r = 0; r < R; ++r) {
          acc[r][m] = ffma2(make_float2(bf_lo(w[r].x), bf_hi(w[r].x)), xf[0], acc[r][m]);
          acc[r][m] = ffma2(make_float2(bf_lo(w[r].y), bf_hi(w[r].y)), xf[1], acc[r][m]);
          acc[r][m] = ffma2(make_float2(bf_lo(w[r].z), bf_hi(w[r].z)), xf[2], acc[r][m]);
          acc[r][m] = ffma2(make_float2(bf_lo(w[r].w), bf_hi(w[r].w)), xf[3], acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float lv = rbf(warp_sum(acc[r][m].x + acc[r][m].y));  // the reference's bf16 logit
      const int v = v0 + r;
      if (v < vocab) {
        if (logits && lane == ((r * MT + m) & 31)) logits[(int64_t)m * vocab + v] = f2bf(lv);
        if (better(lv, v, bv, bi)) {
          bv = lv;
          bi = v;
        }
      }
    }
    if (lane == 0) {
      s_val[warp][m] = bv;
      s_idx[warp][m] = bi;
    }
  }
  __syncthreads();
  if (threadIdx.x < MT) {
    const int m = threadIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < 8; ++w)
      if (better(s_val[w][m], s_idx[w][m], bv, bi)) {
        bv = s_val[w][m];
        bi = s_idx[w][m];
      }
    cand_val[(int64_t)m * ldc + blockIdx.x] = bv;
    cand_idx[(int64_t)m * ldc + blockIdx.x] = bi;
  }
}

__global__ void __launch_bounds__(256) lm_head_pass2(const float* __restrict__ cand_val,
                                                     const int* __restrict__ cand_idx, int ncand, int ldc,
                                                     int64_t* __restrict__ out, int out_stride,
                                                     float* __restrict__ out_val) {
  __shared__ float s_val[256];
  __shared__ int s_idx[256];
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < ncand; c += 256) {
    const float v = cand_val[(int64_t)m * ldc + c];
    const int i = cand_idx[(int64_t)m * ldc + c];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  s_val[threadIdx.x] = bv;
  s_idx[threadIdx.x] = bi;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s && better(s_val[threadIdx.x + s], s_idx[threadIdx.x + s], s_val[threadIdx.x],
                                  s_idx[threadIdx.x])) {
      s_val[threadIdx.x] = s_val[threadIdx.x + s];
      s_idx[threadIdx.x] = s_idx[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[(int64_t)m * out_stride] = s_idx[0] == 0x7fffffff ? 0 : s_idx[0];
    if (out_val) out_val[m] = s_val[0];
  }
}

int lm_blocks(int mt, int vocab) {
  const int R = mt <= 2 ? 8 : (mt <= 4 ? 4 : 2);
  return (vocab + 8 * R - 1) / (8 * R);
}

}  // namespace

// Workspace: [tcgen05 region at offset 0: status word and tile counters at
// fixed offsets (they persist across calls), then M-dependent partials]
// [candidates: M x ldc values][M x ldc indices].  Whatever M a call has,
// nothing but the counters themselves ever writes the counter words.
static int lm_ldc(int vocab) {
  const int a = lm_blocks(8, vocab), b = (vocab + 127) / 128;
  return a > b ? a : b;
}

static size_t round256(size_t x) { return (x + 255) / 256 * 256; }

static size_t lm_cand_offset(int M) {
  const size_t header = tsds_tc_workspace_bytes(0);  // status + counters, no partials
  return round256(M > tsds_gemv_rows_limit() ? tsds_tc_workspace_bytes(M < 256 ? M : 256) : header);
}

extern "C" size_t tsds_lm_head_workspace_bytes(int M, int vocab) {
  if (M <= 0 || vocab <= 0) return 0;
  return lm_cand_offset(M) + (size_t)M * lm_ldc(vocab) * (sizeof(float) + sizeof(int));
}

extern "C" int tsds_lm_head_argmax(const void* x, int ldx, const void* W, void* logits_out, int64_t* argmax_out,
                                   int argmax_stride, float* argmax_val, int M, int vocab, int K, void* workspace,
                                   size_t workspace_bytes, tsds_stream_t stream) {
  TSDS_RETURN_IF(!x || !W || !argmax_out || M <= 0 || vocab <= 0 || K <= 0 || (K % 8) || ldx < K ||
                     argmax_stride <= 0,
                 TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(x) || !tsds_aligned16(W) || (ldx % 8), TSDS_E_ALIGN);
  TSDS_RETURN_IF(workspace_bytes < tsds_lm_head_workspace_bytes(M, vocab) || !workspace, TSDS_E_WORKSPACE);
  const int ldc = lm_ldc(vocab);
  float* cval = (float*)((char*)workspace + lm_cand_offset(M));
  int* cidx = (int*)((char*)cval + (size_t)M * ldc * sizeof(float));
  if (M > tsds_gemv_rows_limit()) {
    char* tcws = (char*)workspace;
    const size_t tcb = lm_cand_offset(M);
    const int tiles = (vocab + 127) / 128;
    for (int m0 = 0; m0 < M; m0 += 256) {
      const int mc = M - m0 < 256 ? M - m0 : 256;
      int st = tsds_tc_gemm(EPI_ARGMAX, (const bf16*)x + (int64_t)m0 * ldx, ldx, (const bf16*)W, vocab, nullptr, 0,
                            logits_out ? (bf16*)logits_out + (int64_t)m0 * vocab : nullptr, vocab, mc, vocab, K, tcws,
                            tcb, cval + (int64_t)m0 * ldc, cidx + (int64_t)m0 * ldc, ldc, stream);
      if (st != TSDS_OK) return st;
      tsds_launch(lm_head_pass2, dim3(mc), dim3(256), 0, stream, (const float*)(cval + (int64_t)m0 * ldc),
                  (const int*)(cidx + (int64_t)m0 * ldc), tiles, ldc, argmax_out + (int64_t)m0 * argmax_stride,
                  argmax_stride, argmax_val ? argmax_val + m0 : (float*)nullptr);
      st = tsds_launch_status();
      if (st != TSDS_OK) return st;
    }
    return TSDS_OK;
  }
  for (int m0 = 0; m0 < M; m0 += 8) {
    const int mt = M - m0 < 8 ? M - m0 : 8;
    const bf16* xs = (const bf16*)x + (int64_t)m0 * ldx;
    bf16* ls = logits_out ? (bf16*)logits_out + (int64_t)m0 * vocab : nullptr;
    const int nb = lm_blocks(mt, vocab);
    float* cv = cval + (int64_t)m0 * ldc;
    int* ci = cidx + (int64_t)m0 * ldc;
#define TSDS_LM_CASE(MTV)                                                                                    \
  case MTV:                                                                                                  \
    tsds_launch(lm_head_pass1<MTV>, dim3(nb), dim3(256), 0, stream, xs, ldx, (const bf16*)W, ls, vocab, K, cv, ci, \
                ldc);                                                                                   \
    break;
    switch (mt) {
      TSDS_LM_CASE(1)
      TSDS_LM_CASE(2)
      TSDS_LM_CASE(3)
      TSDS_LM_CASE(4)
      TSDS_LM_CASE(5)
      TSDS_LM_CASE(6)
      TSDS_LM_CASE(7)
      TSDS_LM_CASE(8)
    }
#undef TSDS_LM_CASE
    int st = tsds_launch_status();
    if (st != TSDS_OK) return st;
    tsds_launch(lm_head_pass2, dim3(mt), dim3(256), 0, stream, (const float*)cv, (const int*)ci, nb, ldc,
                argmax_out + (int64_t)m0 * argmax_stride, argmax_stride,
                argmax_val ? argmax_val + m0 : (float*)nullptr);
    st = tsds_launch_status();
    if (st != TSDS_OK) return st;
  }
  return TSDS_OK;
}
