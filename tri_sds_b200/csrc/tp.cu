// Tensor-parallel glue: residual add of all-reduced fp32 partials, merge of
// per-rank LM-head argmax candidates, and reassembly of vocab-sharded logits.
#include "common.cuh"

using namespace tsds;

namespace {

// x = bf16(x + bf16(sum)): the reference's rounding of `x + proj` with proj the
// bf16 product (qwen_model.py:133-134,143-144), proj summed across ranks in fp32.
__global__ void residual_add_f32_kernel(bf16* __restrict__ x, const float* __restrict__ p, int64_t n) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = f2bf(bf2f(x[i]) + rbf(p[i]));
}

__global__ void argmax_merge_kernel(const float* __restrict__ vals, const int64_t* __restrict__ idx, int M, int tp,
                                    int64_t shard, int64_t* __restrict__ out, int stride) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int r = 0; r < tp; ++r) {
    const float v = vals[(int64_t)r * M + m];
    const int64_t i = idx[(int64_t)r * M + m] + r * shard;
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  out[(int64_t)m * stride] = bi == INT64_MAX ? 0 : bi;
}

// src [tp][M][Vs] -> dst [M][tp * Vs]; 16-byte moves when Vs % 8 == 0
__global__ void gather_shards_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst, int tp, int M, int vs) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, r = blockIdx.y;
  const bf16* s = src + ((int64_t)r * M + m) * vs;
  bf16* d = dst + (int64_t)m * tp * vs + (int64_t)r * vs;
  if ((vs & 7) == 0) {
    for (int c = threadIdx.x; c < vs / 8; c += blockDim.x)
      reinterpret_cast<uint4*>(d)[c] = reinterpret_cast<const uint4*>(s)[c];
  } else {
    for (int c = threadIdx.x; c < vs; c += blockDim.x) d[c] = s[c];
  }
}

}  // namespace

extern "C" int tsds_residual_add_f32(void* x, const float* partial, int M, int N, tsds_stream_t stream) {
  TSDS_RETURN_IF(!x || !partial || M <= 0 || N <= 0, TSDS_E_INVALID);
  const int64_t n = (int64_t)M * N;
  const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  tsds_launch(residual_add_f32_kernel, dim3(blocks), dim3(256), 0, stream, (bf16*)x, partial, n);
  return tsds_launch_status();
}

extern "C" int tsds_argmax_merge(const float* vals, const int64_t* idx, int M, int tp, int64_t vocab_shard,
                                 int64_t* out, int out_stride, tsds_stream_t stream) {
  TSDS_RETURN_IF(!vals || !idx || !out || M <= 0 || tp <= 0 || out_stride <= 0, TSDS_E_INVALID);
  tsds_launch(argmax_merge_kernel, dim3((M + 127) / 128), dim3(128), 0, stream, vals, idx, M, tp, vocab_shard, out,
              out_stride);
  return tsds_launch_status();
}

extern "C" int tsds_gather_shards(const void* src, void* dst, int tp, int M, int vocab_shard, tsds_stream_t stream) {
  TSDS_RETURN_IF(!src || !dst || tp <= 0 || M <= 0 || vocab_shard <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF((vocab_shard % 8) == 0 && (!tsds_aligned16(src) || !tsds_aligned16(dst)), TSDS_E_ALIGN);
  tsds_launch(gather_shards_kernel, dim3(M, tp), dim3(256), 0, stream, (const bf16*)src, (bf16*)dst, tp, M,
              vocab_shard);
  return tsds_launch_status();
}
