// Per-lane arithmetic of the QK-norm + RoPE step, shared by the standalone
// kernel (elementwise.cu) and the fused epilogue of the fused-layer
// kernel (fused_layer.cu) so both round identically.  Head dim 128; lane l of a warp
// holds elements 2l, 2l+1 (first half) and 64+2l, 65+2l (second half), i.e.
// both members of its two rotate-half pairs.
#pragma once

#include "common.cuh"

namespace tsds {

// g0 / g1: the lane's norm weights at 2l, 2l+1 and 64+2l, 65+2l
__device__ __forceinline__ void qk_norm_pair_w(float (&v)[4], uint32_t g0, uint32_t g1, float eps) {
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
  ss = warp_sum(ss);
  const float rstd = 1.0f / sqrtf(ss / 128.0f + eps);
  v[0] = rbf(v[0] * rstd * bf_lo(g0));
  v[1] = rbf(v[1] * rstd * bf_hi(g0));
  v[2] = rbf(v[2] * rstd * bf_lo(g1));
  v[3] = rbf(v[3] * rstd * bf_hi(g1));
}

__device__ __forceinline__ void qk_norm_pair(float (&v)[4], const bf16* __restrict__ gw, int lane, float eps) {
  qk_norm_pair_w(v, *reinterpret_cast<const uint32_t*>(gw + 2 * lane),
                 *reinterpret_cast<const uint32_t*>(gw + 64 + 2 * lane), eps);
}

// RoPE (qwen_model.py:17-24) in bf16 with bf16 tables (qwen_model.py:8-14):
// out1 = bf16(bf16(x1*c) - bf16(x2*s)), out2 = bf16(bf16(x2*c) + bf16(x1*s));
// stores the rotated head row at dst.
// cw / sw: the lane's cos and sin pairs at 2l, 2l+1 of the row's position
__device__ __forceinline__ void rope_store_cs(const float (&v)[4], uint32_t cw, uint32_t sw, int lane, bf16* dst) {
  const float c0 = bf_lo(cw), c1 = bf_hi(cw), s0 = bf_lo(sw), s1 = bf_hi(sw);
  // pairs (v[0], v[2]) at index 2l and (v[1], v[3]) at index 2l+1
  const float o0 = rbf(rbf(v[0] * c0) - rbf(v[2] * s0));
  const float o2 = rbf(rbf(v[2] * c0) + rbf(v[0] * s0));
  const float o1 = rbf(rbf(v[1] * c1) - rbf(v[3] * s1));
  const float o3 = rbf(rbf(v[3] * c1) + rbf(v[1] * s1));
  *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack_bf2(o0, o1);
  *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack_bf2(o2, o3);
}

__device__ __forceinline__ void rope_store(const float (&v)[4], const bf16* __restrict__ cos_t,
                                           const bf16* __restrict__ sin_t, int pos, int lane, bf16* dst) {
  constexpr int D = 128;
  rope_store_cs(v, *reinterpret_cast<const uint32_t*>(cos_t + (int64_t)pos * (D / 2) + 2 * lane),
                *reinterpret_cast<const uint32_t*>(sin_t + (int64_t)pos * (D / 2) + 2 * lane), lane, dst);
}

}  // namespace tsds
