// Row-wise kernels of the verify step: embedding gather, RMSNorm,
// QK-norm + RoPE + KV-cache write, chain bookkeeping, greedy acceptance.
#include "common.cuh"
#include "rowops.cuh"

using namespace tsds;

// ---------------------------------------------------------------------------
// Embedding gather (qwen_model.py:188,199).  One CTA per token row; 16-byte
// vectors.  An id outside [0, vocab) yields a zero row (no out-of-range read).
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int64_t* __restrict__ ids, int ids_stride, const bf16* __restrict__ table,
                             bf16* __restrict__ out, int N, int vocab) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const int64_t id = ids[(int64_t)m * ids_stride];
  const bool ok = id >= 0 && id < vocab;
  const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * (int64_t)N);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)m * N);
  for (int c = threadIdx.x; c < N / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

extern "C" int tsds_embed(const int64_t* ids, int ids_stride, const void* table, void* out, int M, int N,
                          int vocab, tsds_stream_t stream) {
  TSDS_RETURN_IF(M <= 0 || N <= 0 || (N % 8) != 0 || vocab <= 0 || ids_stride <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(table) || !tsds_aligned16(out), TSDS_E_ALIGN);
  tsds_launch(embed_kernel, dim3(M), dim3(128), 0, stream, ids, ids_stride, (const bf16*)table, (bf16*)out, N, vocab);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// RMSNorm (norm.py:42-72): fp32 sum of squares, rstd = 1/sqrt(ms + eps),
// y = x * rstd * w in fp32, a single rounding to bf16.
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                       bf16* __restrict__ out, int n, int ldx, int ldo, float eps) {
  __shared__ float red[8];
  constexpr int V = 4;  // 16-byte vectors a thread holds in registers: rows of n <= 8192
  pdl_trigger();
  const int nv = n / 8;
  const bf16* xr = x + (int64_t)blockIdx.x * ldx;
  bf16* orow = out + (int64_t)blockIdx.x * ldo;
  if (nv <= V * 256) {
    // One read of the row into registers; the weights are constant and are
    // read before the wait, so after it only the row's read is on the
    // latency path.  Same arithmetic and order as the loop below.
    uint4 g[V], xv[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = threadIdx.x + i * 256;
      if (c < nv) g[i] = ldg16(w + c * 8);
    }
    pdl_wait();
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = threadIdx.x + i * 256;
      if (c < nv) xv[i] = ldg16(xr + c * 8);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = threadIdx.x + i * 256;
      if (c < nv) {
        const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float a = bf_lo(u[k]), b = bf_hi(u[k]);
          ss = fmaf(a, a, ss);
          ss = fmaf(b, b, ss);
        }
      }
    }
    ss = block_sum<256>(ss, red);
    const float rstd = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = threadIdx.x + i * 256;
      if (c < nv) {
        const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        const uint32_t gw[4] = {g[i].x, g[i].y, g[i].z, g[i].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = pack_bf2(bf_lo(u[k]) * rstd * bf_lo(gw[k]), bf_hi(u[k]) * rstd * bf_hi(gw[k]));
        *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    return;
  }
  pdl_wait();
  float ss = 0.f;
  for (int c = threadIdx.x; c < n / 8; c += 256) {
    uint4 v = ldg16(xr + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = bf_lo(u[i]), b = bf_hi(u[i]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  ss = block_sum<256>(ss, red);
  const float rstd = 1.0f / sqrtf(ss / (float)n + eps);
  for (int c = threadIdx.x; c < n / 8; c += 256) {
    uint4 v = ldg16(xr + c * 8);
    uint4 g = ldg16(w + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = pack_bf2(bf_lo(u[i]) * rstd * bf_lo(gw[i]), bf_hi(u[i]) * rstd * bf_hi(gw[i]));
    *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

extern "C" int tsds_rms_norm(const void* x, const void* w, void* out, int rows, int n, int ldx, int ldo, float eps,
                             tsds_stream_t stream) {
  TSDS_RETURN_IF(rows <= 0 || n <= 0 || (n % 8) != 0 || ldx < n || ldo < n, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(x) || !tsds_aligned16(w) || !tsds_aligned16(out) || (ldx % 8) || (ldo % 8),
                 TSDS_E_ALIGN);
  tsds_launch(rms_norm_kernel, dim3(rows), dim3(256), 0, stream, (const bf16*)x, (const bf16*)w, (bf16*)out, n, ldx,
              ldo, eps);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// Chain bookkeeping: starts[b] = base[b] + offset; positions[b*T+t] = starts[b]+t.
// ---------------------------------------------------------------------------
__global__ void prep_chain_kernel(const int32_t* __restrict__ base, int offset, int B, int T,
                                  int32_t* __restrict__ starts, int32_t* __restrict__ positions) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int b = i / T, t = i - b * T;
  const int s = base[b] + offset;
  if (t == 0 && starts) starts[b] = s;
  if (positions) positions[i] = s + t;
}

extern "C" int tsds_prep_chain(const int32_t* base, int offset, int B, int T, int32_t* starts, int32_t* positions,
                               tsds_stream_t stream) {
  TSDS_RETURN_IF(B <= 0 || T <= 0 || base == nullptr, TSDS_E_INVALID);
  const int n = B * T;
  tsds_launch(prep_chain_kernel, dim3((n + 127) / 128), dim3(128), 0, stream, base, offset, B, T, starts, positions);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE + KV write, head_dim 128.  One warp per (token row, head
// slot); slots [0,Hq) are q heads, [Hq, Hq+Hkv) k heads, then v heads.
// Lane l owns elements 2l, 2l+1 (first half) and 64+2l, 65+2l (second half),
// i.e. both members of its two rotate-half pairs.
// RoPE follows qwen_model.py:17-24 in bf16: out1 = bf16(bf16(x1*c) - bf16(x2*s)),
// out2 = bf16(bf16(x2*c) + bf16(x1*s)) with bf16 tables (qwen_model.py:8-14).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(
    const bf16* __restrict__ qkv, const bf16* __restrict__ q_norm_w, const bf16* __restrict__ k_norm_w,
    const bf16* __restrict__ cos_t, const bf16* __restrict__ sin_t, const int32_t* __restrict__ positions,
    const int32_t* __restrict__ starts, bf16* __restrict__ q_out, bf16* __restrict__ k_cache,
    bf16* __restrict__ v_cache, int M, int T, int Hq, int Hkv, int S, int rope_len, float eps,
    const int64_t* __restrict__ out_loc, int64_t pool_rows, int32_t* __restrict__ status) {
  constexpr int D = 128;
  pdl_trigger();
  const int slots = Hq + 2 * Hkv;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int m = gw / slots, h = gw - m * slots;
  const bool is_q = h < Hq;
  const bf16* nw = is_q ? q_norm_w : k_norm_w;
  // the head's norm weights are constant: read before the wait, so only the
  // previous kernels' outputs are on the latency path after it
  uint32_t g0 = 0, g1 = 0;
  if (gw < M * slots && h < Hq + Hkv && nw) {
    g0 = *reinterpret_cast<const uint32_t*>(nw + 2 * lane);
    g1 = *reinterpret_cast<const uint32_t*>(nw + 64 + 2 * lane);
  }
  pdl_wait();
  if (gw >= M * slots) return;
  const int qkv_dim = slots * D;
  const bf16* src = qkv + (int64_t)m * qkv_dim + (int64_t)h * D;
  const uint32_t a = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
  const uint32_t c = *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane);
  float v[4] = {bf_lo(a), bf_hi(a), bf_lo(c), bf_hi(c)};
  const int b = m / T, t = m - b * T;
  const int pos = positions[m];
  // the rotation of this position, requested before the norm needs the row
  uint32_t cw = 0, sw = 0;
  if (h < Hq + Hkv && pos >= 0 && pos < rope_len) {
    cw = *reinterpret_cast<const uint32_t*>(cos_t + (int64_t)pos * (D / 2) + 2 * lane);
    sw = *reinterpret_cast<const uint32_t*>(sin_t + (int64_t)pos * (D / 2) + 2 * lane);
  }
  // K/V row of head kvh: the contiguous cache's row starts[b] + t of slab
  // (b, kvh), or (pooled caches, out_loc given) pool row out_loc[m], head kvh
  int64_t slot = 0;
  int row_in_seq = 0;
  if (out_loc) {
    slot = out_loc[m];
    if (slot < 0 || slot >= pool_rows) {  // never written out of the pool
      if (lane == 0 && h == Hq) atomicExch(status, TSDS_E_INDEX);
      return;
    }
  } else {
    row_in_seq = starts[b] + t;
  }
  // rows / positions past the cache or the RoPE table are never written
  // (the host keeps lengths below S; this only prevents out-of-range stores)
  if (row_in_seq < 0 || row_in_seq >= S || pos < 0 || pos >= rope_len) return;
  auto kv_row = [&](int kvh) -> int64_t {
    return out_loc ? slot * Hkv + kvh : ((int64_t)b * Hkv + kvh) * S + row_in_seq;
  };
  if (h >= Hq + Hkv) {  // v head: copy into the cache
    const int kvh = h - Hq - Hkv;
    const int64_t row = kv_row(kvh);
    bf16* dst = v_cache + row * D;
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = a;
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = c;
    return;
  }
  if (nw) qk_norm_pair_w(v, g0, g1, eps);
  bf16* dst;
  if (is_q) {
    dst = q_out + ((int64_t)m * Hq + h) * D;
  } else {
    const int kvh = h - Hq;
    dst = k_cache + kv_row(kvh) * D;
  }
  rope_store_cs(v, cw, sw, lane, dst);
}

extern "C" int tsds_qk_norm_rope_kv(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                                    const void* sin, const int32_t* positions, const int32_t* starts, void* q_out,
                                    void* k_cache, void* v_cache, int B, int T, int Hq, int Hkv, int D, int S,
                                    int rope_len, float eps, tsds_stream_t stream) {
  TSDS_RETURN_IF(D != 128, TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF(B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || (Hq % Hkv) != 0 || S <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(!qkv || !cos || !sin || !positions || !starts || !q_out || !k_cache || !v_cache, TSDS_E_INVALID);
  const int M = B * T;
  const int warps = M * (Hq + 2 * Hkv);
  tsds_launch(qk_norm_rope_kv_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream,
      (const bf16*)qkv, (const bf16*)q_norm_w, (const bf16*)k_norm_w, (const bf16*)cos, (const bf16*)sin, positions,
      starts, (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, M, T, Hq, Hkv, S, rope_len, eps, (const int64_t*)nullptr,
      (int64_t)0, (int32_t*)nullptr);
  return tsds_launch_status();
}

extern "C" int tsds_qk_norm_rope_kv_paged(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                                          const void* sin, const int32_t* positions, const int64_t* out_loc,
                                          void* q_out, void* k_pool, void* v_pool, int M, int Hq, int Hkv, int D,
                                          int64_t pool_rows, int rope_len, float eps, int32_t* status,
                                          tsds_stream_t stream) {
  TSDS_RETURN_IF(D != 128, TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF(M <= 0 || Hq <= 0 || Hkv <= 0 || (Hq % Hkv) != 0 || pool_rows <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(!qkv || !cos || !sin || !positions || !out_loc || !q_out || !k_pool || !v_pool || !status,
                 TSDS_E_INVALID);
  const int warps = M * (Hq + 2 * Hkv);
  // one "sequence" of M rows: row m's position comes from positions[m], its K/V row from out_loc[m]
  tsds_launch(qk_norm_rope_kv_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream,
      (const bf16*)qkv, (const bf16*)q_norm_w, (const bf16*)k_norm_w, (const bf16*)cos, (const bf16*)sin, positions,
      (const int32_t*)nullptr, (bf16*)q_out, (bf16*)k_pool, (bf16*)v_pool, M, M, Hq, Hkv, 1, rope_len, eps, out_loc,
      pool_rows, status);
  return tsds_launch_status();
}

// Pooled KV: the pool rows of the new tokens, out_loc[b*T + t] =
// table[req(b) * table_ld + starts[b] + t] (what SGLang hands a forward as
// out_cache_loc), for engines that own their token table.
__global__ void table_rows_kernel(const int32_t* __restrict__ table, int64_t table_ld,
                                  const int64_t* __restrict__ req_rows, const int32_t* __restrict__ starts, int B,
                                  int T, int64_t* __restrict__ out_loc) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int b = i / T, t = i - b * T;
  const int64_t p = (int64_t)starts[b] + t;
  const int64_t req = req_rows ? req_rows[b] : b;
  out_loc[i] = p < table_ld ? (int64_t)table[req * table_ld + p] : -1;
}

extern "C" int tsds_table_rows(const int32_t* table, int64_t table_ld, const int64_t* req_rows,
                               const int32_t* starts, int B, int T, int64_t* out_loc, tsds_stream_t stream) {
  TSDS_RETURN_IF(!table || table_ld <= 0 || !starts || !out_loc || B <= 0 || T <= 0, TSDS_E_INVALID);
  const int n = B * T;
  tsds_launch(table_rows_kernel, dim3((n + 127) / 128), dim3(128), 0, stream, table, table_ld, req_rows, starts, B, T,
              out_loc);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// Greedy acceptance + commit (one thread per sequence).
// ---------------------------------------------------------------------------
__global__ void accept_greedy_kernel(const int64_t* __restrict__ draft, const int64_t* __restrict__ target,
                                     int32_t* __restrict__ accept_len, int64_t* __restrict__ tokens,
                                     int32_t* __restrict__ target_len, int64_t* __restrict__ last,
                                     int64_t* __restrict__ cur, int B, int K) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t* d = draft + (int64_t)b * K;
  const int64_t* y = target + (int64_t)b * (K + 1);
  int n = 0;
  while (n < K && d[n] == y[n]) ++n;
  for (int i = 0; i <= K; ++i) tokens[(int64_t)b * (K + 1) + i] = i <= n ? y[i] : -1;
  accept_len[b] = n;
  const int64_t c = cur[b];
  last[b] = n == 0 ? c : d[n - 1];
  cur[b] = y[n];
  target_len[b] += n + 1;
}

extern "C" int tsds_accept_greedy(const int64_t* draft, const int64_t* target, int32_t* accept_len, int64_t* tokens,
                                  int32_t* target_len, int64_t* last, int64_t* cur, int B, int K,
                                  tsds_stream_t stream) {
  TSDS_RETURN_IF(B <= 0 || K < 0, TSDS_E_INVALID);
  tsds_launch(accept_greedy_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, draft, target, accept_len, tokens,
              target_len, last, cur, B, K);
  return tsds_launch_status();
}

__global__ void gather_ids_kernel(const int64_t* __restrict__ cur, const int64_t* __restrict__ last,
                                  const int64_t* __restrict__ draft, int64_t* __restrict__ verify_ids,
                                  int64_t* __restrict__ draft_ids2, int B, int K) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (verify_ids) {
    verify_ids[(int64_t)b * (K + 1)] = cur[b];
    for (int i = 0; i < K; ++i) verify_ids[(int64_t)b * (K + 1) + 1 + i] = draft[(int64_t)b * K + i];
  }
  if (draft_ids2) {
    draft_ids2[2 * b] = last[b];
    draft_ids2[2 * b + 1] = cur[b];
  }
}

extern "C" int tsds_gather_ids(const int64_t* cur, const int64_t* last, const int64_t* draft, int64_t* verify_ids,
                               int64_t* draft_ids2, int B, int K, tsds_stream_t stream) {
  TSDS_RETURN_IF(B <= 0 || K < 0 || !cur, TSDS_E_INVALID);
  TSDS_RETURN_IF(verify_ids && !draft && K > 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(draft_ids2 && !last, TSDS_E_INVALID);
  tsds_launch(gather_ids_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, cur, last, draft, verify_ids, draft_ids2, B,
              K);
  return tsds_launch_status();
}
