// Tree speculative decoding kernels: draft-tree construction from the EAGLE
// head's logits, acceptance on the verified tree (rejection sampling at
// temperature 1 with caller-supplied uniforms, or greedy), KV compaction.
//
// The semantics are the oracle's (oracle/eagle.py), written down there
// because the reference delegates all of this to SGLang.  Candidate
// bookkeeping is per sequence and tiny (<= 72 candidates), so it runs in one
// thread per sequence; the vocabulary-wide work (top-k, softmax, residual
// distributions, inverse-CDF draws) runs on whole CTAs.
#include "common.cuh"

using namespace tsds;

namespace {

constexpr int MAXC = 72;        // candidates per sequence: 1 + 4 + 16 * 4 (+ slack)
constexpr int MAXK = 8;         // top-k bound
constexpr int MAXROWS = 32;     // head cache rows per sequence

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// ---------------------------------------------------------------------------
// top-k (value desc, index asc) and log-sum-exp of each logits row
// ---------------------------------------------------------------------------
template <int K>
__device__ __forceinline__ void insert_topk(float (&v)[K], int (&ix)[K], float x, int i) {
  if (!better(x, i, v[K - 1], ix[K - 1])) return;
  int p = K - 1;
  while (p > 0 && better(x, i, v[p - 1], ix[p - 1])) {
    v[p] = v[p - 1];
    ix[p] = ix[p - 1];
    --p;
  }
  v[p] = x;
  ix[p] = i;
}

template <int K>
__global__ void __launch_bounds__(512) topk_lse_kernel(const bf16* __restrict__ logits, int ld, int V,
                                                       float* __restrict__ vals, int* __restrict__ idx,
                                                       float* __restrict__ lse) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_v[16][K];
  __shared__ int s_i[16][K];
  __shared__ float s_m[16], s_s[16];
  const bf16* row = logits + (int64_t)blockIdx.x * ld;
  float tv[K];
  int ti[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    tv[k] = -INFINITY;
    ti[k] = 0x7fffffff;
  }
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = bf2f(row[i]);
    insert_topk<K>(tv, ti, x, i);
    if (x > m) {
      s = s * expf(m - x) + 1.f;
      m = x;
    } else {
      s += expf(x - m);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // log-sum-exp across the warp, then across warps
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + (om == -INFINITY ? 0.f : os * expf(om - nm));
    m = nm;
  }
  // top-k across the warp: K rounds of "best head wins, its owner pops"
  float wv[K];
  int wi[K];
  int head = 0;
  for (int k = 0; k < K; ++k) {
    float bv = head < K ? tv[head] : -INFINITY;
    int bi = head < K ? ti[head] : 0x7fffffff;
    int owner = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int oo = __shfl_xor_sync(0xffffffffu, owner, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
        owner = oo;
      }
    }
    wv[k] = bv;
    wi[k] = bi;
    if (owner == lane) ++head;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = s;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      s_v[warp][k] = wv[k];
      s_i[warp][k] = wi[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = blockDim.x >> 5;
    float M = -INFINITY, S = 0.f;
    for (int w = 0; w < nw; ++w) {
      const float nm = fmaxf(M, s_m[w]);
      S = (M == -INFINITY ? 0.f : S * expf(M - nm)) + (s_m[w] == -INFINITY ? 0.f : s_s[w] * expf(s_m[w] - nm));
      M = nm;
    }
    lse[blockIdx.x] = M + logf(S);
    int hp[16];
    for (int w = 0; w < nw; ++w) hp[w] = 0;
    for (int k = 0; k < K; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff, bw = 0;
      for (int w = 0; w < nw; ++w)
        if (hp[w] < K && better(s_v[w][hp[w]], s_i[w][hp[w]], bv, bi)) {
          bv = s_v[w][hp[w]];
          bi = s_i[w][hp[w]];
          bw = w;
        }
      ++hp[bw];
      vals[(int64_t)blockIdx.x * K + k] = bv;
      idx[(int64_t)blockIdx.x * K + k] = bi;
    }
  }
}

// ---------------------------------------------------------------------------
// tree state (one per sequence, in global memory)
// ---------------------------------------------------------------------------
struct TreeState {
  int n_cand, n_frontier, n_rows;
  int frontier[MAXK];
  long long tok[MAXC];
  int parent[MAXC], depth[MAXC], rank[MAXC], hrow[MAXC], featrow[MAXC], lrow[MAXC];
  float score[MAXC];
  unsigned rowmask[MAXROWS];
};

struct PassIO {  // inputs of the next head pass, [B * topk] each
  long long* tok;
  int* featrow;
  int* pos;
  unsigned* mask;
  int* starts;  // [B]: first head-cache row of the pass
};

__device__ void write_pass(TreeState& st, const PassIO& io, int b, int Tn, int L) {
  for (int t = 0; t < Tn; ++t) {
    const int c = st.frontier[t];
    const int lr = st.n_rows + t;
    unsigned m = 1u << lr;
    if (st.parent[c] >= 0) m |= st.rowmask[st.lrow[st.parent[c]]];
    st.lrow[c] = lr;
    st.rowmask[lr] = m;
    io.tok[b * Tn + t] = st.tok[c];
    io.featrow[b * Tn + t] = st.featrow[c];
    io.pos[b * Tn + t] = L + st.depth[c];
    io.mask[b * Tn + t] = m;
  }
  io.starts[b] = st.n_rows;
}

__global__ void tree_init_kernel(TreeState* __restrict__ states, const long long* __restrict__ cur,
                                 const int* __restrict__ lengths, PassIO io, int B) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  TreeState& st = states[b];
  st.n_cand = 1;
  st.n_rows = 0;
  st.tok[0] = cur[b];
  st.parent[0] = -1;
  st.depth[0] = 0;
  st.rank[0] = 0;
  st.hrow[0] = -1;
  st.featrow[0] = -1;
  st.score[0] = 0.f;
  st.frontier[0] = 0;
  st.n_frontier = 1;
  write_pass(st, io, b, 1, lengths[b]);
}

// After a head pass over T frontier nodes per sequence (rows row_base + b*T + t):
// add their top-k children as candidates and choose the next frontier.
__global__ void tree_step_kernel(TreeState* __restrict__ states, const float* __restrict__ vals,
                                 const int* __restrict__ idx, const float* __restrict__ lse, int row_base, int T,
                                 int k, int next_T, const int* __restrict__ lengths, PassIO io, int B) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  TreeState& st = states[b];
  const int first_new = st.n_cand;
  for (int t = 0; t < T; ++t) {
    const int c = st.frontier[t];
    const int hr = row_base + b * T + t;
    st.hrow[c] = hr;
    for (int r = 0; r < k && st.n_cand < MAXC; ++r) {
      const int n = st.n_cand++;
      st.tok[n] = idx[(int64_t)hr * k + r];
      st.parent[n] = c;
      st.depth[n] = st.depth[c] + 1;
      st.rank[n] = r;
      st.hrow[n] = -1;
      st.featrow[n] = hr;
      st.lrow[n] = -1;
      st.score[n] = st.score[c] + (vals[(int64_t)hr * k + r] - lse[hr]);
    }
  }
  st.n_rows += T;
  if (next_T <= 0) return;
  // next frontier: the next_T best new candidates (score desc, creation asc), kept in creation order
  int chosen[MAXK];
  int nch = 0;
  for (int sel = 0; sel < next_T; ++sel) {
    int best = -1;
    for (int n = first_new; n < st.n_cand; ++n) {
      bool used = false;
      for (int q = 0; q < nch; ++q) used |= chosen[q] == n;
      if (used) continue;
      if (best < 0 || st.score[n] > st.score[best]) best = n;
    }
    chosen[nch++] = best;
  }
  for (int i = 1; i < nch; ++i)
    for (int j = i; j > 0 && chosen[j] < chosen[j - 1]; --j) {
      const int tmp = chosen[j];
      chosen[j] = chosen[j - 1];
      chosen[j - 1] = tmp;
    }
  for (int i = 0; i < nch; ++i) st.frontier[i] = chosen[i];
  st.n_frontier = nch;
  write_pass(st, io, b, next_T, lengths[b]);
}

struct VerifyIO {
  long long* ids;    // [B][NN]
  int* pos;          // [B][NN]  positions L + depth
  unsigned* mask;    // [B][NN]  ancestor-or-self bits over node indices
  int* hrow;         // [B][NN]  head row of the node's children distribution (-1)
  int* children;     // [B][NN][k] child node indices in draft-rank order (-1)
  int* starts;       // [B]      = lengths (target verify)
};

// Keep the n_nodes best candidates (score desc, depth asc, creation asc) plus
// the root; emit them in creation order (parents first).
__global__ void tree_finalize_kernel(const TreeState* __restrict__ states, int n_nodes, int k,
                                     const int* __restrict__ lengths, VerifyIO io, int B) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const TreeState& st = states[b];
  const int NN = n_nodes + 1;
  bool keep[MAXC];
  for (int n = 0; n < st.n_cand; ++n) keep[n] = n == 0;
  for (int sel = 0; sel < n_nodes && sel < st.n_cand - 1; ++sel) {
    int best = -1;
    for (int n = 1; n < st.n_cand; ++n) {
      if (keep[n]) continue;
      if (best < 0 || st.score[n] > st.score[best] ||
          (st.score[n] == st.score[best] && st.depth[n] < st.depth[best]))
        best = n;
    }
    keep[best] = true;
  }
  int pos_of[MAXC];
  int j = 0;
  for (int n = 0; n < st.n_cand; ++n) pos_of[n] = keep[n] ? j++ : -1;
  const int L = lengths[b];
  unsigned masks[MAXC];
  for (int n = 0; n < st.n_cand; ++n) {
    if (!keep[n]) continue;
    const int v = pos_of[n];
    const int p = st.parent[n];
    masks[v] = (1u << v) | (p >= 0 && pos_of[p] >= 0 ? masks[pos_of[p]] : 0u);
    io.ids[b * NN + v] = st.tok[n];
    io.pos[b * NN + v] = L + st.depth[n];
    io.mask[b * NN + v] = masks[v];
    io.hrow[b * NN + v] = st.hrow[n];
    for (int r = 0; r < k; ++r) io.children[(b * NN + v) * k + r] = -1;
  }
  for (int v = j; v < NN; ++v) {  // fewer candidates than nodes: pad with masked-out copies of the root
    io.ids[b * NN + v] = st.tok[0];
    io.pos[b * NN + v] = L;
    io.mask[b * NN + v] = 1u << v;
    io.hrow[b * NN + v] = -1;
    for (int r = 0; r < k; ++r) io.children[(b * NN + v) * k + r] = -1;
  }
  for (int n = 1; n < st.n_cand; ++n) {
    if (!keep[n]) continue;
    const int pv = pos_of[st.parent[n]];
    if (pv >= 0) io.children[(b * NN + pv) * k + st.rank[n]] = pos_of[n];
  }
  // compact each children list (ranks of kept children, in rank order)
  for (int v = 0; v < j; ++v) {
    int w = 0;
    for (int r = 0; r < k; ++r) {
      const int c = io.children[(b * NN + v) * k + r];
      if (c >= 0) io.children[(b * NN + v) * k + w++] = c;
    }
    for (; w < k; ++w) io.children[(b * NN + v) * k + w] = -1;
  }
  io.starts[b] = L;
}

// ---------------------------------------------------------------------------
// acceptance on the verified tree
// ---------------------------------------------------------------------------
__device__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

__device__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
  return t;
}

// dst = softmax(row) over V (fp32), returns nothing; all threads participate
__device__ void softmax_row(const bf16* __restrict__ row, float* __restrict__ dst, int V, float* red) {
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, bf2f(row[i]));
  m = block_reduce_max(m, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float e = expf(bf2f(row[i]) - m);
    dst[i] = e;
    s += e;
  }
  s = block_reduce_sum(s, red);
  const float inv = 1.0f / s;
  for (int i = threadIdx.x; i < V; i += blockDim.x) dst[i] *= inv;
  __syncthreads();
}

// First index whose inclusive prefix sum exceeds u * total (contiguous chunks per thread).
__device__ int inverse_cdf(const float* __restrict__ p, int V, float u, float* red, int* s_idx) {
  const int nt = blockDim.x;
  const int chunk = (V + nt - 1) / nt;
  const int lo = threadIdx.x * chunk, hi = min(V, lo + chunk);
  float part = 0.f;
  for (int i = lo; i < hi; ++i) part += p[i];
  // inclusive scan of the per-thread parts (thread order = index order)
  __shared__ float s_part[1024];
  s_part[threadIdx.x] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float run = 0.f;
    for (int t = 0; t < nt; ++t) {
      run += s_part[t];
      s_part[t] = run;
    }
    *s_idx = -1;
  }
  __syncthreads();
  const float total = s_part[nt - 1];
  const float thr = u * total;
  const float before = threadIdx.x == 0 ? 0.f : s_part[threadIdx.x - 1];
  if (before <= thr && s_part[threadIdx.x] > thr) {
    float run = before;
    int pick = hi - 1;
    for (int i = lo; i < hi; ++i) {
      run += p[i];
      if (run > thr) {
        pick = i;
        break;
      }
    }
    *s_idx = pick;
  }
  __syncthreads();
  int r = *s_idx;
  if (r < 0) {  // rounding left thr at or above the total: the last index with mass
    if (threadIdx.x == 0) {
      int i = V - 1;
      while (i > 0 && p[i] == 0.f) --i;
      *s_idx = i;
    }
    __syncthreads();
    r = *s_idx;
  }
  __syncthreads();
  return r;
}

struct AcceptIO {
  const bf16* target_logits;   // [B*NN][V]
  const long long* target_argmax;  // [B*NN]
  const bf16* head_logits;     // [rows][V]
  const long long* ids;        // [B][NN]
  const int* hrow;             // [B][NN]
  const int* children;         // [B][NN][k]
  const float* U;              // [B][depth+1][k+1] (NULL: greedy)
  float* scratch;              // [B][2][V]
  int* path;                   // [B][depth+1] node indices (-1 pad)
  int* accept_len;             // [B]
  long long* tokens;           // [B][depth+2]: accepted tokens then the bonus (-1 pad)
  long long* cur;              // [B] <- bonus
  int NN, V, k, depth;
};

__global__ void __launch_bounds__(1024) accept_tree_kernel(AcceptIO io) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int s_idx, s_next, s_done;
  __shared__ float s_px, s_qx;
  const int b = blockIdx.x;
  const int NN = io.NN, V = io.V, k = io.k;
  float* P = io.scratch + (size_t)b * 2 * V;
  float* Q = P + V;
  int node = 0, d = 0, bonus = 0;
  for (;;) {
    const int* kids = io.children + ((size_t)b * NN + node) * k;
    if (io.U == nullptr) {  // greedy
      if (threadIdx.x == 0) {
        const long long y = io.target_argmax[(size_t)b * NN + node];
        s_next = -1;
        for (int i = 0; i < k && kids[i] >= 0; ++i)
          if (io.ids[(size_t)b * NN + kids[i]] == y) {
            s_next = kids[i];
            break;
          }
        s_idx = (int)y;
      }
      __syncthreads();
      const int nxt = s_next;
      bonus = s_idx;
      __syncthreads();
      if (nxt < 0) break;
      if (threadIdx.x == 0) io.path[b * (io.depth + 1) + d] = nxt;
      node = nxt;
      ++d;
      continue;
    }
    const float* u = io.U + ((size_t)b * (io.depth + 1) + d) * (k + 1);
    softmax_row(io.target_logits + ((size_t)b * NN + node) * V, P, V, red);
    const bool has_kids = kids[0] >= 0;
    if (has_kids) softmax_row(io.head_logits + (size_t)io.hrow[(size_t)b * NN + node] * V, Q, V, red);
    int nxt = -1;
    for (int i = 0; i < k && has_kids && kids[i] >= 0; ++i) {
      const int c = kids[i];
      const int x = (int)io.ids[(size_t)b * NN + c];
      if (threadIdx.x == 0) {
        s_px = P[x];
        s_qx = Q[x];
      }
      __syncthreads();
      const bool acc = u[i] * s_qx < s_px;
      __syncthreads();
      if (acc) {
        nxt = c;
        break;
      }
      // residual p <- norm(max(p - q, 0)); q <- q without x, renormalised
      float sp = 0.f, sq = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float r = fmaxf(P[j] - Q[j], 0.f);
        P[j] = r;
        sp += r;
        if (j == x) Q[j] = 0.f;
        sq += Q[j];
      }
      sp = block_reduce_sum(sp, red);
      sq = block_reduce_sum(sq, red);
      const float ip = sp > 0.f ? 1.0f / sp : 0.f, iq = sq > 0.f ? 1.0f / sq : 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        P[j] *= ip;
        Q[j] *= iq;
      }
      __syncthreads();
    }
    if (nxt < 0) {
      bonus = inverse_cdf(P, V, u[k], red, &s_idx);
      break;
    }
    if (threadIdx.x == 0) io.path[b * (io.depth + 1) + d] = nxt;
    node = nxt;
    ++d;
  }
  if (threadIdx.x == 0) {
    for (int i = d; i < io.depth + 1; ++i) io.path[b * (io.depth + 1) + i] = -1;
    io.accept_len[b] = d;
    long long* tk = io.tokens + (size_t)b * (io.depth + 2);
    for (int i = 0; i < io.depth + 2; ++i) tk[i] = -1;
    for (int i = 0; i < d; ++i) tk[i] = io.ids[(size_t)b * NN + io.path[b * (io.depth + 1) + i]];
    tk[d] = bonus;
    io.cur[b] = bonus;
  }
}

// KV compaction: rows L + path[j] -> L + 1 + j of every layer; the blocks of
// layer index == layers copy the next root feature (hidden state of the last
// accepted node).
__global__ void tree_compact_kernel(bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int layers, int B,
                                    int Hkv, int S, const int* __restrict__ lengths, const int* __restrict__ path,
                                    const int* __restrict__ accept_len, int depth, const bf16* __restrict__ hidden,
                                    int NN, int N, bf16* __restrict__ root_feat) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 128;
  const int b = blockIdx.x, layer = blockIdx.y;
  const int a = accept_len[b];
  const int L = lengths[b];
  if (layer == layers) {
    const int last = a > 0 ? path[b * (depth + 1) + a - 1] : 0;
    const bf16* src = hidden + ((size_t)b * NN + last) * N;
    for (int i = threadIdx.x; i < N / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(root_feat + (size_t)b * N)[i] = reinterpret_cast<const uint4*>(src)[i];
    return;
  }
  // each thread moves 16 bytes; rows are 256 bytes (D = 128 bf16)
  for (int j = 0; j < a; ++j) {
    const int from = L + path[b * (depth + 1) + j], to = L + 1 + j;
    if (from == to || from >= S || to >= S) continue;
    for (int w = threadIdx.x; w < Hkv * 2 * (D / 8); w += blockDim.x) {
      const int h = w / (2 * (D / 8)), rest = w % (2 * (D / 8));
      bf16* base = rest < D / 8 ? k_cache : v_cache;
      const int c = rest % (D / 8);
      const size_t slab = (((size_t)layer * B + b) * Hkv + h) * S;
      uint4* dst = reinterpret_cast<uint4*>(base + (slab + to) * D) + c;
      const uint4* srcp = reinterpret_cast<const uint4*>(base + (slab + from) * D) + c;
      *dst = *srcp;
    }
    __syncthreads();  // later moves never read an earlier destination, but keep rows ordered
  }
}

__global__ void tree_advance_kernel(int* __restrict__ lengths, const int* __restrict__ accept_len, int B) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lengths[b] += accept_len[b] + 1;
}

}  // namespace

extern "C" size_t tsds_tree_state_bytes(int B) { return (size_t)B * sizeof(TreeState); }

extern "C" int tsds_logits_topk(const void* logits, int ld, int M, int V, int k, float* vals, int32_t* idx,
                                float* lse, tsds_stream_t stream) {
  TSDS_RETURN_IF(!logits || !vals || !idx || !lse || M <= 0 || V <= 0 || ld < V, TSDS_E_INVALID);
  switch (k) {
    case 1: tsds_launch(topk_lse_kernel<1>, dim3(M), dim3(512), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 2: tsds_launch(topk_lse_kernel<2>, dim3(M), dim3(512), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 4: tsds_launch(topk_lse_kernel<4>, dim3(M), dim3(512), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 8: tsds_launch(topk_lse_kernel<8>, dim3(M), dim3(512), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    default: return TSDS_E_UNSUPPORTED;
  }
  return tsds_launch_status();
}

extern "C" int tsds_tree_init(void* states, const int64_t* cur, const int32_t* lengths, int64_t* pass_tok,
                              int32_t* pass_featrow, int32_t* pass_pos, uint32_t* pass_mask, int32_t* pass_starts,
                              int B, tsds_stream_t stream) {
  TSDS_RETURN_IF(!states || !cur || !lengths || B <= 0, TSDS_E_INVALID);
  PassIO io{(long long*)pass_tok, pass_featrow, pass_pos, (unsigned*)pass_mask, pass_starts};
  tsds_launch(tree_init_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, (TreeState*)states, (const long long*)cur,
              (const int*)lengths, io, B);
  return tsds_launch_status();
}

extern "C" int tsds_tree_step(void* states, const float* vals, const int32_t* idx, const float* lse, int row_base,
                              int T, int k, int next_T, const int32_t* lengths, int64_t* pass_tok,
                              int32_t* pass_featrow, int32_t* pass_pos, uint32_t* pass_mask, int32_t* pass_starts,
                              int B, tsds_stream_t stream) {
  TSDS_RETURN_IF(!states || B <= 0 || T <= 0 || k <= 0 || k > MAXK || next_T > MAXK, TSDS_E_INVALID);
  PassIO io{(long long*)pass_tok, pass_featrow, pass_pos, (unsigned*)pass_mask, pass_starts};
  tsds_launch(tree_step_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, (TreeState*)states, vals, (const int*)idx,
              lse, row_base, T, k, next_T, (const int*)lengths, io, B);
  return tsds_launch_status();
}

extern "C" int tsds_tree_finalize(const void* states, int n_nodes, int k, const int32_t* lengths, int64_t* ids,
                                  int32_t* positions, uint32_t* masks, int32_t* hrow, int32_t* children,
                                  int32_t* starts, int B, tsds_stream_t stream) {
  TSDS_RETURN_IF(!states || n_nodes < 1 || n_nodes + 1 > 32 || k < 1 || k > MAXK || B <= 0, TSDS_E_INVALID);
  VerifyIO io{(long long*)ids, positions, (unsigned*)masks, hrow, children, starts};
  tsds_launch(tree_finalize_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, (const TreeState*)states, n_nodes, k,
              (const int*)lengths, io, B);
  return tsds_launch_status();
}

extern "C" int tsds_accept_tree(const void* target_logits, const int64_t* target_argmax, const void* head_logits,
                                const int64_t* ids, const int32_t* hrow, const int32_t* children, const float* U,
                                float* scratch, int32_t* path, int32_t* accept_len, int64_t* tokens, int64_t* cur,
                                int B, int n_nodes, int V, int k, int depth, tsds_stream_t stream) {
  TSDS_RETURN_IF(B <= 0 || n_nodes < 1 || V <= 0 || k < 1 || k > MAXK || depth < 1, TSDS_E_INVALID);
  TSDS_RETURN_IF(U != nullptr && (!target_logits || !head_logits || !scratch), TSDS_E_INVALID);
  TSDS_RETURN_IF(U == nullptr && !target_argmax, TSDS_E_INVALID);
  AcceptIO io{(const bf16*)target_logits, (const long long*)target_argmax, (const bf16*)head_logits,
              (const long long*)ids, hrow, children, U, scratch, path, accept_len, (long long*)tokens,
              (long long*)cur, n_nodes + 1, V, k, depth};
  tsds_launch(accept_tree_kernel, dim3(B), dim3(1024), 0, stream, io);
  return tsds_launch_status();
}

extern "C" int tsds_tree_commit(void* k_cache, void* v_cache, int layers, int B, int Hkv, int S, int D,
                                int32_t* lengths, const int32_t* path, const int32_t* accept_len, int depth,
                                const void* hidden, int n_nodes, int N, void* root_feat, tsds_stream_t stream) {
  TSDS_RETURN_IF(D != 128, TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF(!k_cache || !v_cache || !lengths || !path || !accept_len || !hidden || !root_feat || layers <= 0 ||
                     B <= 0 || (N % 8) != 0,
                 TSDS_E_INVALID);
  tsds_launch(tree_compact_kernel, dim3(B, layers + 1), dim3(256), 0, stream, (bf16*)k_cache, (bf16*)v_cache, layers,
              B, Hkv, S, (const int*)lengths, (const int*)path, (const int*)accept_len, depth, (const bf16*)hidden,
              n_nodes + 1, N, (bf16*)root_feat);
  int st = tsds_launch_status();
  if (st != TSDS_OK) return st;
  tsds_launch(tree_advance_kernel, dim3((B + 63) / 64), dim3(64), 0, stream, (int*)lengths, (const int*)accept_len, B);
  return tsds_launch_status();
}

// X2[m] = [feature | embedding(token)] for the head's pass rows m = b*T + t.
__global__ void eagle_inputs_kernel(const bf16* __restrict__ root_feat, const bf16* __restrict__ head_feat,
                                    const int* __restrict__ featrow, const long long* __restrict__ tok,
                                    const bf16* __restrict__ embed, bf16* __restrict__ out, int T, int N, int vocab) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, b = m / T;
  const int fr = featrow[m];
  const bf16* f = fr < 0 ? root_feat + (size_t)b * N : head_feat + (size_t)fr * N;
  const long long id = tok[m];
  const bool ok = id >= 0 && id < vocab;
  const bf16* e = embed + (size_t)(ok ? id : 0) * N;
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)m * 2 * N);
  for (int c = threadIdx.x; c < N / 8; c += blockDim.x) {
    dst[c] = reinterpret_cast<const uint4*>(f)[c];
    dst[N / 8 + c] = ok ? reinterpret_cast<const uint4*>(e)[c] : make_uint4(0, 0, 0, 0);
  }
}

extern "C" int tsds_eagle_inputs(const void* root_feat, const void* head_feat, const int32_t* featrow,
                                 const int64_t* tok, const void* embed, void* out, int B, int T, int N, int vocab,
                                 tsds_stream_t stream) {
  TSDS_RETURN_IF(!root_feat || !featrow || !tok || !embed || !out || B <= 0 || T <= 0 || (N % 8), TSDS_E_INVALID);
  tsds_launch(eagle_inputs_kernel, dim3(B * T), dim3(128), 0, stream, (const bf16*)root_feat, (const bf16*)head_feat,
              (const int*)featrow, (const long long*)tok, (const bf16*)embed, (bf16*)out, T, N, vocab);
  return tsds_launch_status();
}
