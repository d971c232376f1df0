// Tree speculative decoding kernels: draft-tree construction from the EAGLE
// head's logits, acceptance on the verified tree (rejection sampling at
// temperature 1 with caller-supplied uniforms, or greedy), KV compaction.
//
// The semantics are the oracle's (oracle/eagle.py), written down there
// because the reference delegates all of this to SGLang.  Candidate
// bookkeeping is per sequence and tiny (<= 72 candidates), so it runs in one
// thread per sequence; the vocabulary-wide work (top-k, softmax, residual
// distributions, inverse-CDF draws) runs on whole CTAs.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

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
  // insertion with static register indices (no local-memory array)
#pragma unroll
  for (int p = K - 1; p >= 0; --p) {
    if (p > 0 && better(x, i, v[p - 1], ix[p - 1])) {
      v[p] = v[p - 1];
      ix[p] = ix[p - 1];
    } else {
      v[p] = x;
      ix[p] = i;
      break;
    }
  }
}

// online log-sum-exp state (m, s): sum = s * exp(m)
__device__ __forceinline__ void lse_merge(float& m, float& s, float om, float os) {
  const float nm = fmaxf(m, om);
  if (nm == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
  m = nm;
}

constexpr int TOPK_THREADS = 512;
constexpr int TOPK_WARPS = TOPK_THREADS / 32;
constexpr int TOPK_UNROLL = 8;   // 16-byte loads in flight per thread

template <int K>
__device__ __forceinline__ void topk_take8(float (&tv)[K], int (&ti)[K], float& m, float& s, uint4 q, int i0) {
  const bf16* e = reinterpret_cast<const bf16*>(&q);
  float x[8];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    x[j] = bf2f(e[j]);
    if (x[j] != x[j]) x[j] = -INFINITY;  // NaN ranks last: every emitted index is a real token
    mx = fmaxf(mx, x[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) insert_topk<K>(tv, ti, x[j], i0 + j);
  if (mx == -INFINITY) return;
  float t = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) t += __expf(x[j] - mx);
  lse_merge(m, s, mx, t);
}

constexpr int TOPK_CL = 8;   // CTAs per row (one cluster)

// One cluster of TOPK_CL CTAs per row (grid (TOPK_CL, rows)); CTA rank c
// reads the vocabulary slice [c*vs, (c+1)*vs) as 16-byte vectors when the
// row is aligned, TOPK_UNROLL of them in flight per thread.  Rank 0 merges
// the ranks' lists and log-sum-exps from distributed shared memory.  All
// reductions run in a fixed order, so the result is deterministic.
template <int K>
__global__ void __cluster_dims__(TOPK_CL, 1, 1) __launch_bounds__(TOPK_THREADS, 1)
    topk_lse_kernel(const bf16* __restrict__ logits, int ld, int V, float* __restrict__ vals,
                    int* __restrict__ idx, float* __restrict__ lse) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cl = cg::this_cluster();
  __shared__ float s_v[TOPK_WARPS][K];
  __shared__ int s_i[TOPK_WARPS][K];
  __shared__ float s_m[TOPK_WARPS], s_s[TOPK_WARPS];
  __shared__ float c_v[K];   // this CTA's result, read by rank 0
  __shared__ int c_i[K];
  __shared__ float c_ms[2];
  const int rank = blockIdx.x, rowi = blockIdx.y;
  const int vs = ((V + TOPK_CL - 1) / TOPK_CL + 7) / 8 * 8;
  const int v0 = min(V, rank * vs), v1 = min(V, v0 + vs);
  const bf16* row = logits + (int64_t)rowi * ld;
  float tv[K];
  int ti[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    tv[k] = -INFINITY;
    ti[k] = 0x7fffffff;
  }
  float m = -INFINITY, s = 0.f;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  const int nvec = vec ? (v1 - v0) / 8 : 0;
  const uint4* rv = reinterpret_cast<const uint4*>(row + v0);
  for (int base = threadIdx.x; base < nvec; base += TOPK_UNROLL * TOPK_THREADS) {
    uint4 q[TOPK_UNROLL];
#pragma unroll
    for (int u = 0; u < TOPK_UNROLL; ++u) {
      const int i = base + u * TOPK_THREADS;
      if (i < nvec) q[u] = __ldg(rv + i);
    }
#pragma unroll
    for (int u = 0; u < TOPK_UNROLL; ++u) {
      const int i = base + u * TOPK_THREADS;
      if (i < nvec) topk_take8<K>(tv, ti, m, s, q[u], v0 + 8 * i);
    }
  }
  for (int i = v0 + nvec * 8 + threadIdx.x; i < v1; i += TOPK_THREADS) {
    float x = bf2f(row[i]);
    if (x != x) x = -INFINITY;
    insert_topk<K>(tv, ti, x, i);
    lse_merge(m, s, x, 1.f);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, om, os);
  }
  // top-k across the warp: K rounds of "best head wins, its owner pops"
  int head = 0;
  for (int k = 0; k < K; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (j == head) {
        bv = tv[j];
        bi = ti[j];
      }
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
    if (lane == 0) {
      s_v[warp][k] = bv;
      s_i[warp][k] = bi;
    }
    if (owner == lane) ++head;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    // lse over the warps (fixed order: the shuffle tree)
    float wm = lane < TOPK_WARPS ? s_m[lane] : -INFINITY, ws = lane < TOPK_WARPS ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, wm, o), os = __shfl_xor_sync(0xffffffffu, ws, o);
      lse_merge(wm, ws, om, os);
    }
    if (lane == 0) {
      c_ms[0] = wm;
      c_ms[1] = ws;
    }
    // top-k over the warps' lists: lane w holds warp w's list
    int hp = lane < TOPK_WARPS ? 0 : K;
    for (int k = 0; k < K; ++k) {
      float bv = hp < K ? s_v[lane][hp] : -INFINITY;
      int bi = hp < K ? s_i[lane][hp] : 0x7fffffff;
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
      if (owner == lane) ++hp;
      if (lane == 0) {
        c_v[k] = bv;
        c_i[k] = bi;
      }
    }
  }
  cl.sync();
  if (rank == 0 && warp == 0) {
    // lane q < TOPK_CL holds rank q's list and log-sum-exp
    const float* rv_ = lane < TOPK_CL ? cl.map_shared_rank(c_v, lane) : nullptr;
    const int* ri_ = lane < TOPK_CL ? cl.map_shared_rank(c_i, lane) : nullptr;
    const float* rms = lane < TOPK_CL ? cl.map_shared_rank(c_ms, lane) : nullptr;
    float wm = rms ? rms[0] : -INFINITY, ws = rms ? rms[1] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, wm, o), os = __shfl_xor_sync(0xffffffffu, ws, o);
      lse_merge(wm, ws, om, os);
    }
    if (lane == 0) lse[rowi] = wm + logf(ws);
    int hp = lane < TOPK_CL ? 0 : K;
    for (int k = 0; k < K; ++k) {
      float bv = hp < K ? rv_[hp] : -INFINITY;
      int bi = hp < K ? ri_[hp] : 0x7fffffff;
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
      if (owner == lane) ++hp;
      if (lane == 0) {
        vals[(int64_t)rowi * K + k] = bv;
        idx[(int64_t)rowi * K + k] = bi;
      }
    }
  }
  cl.sync();  // the other ranks' shared memory stays valid until rank 0 is done
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
  pdl_trigger();
  pdl_wait();
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
// The state is copied to shared memory by the CTA and back afterwards: the
// serial bookkeeping then runs on shared-memory latency.
constexpr int STATE_THREADS = 64;
constexpr int STATE_WORDS = (int)(sizeof(TreeState) / 4);
static_assert(sizeof(TreeState) % 4 == 0, "TreeState copies as 32-bit words");

__device__ __forceinline__ void state_copy(uint32_t* dst, const uint32_t* src) {
  for (int i = threadIdx.x; i < STATE_WORDS; i += blockDim.x) dst[i] = src[i];
}

__device__ void tree_step_one(TreeState& st, const float* __restrict__ vals, const int* __restrict__ idx,
                              const float* __restrict__ lse, int row_base, int T, int k, int next_T, int L,
                              const PassIO& io, int b);

// One CTA per sequence.
__global__ void __launch_bounds__(STATE_THREADS) tree_step_kernel(TreeState* __restrict__ states,
                                                                  const float* __restrict__ vals,
                                                                  const int* __restrict__ idx,
                                                                  const float* __restrict__ lse, int row_base, int T,
                                                                  int k, int next_T, const int* __restrict__ lengths,
                                                                  PassIO io, int B) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(8) TreeState sst;
  const int b = blockIdx.x;
  state_copy(reinterpret_cast<uint32_t*>(&sst), reinterpret_cast<const uint32_t*>(&states[b]));
  __syncthreads();
  if (threadIdx.x == 0) tree_step_one(sst, vals, idx, lse, row_base, T, k, next_T, lengths[b], io, b);
  __syncthreads();
  state_copy(reinterpret_cast<uint32_t*>(&states[b]), reinterpret_cast<const uint32_t*>(&sst));
}

__device__ void tree_step_one(TreeState& st, const float* __restrict__ vals, const int* __restrict__ idx,
                              const float* __restrict__ lse, int row_base, int T, int k, int next_T, int L,
                              const PassIO& io, int b) {
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
  write_pass(st, io, b, next_T, L);
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
// the root; emit them in creation order (parents first).  One CTA per
// sequence: each thread ranks one candidate against all others, then one
// thread lays out the kept nodes from shared memory.
__global__ void __launch_bounds__(STATE_THREADS) tree_finalize_kernel(const TreeState* __restrict__ states,
                                                                      int n_nodes, int k,
                                                                      const int* __restrict__ lengths, VerifyIO io,
                                                                      int B) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(8) TreeState st;
  __shared__ bool keep[MAXC];
  __shared__ int ch[32][MAXK];
  const int b = blockIdx.x;
  state_copy(reinterpret_cast<uint32_t*>(&st), reinterpret_cast<const uint32_t*>(&states[b]));
  __syncthreads();
  const int nc = st.n_cand;
  for (int n = threadIdx.x; n < nc; n += blockDim.x) {
    if (n == 0) {
      keep[0] = true;
      continue;
    }
    // a strict total order (NaN scores rank last), so exactly
    // min(n_nodes, nc - 1) candidates are kept
    int rank = 0;
    float sn = st.score[n];
    if (sn != sn) sn = -INFINITY;
    const int dn = st.depth[n];
    for (int m = 1; m < nc; ++m) {
      float sm = st.score[m];
      if (sm != sm) sm = -INFINITY;
      const int dm = st.depth[m];
      rank += (sm > sn || (sm == sn && (dm < dn || (dm == dn && m < n)))) ? 1 : 0;
    }
    keep[n] = rank < n_nodes;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int NN = n_nodes + 1;
  int pos_of[MAXC];
  int j = 0;
  for (int n = 0; n < nc; ++n) pos_of[n] = keep[n] && j < NN ? j++ : -1;
  const int L = lengths[b];
  unsigned masks[32];
  for (int v = 0; v < NN; ++v)
    for (int r = 0; r < k; ++r) ch[v][r] = -1;
  for (int n = 0; n < nc; ++n) {
    if (pos_of[n] < 0) continue;
    const int v = pos_of[n];
    const int p = st.parent[n];
    masks[v] = (1u << v) | (p >= 0 && pos_of[p] >= 0 ? masks[pos_of[p]] : 0u);
    io.ids[b * NN + v] = st.tok[n];
    io.pos[b * NN + v] = L + st.depth[n];
    io.mask[b * NN + v] = masks[v];
    io.hrow[b * NN + v] = st.hrow[n];
    if (n > 0 && pos_of[p] >= 0) ch[pos_of[p]][st.rank[n]] = v;
  }
  for (int v = j; v < NN; ++v) {  // fewer candidates than nodes: pad with masked-out copies of the root
    io.ids[b * NN + v] = st.tok[0];
    io.pos[b * NN + v] = L;
    io.mask[b * NN + v] = 1u << v;
    io.hrow[b * NN + v] = -1;
  }
  // children lists: kept children in rank order, then -1
  for (int v = 0; v < NN; ++v) {
    int w = 0;
    for (int r = 0; r < k; ++r)
      if (ch[v][r] >= 0) io.children[(b * NN + v) * k + w++] = ch[v][r];
    for (; w < k; ++w) io.children[(b * NN + v) * k + w] = -1;
  }
  io.starts[b] = L;
}

// ---------------------------------------------------------------------------
// acceptance on the verified tree
// ---------------------------------------------------------------------------
// Rejection sampling at one node works on p = softmax(target row) and
// q = softmax(head row).  Rejecting child x_l turns (p_l, q_l) into
//   p_{l+1} = max(p_l - q_l, 0) / Z_{l+1},   Z_{l+1} = sum_j max(p_l - q_l, 0)
//   q_{l+1} = q_l without x_l, renormalised   (q_0(j) / (1 - sum_{i<=l} q_0(x_i)))
// so p_r(j) and q_r(j) follow element-wise from the two bf16 logits, the two
// log-sum-exps and the scalars Z_l: nothing of vocabulary size is stored.
// One vocabulary pass per visited node (both log-sum-exps), one per
// rejected child (its Z) and one for the bonus draw (inverse CDF).
//
// Each sequence runs on one cluster of ACC_CL CTAs; CTA rank c owns the
// vocabulary slice [c*vs, (c+1)*vs).  CTA-level partial results are
// exchanged through distributed shared memory and combined in rank order,
// so every CTA holds bit-identical scalars and takes the same decisions;
// rank 0 writes the outputs.
constexpr int ACC_CL = 8;
constexpr int ACC_THREADS = 512;
constexpr int ACC_WARPS = ACC_THREADS / 32;

struct AccNode {
  float lse_t, lse_h;
  int r;                  // children rejected so far
  int X[MAXK];            // their tokens
  float invZ[MAXK + 1];   // 1 / Z_l, l >= 1
  float invQ[MAXK + 1];   // 1 / (1 - sum_{i<l} q_0(x_i)), invQ[0] = 1
};

// rule ACC_RULE_TARGET takes the draft as deterministic: q_l is one-hot on
// the child x_l under test, so p_{l+1} = p_l without x_l, renormalised, the
// acceptance test is u < p_l(x_l), and the head logits are not read.
constexpr int ACC_RULE_DRAFT = 0, ACC_RULE_TARGET = 1;

template <int RULE>
__device__ __forceinline__ float acc_p(const AccNode& a, float tj, float hj, int j) {
  float p = expf(tj - a.lse_t);
  if (a.r == 0) return p;
  if constexpr (RULE == ACC_RULE_TARGET) {
    for (int l = 0; l < a.r; ++l) p = a.X[l] == j ? 0.f : p * a.invZ[l + 1];
    return p;
  } else {
    const float q0 = expf(hj - a.lse_h);
    bool ex = false;
    for (int l = 0; l < a.r; ++l) {
      const float ql = ex ? 0.f : q0 * a.invQ[l];
      p = fmaxf(p - ql, 0.f) * a.invZ[l + 1];
      ex |= a.X[l] == j;
    }
    return p;
  }
}

// q_r(j) while child x is under test
template <int RULE>
__device__ __forceinline__ float acc_q(const AccNode& a, float hj, int j, int x) {
  if constexpr (RULE == ACC_RULE_TARGET) {
    return j == x ? 1.f : 0.f;
  } else {
    for (int l = 0; l < a.r; ++l)
      if (a.X[l] == j) return 0.f;
    return expf(hj - a.lse_h) * a.invQ[a.r];
  }
}

// deterministic block reductions (fixed shuffle tree, then warp order)
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < ACC_WARPS ? red[lane] : 0.f;
  t = warp_sum(t);
  return __shfl_sync(0xffffffffu, t, 0);
}

__device__ void block_lse(float& m, float& s, float* red_m, float* red_s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, om, os);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  m = lane < ACC_WARPS ? red_m[lane] : -INFINITY;
  s = lane < ACC_WARPS ? red_s[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, om, os);
  }
  m = __shfl_sync(0xffffffffu, m, 0);
  s = __shfl_sync(0xffffffffu, s, 0);
}

// Cluster exchange: each CTA publishes up to 4 floats; after the barrier
// every thread reads all ranks' values.  Double-buffered by phase: a CTA
// can only rewrite a buffer after the next barrier, which every CTA reaches
// after it has finished reading it.
struct Xch {
  float v[2][4];
};

__device__ __forceinline__ float* xch_publish(Xch& x, int phase) { return x.v[phase & 1]; }

__device__ __forceinline__ const float* xch_remote(cg::cluster_group& cl, Xch& x, int phase, int rank) {
  return cl.map_shared_rank(x.v[phase & 1], rank);
}

// Visit elements j in [v0, v1) of the two rows in strided 8-wide groups
// (16-byte loads, 4 groups in flight per thread); f(j, t_j, h_j).  h may be null.
template <typename F>
__device__ __forceinline__ void for_each_strided(const bf16* t, const bf16* h, int v0, int v1, F f) {
  const bool vec = ((reinterpret_cast<uintptr_t>(t) | reinterpret_cast<uintptr_t>(h)) & 15u) == 0 && (v0 & 7) == 0;
  const int g0 = v0 / 8, ng = vec ? (v1 - v0) / 8 : 0;
  constexpr int U = 4;
  for (int base = threadIdx.x; base < ng; base += U * ACC_THREADS) {
    uint4 qt[U], qh[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * ACC_THREADS;
      if (i < ng) {
        qt[u] = __ldg(reinterpret_cast<const uint4*>(t) + g0 + i);
        qh[u] = h ? __ldg(reinterpret_cast<const uint4*>(h) + g0 + i) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * ACC_THREADS;
      if (i < ng) {
        const bf16* et = reinterpret_cast<const bf16*>(&qt[u]);
        const bf16* eh = reinterpret_cast<const bf16*>(&qh[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) f(8 * (g0 + i) + e, bf2f(et[e]), bf2f(eh[e]));
      }
    }
  }
  for (int j = v0 + ng * 8 + threadIdx.x; j < v1; j += ACC_THREADS) f(j, bf2f(t[j]), h ? bf2f(h[j]) : 0.f);
}

struct AcceptIO {
  const bf16* target_logits;   // [B*NN][V]
  const long long* target_argmax;  // [B*NN]
  const bf16* head_logits;     // [rows][V]
  const long long* ids;        // [B][NN]
  const int* hrow;             // [B][NN]
  const int* children;         // [B][NN][k]
  const float* U;              // [B][depth+1][k+1] (NULL: greedy)
  float* scratch;              // unused (kept in the ABI; may be null)
  int* path;                   // [B][depth+1] node indices (-1 pad)
  int* accept_len;             // [B]
  long long* tokens;           // [B][depth+2]: accepted tokens then the bonus (-1 pad)
  long long* cur;              // [B] <- bonus
  int NN, V, k, depth;
};

// grid (ACC_CL, B): blockIdx.x = rank in the sequence's cluster
template <int RULE>
__global__ void __cluster_dims__(ACC_CL, 1, 1) __launch_bounds__(ACC_THREADS, 1) accept_tree_kernel(AcceptIO io) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cl = cg::this_cluster();
  __shared__ float red[64];
  __shared__ int s_next, s_idx, s_pick, s_last;
  __shared__ AccNode s_node;
  __shared__ Xch xch;
  const int rank = blockIdx.x, b = blockIdx.y;
  const int NN = io.NN, V = io.V, k = io.k;
  const int vs = ((V + ACC_CL - 1) / ACC_CL + 7) / 8 * 8;
  const int v0 = min(V, rank * vs), v1 = min(V, v0 + vs);
  int phase = 0;
  int node = 0, d = 0, bonus = 0;
  for (;;) {
    const int* kids = io.children + ((size_t)b * NN + node) * k;
    if (io.U == nullptr) {  // greedy: no vocabulary work; every rank follows the same path
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
      if (rank == 0 && threadIdx.x == 0) io.path[b * (io.depth + 1) + d] = nxt;
      node = nxt;
      ++d;
      continue;
    }
    const float* u = io.U + ((size_t)b * (io.depth + 1) + d) * (k + 1);
    const bool has_kids = kids[0] >= 0;
    const bf16* trow = io.target_logits + ((size_t)b * NN + node) * V;
    const bf16* hrow = has_kids && RULE == ACC_RULE_DRAFT
                           ? io.head_logits + (size_t)io.hrow[(size_t)b * NN + node] * V
                           : nullptr;
    // both log-sum-exps in one pass over this rank's slice, then across the cluster
    float mt = -INFINITY, st = 0.f, mh = -INFINITY, sh = 0.f;
    for_each_strided(trow, hrow, v0, v1, [&](int, float tj, float hj) {
      lse_merge(mt, st, tj, 1.f);
      if (hrow) lse_merge(mh, sh, hj, 1.f);
    });
    block_lse(mt, st, red, red + 32);
    block_lse(mh, sh, red, red + 32);
    if (threadIdx.x == 0) {
      float* o = xch_publish(xch, phase);
      o[0] = mt;
      o[1] = st;
      o[2] = mh;
      o[3] = sh;
    }
    cl.sync();
    mt = -INFINITY, st = 0.f, mh = -INFINITY, sh = 0.f;
    for (int q = 0; q < ACC_CL; ++q) {
      const float* o = xch_remote(cl, xch, phase, q);
      lse_merge(mt, st, o[0], o[1]);
      lse_merge(mh, sh, o[2], o[3]);
    }
    ++phase;
    if (threadIdx.x == 0) {
      s_node.lse_t = mt + logf(st);
      s_node.lse_h = hrow ? mh + logf(sh) : 0.f;
      s_node.r = 0;
      s_node.invQ[0] = 1.f;
    }
    __syncthreads();
    int nxt = -1;
    float qrem = 1.f;
    for (int i = 0; i < k && has_kids && kids[i] >= 0; ++i) {
      const int c = kids[i];
      const int x = (int)io.ids[(size_t)b * NN + c];
      const int xr = min(max(x, 0), V - 1);  // row index for the logits reads (ids come from top-k)
      // rank 0 decides and broadcasts: the ranks' control flow (and so their
      // cluster barriers) cannot diverge
      if (rank == 0 && threadIdx.x == 0) {
        const float tx = bf2f(trow[xr]), hx = hrow ? bf2f(hrow[xr]) : 0.f;
        xch_publish(xch, phase)[0] = u[i] * acc_q<RULE>(s_node, hx, x, x) < acc_p<RULE>(s_node, tx, hx, x) ? 1.f : 0.f;
      }
      cl.sync();
      const bool acc = xch_remote(cl, xch, phase, 0)[0] != 0.f;
      ++phase;
      if (acc) {
        nxt = c;
        break;
      }
      // rejected: Z_{r+1} over the vocabulary, then record x
      float z = 0.f;
      for_each_strided(trow, hrow, v0, v1, [&](int j, float tj, float hj) {
        z += fmaxf(acc_p<RULE>(s_node, tj, hj, j) - acc_q<RULE>(s_node, hj, j, x), 0.f);
      });
      z = block_sum(z, red);
      if (threadIdx.x == 0) xch_publish(xch, phase)[0] = z;
      cl.sync();
      z = 0.f;
      for (int q = 0; q < ACC_CL; ++q) z += xch_remote(cl, xch, phase, q)[0];
      ++phase;
      if (threadIdx.x == 0) {
        const int r = s_node.r;
        if (hrow) qrem -= expf(bf2f(hrow[xr]) - s_node.lse_h);
        s_node.invZ[r + 1] = z > 0.f ? 1.0f / z : 0.f;
        s_node.invQ[r + 1] = qrem > 0.f ? 1.0f / qrem : 0.f;
        s_node.X[r] = x;
        s_node.r = r + 1;
      }
      __syncthreads();
    }
    if (nxt >= 0) {
      if (rank == 0 && threadIdx.x == 0) io.path[b * (io.depth + 1) + d] = nxt;
      node = nxt;
      ++d;
      continue;
    }
    // bonus: first index whose inclusive prefix sum of p_r exceeds u[k] * total
    // (contiguous chunks per thread inside the rank's slice); if rounding
    // leaves none, the last index with mass (the oracle's inverse_cdf)
    const int n = v1 - v0;
    const int chunk = (n + ACC_THREADS - 1) / ACC_THREADS;
    const int lo = v0 + min(n, (int)threadIdx.x * chunk), hi = v0 + min(n, ((int)threadIdx.x + 1) * chunk);
    float part = 0.f;
    int last = -1;
    for (int j = lo; j < hi; ++j) {
      const float pj = acc_p<RULE>(s_node, bf2f(trow[j]), hrow ? bf2f(hrow[j]) : 0.f, j);
      part += pj;
      if (pj > 0.f) last = j;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float incl = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (threadIdx.x == 0) {
      s_pick = -1;
      s_last = -1;
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    if (last >= 0) atomicMax(&s_last, last);
    __syncthreads();
    if (warp == 0) {
      float w = lane < ACC_WARPS ? red[lane] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < ACC_WARPS) red[32 + lane] = w;  // inclusive prefix over warps
    }
    __syncthreads();
    const float cta_total = red[32 + ACC_WARPS - 1];
    incl += warp == 0 ? 0.f : red[32 + warp - 1];
    if (threadIdx.x == 0) {
      float* o = xch_publish(xch, phase);
      o[0] = cta_total;
      o[1] = __int_as_float(s_last);
    }
    cl.sync();
    float base = 0.f, total = 0.f;
    int glast = -1;
    for (int q = 0; q < ACC_CL; ++q) {
      const float* o = xch_remote(cl, xch, phase, q);
      if (q < rank) base += o[0];
      total += o[0];
      glast = max(glast, __float_as_int(o[1]));
    }
    ++phase;
    const float thr = u[k] * total;
    const float before = base + incl - part;
    if (lo < hi && before <= thr && base + incl > thr) {
      float run = before;
      int pick = hi - 1;
      for (int j = lo; j < hi; ++j) {
        run += acc_p<RULE>(s_node, bf2f(trow[j]), hrow ? bf2f(hrow[j]) : 0.f, j);
        if (run > thr) {
          pick = j;
          break;
        }
      }
      s_pick = pick;
    }
    __syncthreads();
    if (threadIdx.x == 0) xch_publish(xch, phase)[0] = __int_as_float(s_pick);
    cl.sync();
    int pick = -1;
    for (int q = 0; q < ACC_CL && pick < 0; ++q) pick = __float_as_int(xch_remote(cl, xch, phase, q)[0]);
    ++phase;
    bonus = pick >= 0 ? pick : max(glast, 0);
    break;
  }
  // no CTA may exit while another can still read its shared memory
  cl.sync();
  if (rank == 0 && threadIdx.x == 0) {
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
  pdl_trigger();
  pdl_wait();
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
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lengths[b] += accept_len[b] + 1;
}

}  // namespace

extern "C" size_t tsds_tree_state_bytes(int B) { return (size_t)B * sizeof(TreeState); }

extern "C" int tsds_logits_topk(const void* logits, int ld, int M, int V, int k, float* vals, int32_t* idx,
                                float* lse, tsds_stream_t stream) {
  TSDS_RETURN_IF(!logits || !vals || !idx || !lse || M <= 0 || V <= 0 || ld < V, TSDS_E_INVALID);
  switch (k) {
    case 1: tsds_launch(topk_lse_kernel<1>, dim3(TOPK_CL, M), dim3(TOPK_THREADS), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 2: tsds_launch(topk_lse_kernel<2>, dim3(TOPK_CL, M), dim3(TOPK_THREADS), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 4: tsds_launch(topk_lse_kernel<4>, dim3(TOPK_CL, M), dim3(TOPK_THREADS), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
    case 8: tsds_launch(topk_lse_kernel<8>, dim3(TOPK_CL, M), dim3(TOPK_THREADS), 0, stream, (const bf16*)logits, ld, V, vals, idx, lse); break;
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
  tsds_launch(tree_step_kernel, dim3(B), dim3(STATE_THREADS), 0, stream, (TreeState*)states, vals, (const int*)idx,
              lse, row_base, T, k, next_T, (const int*)lengths, io, B);
  return tsds_launch_status();
}

extern "C" int tsds_tree_finalize(const void* states, int n_nodes, int k, const int32_t* lengths, int64_t* ids,
                                  int32_t* positions, uint32_t* masks, int32_t* hrow, int32_t* children,
                                  int32_t* starts, int B, tsds_stream_t stream) {
  TSDS_RETURN_IF(!states || n_nodes < 1 || n_nodes + 1 > 32 || k < 1 || k > MAXK || B <= 0, TSDS_E_INVALID);
  VerifyIO io{(long long*)ids, positions, (unsigned*)masks, hrow, children, starts};
  tsds_launch(tree_finalize_kernel, dim3(B), dim3(STATE_THREADS), 0, stream, (const TreeState*)states, n_nodes, k,
              (const int*)lengths, io, B);
  return tsds_launch_status();
}

extern "C" int tsds_accept_tree_rule(const void* target_logits, const int64_t* target_argmax,
                                     const void* head_logits, const int64_t* ids, const int32_t* hrow,
                                     const int32_t* children, const float* U, int rule, int32_t* path,
                                     int32_t* accept_len, int64_t* tokens, int64_t* cur, int B, int n_nodes, int V,
                                     int k, int depth, tsds_stream_t stream) {
  TSDS_RETURN_IF(B <= 0 || n_nodes < 1 || V <= 0 || k < 1 || k > MAXK || depth < 1, TSDS_E_INVALID);
  TSDS_RETURN_IF(rule != ACC_RULE_DRAFT && rule != ACC_RULE_TARGET, TSDS_E_INVALID);
  TSDS_RETURN_IF(U != nullptr && !target_logits, TSDS_E_INVALID);
  TSDS_RETURN_IF(U != nullptr && rule == ACC_RULE_DRAFT && !head_logits, TSDS_E_INVALID);
  TSDS_RETURN_IF(U == nullptr && !target_argmax, TSDS_E_INVALID);
  AcceptIO io{(const bf16*)target_logits, (const long long*)target_argmax, (const bf16*)head_logits,
              (const long long*)ids, hrow, children, U, nullptr, path, accept_len, (long long*)tokens,
              (long long*)cur, n_nodes + 1, V, k, depth};
  if (rule == ACC_RULE_TARGET)
    tsds_launch(accept_tree_kernel<ACC_RULE_TARGET>, dim3(ACC_CL, B), dim3(ACC_THREADS), 0, stream, io);
  else
    tsds_launch(accept_tree_kernel<ACC_RULE_DRAFT>, dim3(ACC_CL, B), dim3(ACC_THREADS), 0, stream, io);
  return tsds_launch_status();
}

extern "C" int tsds_accept_tree(const void* target_logits, const int64_t* target_argmax, const void* head_logits,
                                const int64_t* ids, const int32_t* hrow, const int32_t* children, const float* U,
                                float* scratch, int32_t* path, int32_t* accept_len, int64_t* tokens, int64_t* cur,
                                int B, int n_nodes, int V, int k, int depth, tsds_stream_t stream) {
  (void)scratch;
  return tsds_accept_tree_rule(target_logits, target_argmax, head_logits, ids, hrow, children, U, ACC_RULE_DRAFT,
                               path, accept_len, tokens, cur, B, n_nodes, V, k, depth, stream);
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

// Pooled KV commit: one CTA per sequence.  Thread 0 swaps the accepted
// nodes' table entries with the positions after the root, so the table stays
// a permutation of its rows: the rejected nodes' rows move to the positions
// past the new length, where the next forward writes, and no pool row ever
// backs two positions.  Increasing j is safe: path[j] > path[j'] for j' < j,
// and position L + path[j] is never one an earlier swap wrote (those are
// L + 1 + j' < L + path[j] and L + path[j'] != L + path[j]).  It then lists
// the kept pool rows and advances the length; the CTA copies the last
// accepted node's hidden state to root_feat.
__global__ void tree_commit_paged_kernel(int* __restrict__ table, long long table_ld,
                                         const long long* __restrict__ req_rows, int* __restrict__ lengths,
                                         const int* __restrict__ path, const int* __restrict__ accept_len, int depth,
                                         long long* __restrict__ kept, const bf16* __restrict__ hidden, int NN, int N,
                                         bf16* __restrict__ root_feat) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int a = accept_len[b];
  const int L = lengths[b];
  if (root_feat) {
    const int last = a > 0 ? path[b * (depth + 1) + a - 1] : 0;
    const bf16* src = hidden + ((size_t)b * NN + last) * N;
    for (int i = threadIdx.x; i < N / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(root_feat + (size_t)b * N)[i] = reinterpret_cast<const uint4*>(src)[i];
  }
  if (threadIdx.x != 0) return;
  int* row = table + (req_rows ? req_rows[b] : (long long)b) * table_ld;
  for (int j = 0; j < a; ++j) {
    const int from = L + path[b * (depth + 1) + j], to = L + 1 + j;
    const int r = row[from];
    row[from] = row[to];
    row[to] = r;
  }
  if (kept)
    for (int i = 0; i < depth + 2; ++i) kept[(long long)b * (depth + 2) + i] = i <= a ? row[L + i] : -1;
  lengths[b] = L + a + 1;
}

extern "C" int tsds_tree_commit_paged(int32_t* token_table, int64_t table_ld, const int64_t* req_rows,
                                      int32_t* lengths, const int32_t* path, const int32_t* accept_len, int depth,
                                      int64_t* kept_rows, const void* hidden, int n_nodes, int N, void* root_feat,
                                      int B, tsds_stream_t stream) {
  TSDS_RETURN_IF(!token_table || table_ld <= 0 || !lengths || !path || !accept_len || depth < 1 || B <= 0,
                 TSDS_E_INVALID);
  TSDS_RETURN_IF(root_feat && (!hidden || n_nodes < 1 || N <= 0 || (N % 8) != 0), TSDS_E_INVALID);
  tsds_launch(tree_commit_paged_kernel, dim3(B), dim3(128), 0, stream, (int*)token_table, (long long)table_ld,
              (const long long*)req_rows, (int*)lengths, (const int*)path, (const int*)accept_len, depth,
              (long long*)kept_rows, (const bf16*)hidden, n_nodes + 1, N, (bf16*)root_feat);
  return tsds_launch_status();
}

// X2[m] = [feature | embedding(token)] for the head's pass rows m = b*T + t.
__global__ void eagle_inputs_kernel(const bf16* __restrict__ root_feat, const bf16* __restrict__ head_feat,
                                    const int* __restrict__ featrow, const long long* __restrict__ tok,
                                    const bf16* __restrict__ embed, bf16* __restrict__ out, int T, int N, int vocab) {
  pdl_trigger();
  pdl_wait();
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
