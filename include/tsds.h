/*
 * tsds.h - C ABI of libtsds.so, the sm_100a speculative-decoding hot path.
 *
 * Every entry point takes device pointers, sizes and a cudaStream_t, launches
 * asynchronously on that stream, never allocates, never synchronises, and
 * returns TSDS_OK or a TSDS_E_* code (bad shape / alignment, launch error).
 * The caller owns every buffer, including the workspace some entry points
 * take (query its size with the matching *_workspace_bytes function).
 * Calls on different streams with different workspaces may run
 * concurrently, also from several host threads (the library's host-side
 * caches are thread-safe); calls that share a workspace must be ordered.
 * The tsds_set_* tuning switches are process-wide and apply to calls made
 * after them.
 *
 * Element types: bf16 buffers are "const void*" / "void*" holding
 * __nv_bfloat16; token ids are int64 (torch.long); lengths, positions and
 * accept lengths are int32.
 *
 * Layouts (row-major):
 *   activations  x[M][N]        M = B*T token rows, sequence b owns rows b*T..b*T+T-1
 *   weights      W[out][in]     the HF nn.Linear layout ("in" contiguous)
 *   KV cache     C[B][Hkv][S][D] one tensor per layer (qwen_model.py:86-94)
 *   RoPE tables  cos/sin[P][D/2] bf16 (qwen_model.py:8-14)
 *
 * Each declaration names the reference interface it replaces (file:line in
 * the reference project, Mog9/tri-sds).
 */
#ifndef TSDS_H
#define TSDS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tsds_stream_t; /* == cudaStream_t */

enum {
  TSDS_OK = 0,
  TSDS_E_INVALID = 1,     /* shape / argument out of the supported range */
  TSDS_E_ALIGN = 2,       /* pointer or leading dimension not 16-byte aligned */
  TSDS_E_LAUNCH = 3,      /* the CUDA launch itself failed */
  TSDS_E_WORKSPACE = 4,   /* workspace smaller than *_workspace_bytes */
  TSDS_E_TIMEOUT = 5,     /* a device-side bounded wait gave up (status word) */
  TSDS_E_UNSUPPORTED = 6, /* no kernel instantiated for this configuration */
  TSDS_E_DEVICE = 7,      /* device query failed / not an sm_100 device */
  TSDS_E_SCRATCH_LIMIT = 8, /* request larger than a built-in scratch area */
  TSDS_E_RUNTIME = 9,       /* a CUDA runtime call (allocation, IPC mapping) failed */
  TSDS_E_INDEX = 10         /* a device-side table entry (KV pool row) outside its pool:
                               the access was redirected to row 0 (status word) */
};

/* Human-readable name of a status code (static string). */
const char* tsds_status_string(int status);
/* ABI version: bumps on any signature change. */
int tsds_abi_version(void);
/* Programmatic dependent launch of the library's kernels (default on): a
 * kernel may start while the previous one in the stream drains; each waits
 * (griddepcontrol.wait) before touching data earlier kernels produce. */
void tsds_set_pdl(int on);
/* Number of kernels this library has enqueued in the process so far (host
 * counter; a launch recorded into a CUDA graph counts once, at capture). */
int64_t tsds_launch_count(void);

/* ---------------------------------------------------------------------------
 * Embedding gather: out[m][:] = table[ids[m * ids_stride]][:]; an id outside
 * [0, vocab) gives a zero row.
 * Replaces state.embed_w[input_ids] (qwen_model.py:188,199; eagle_head.py:113).
 */
int tsds_embed(const int64_t* ids, int ids_stride, const void* table, void* out, int M, int N,
               int vocab, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * RMSNorm: out = x * rsqrt(mean(x^2) + eps) * w in fp32, one cast to bf16.
 * Replaces rms_norm / _rms_norm_kernel (norm.py:42-72).
 * x, out: [rows][n] with row strides ldx, ldo (elements).
 */
int tsds_rms_norm(const void* x, const void* w, void* out, int rows, int n, int ldx, int ldo,
                  float eps, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence bookkeeping for one forward of T new tokens per sequence (chain):
 *   starts[b]    = base[b] + offset      (first cache row written)
 *   positions[m] = starts[b] + t         (RoPE position of row m = b*T+t)
 * Replaces the host-side start_pos / positions of qwen_model.py:102,185.
 */
int tsds_prep_chain(const int32_t* base, int offset, int B, int T, int32_t* starts,
                    int32_t* positions, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Projection of the new tokens into q and the KV cache, after the fused
 * GEMM has produced qkv[M][Hq*D + 2*Hkv*D] (bf16):
 *   q, k <- RMSNorm_D(q, q_norm_w), RMSNorm_D(k, k_norm_w)   (skipped if NULL)
 *   q, k <- rotate-half RoPE at positions[m], bf16 rounding as the reference
 *   q_out[m][h*D..]                       = q
 *   k_cache[b][kvh][starts[b]+t][..]      = k ;  v_cache likewise = v
 *   (rows with starts[b]+t outside [0, S) or positions[m] outside
 *    [0, rope_len) - the RoPE tables' length - are skipped)
 * Replaces the QK-norm (absent in the reference), apply_rope and the cache
 * stores of qwen_model.py:109-119 / 154-164, and the RoPE + KV-write half
 * of _rmsnorm_qkv_rope_kernel (fused_qwen_decode.py:212-250).
 */
int tsds_qk_norm_rope_kv(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                         const void* cos, const void* sin, const int32_t* positions,
                         const int32_t* starts, void* q_out, void* k_cache, void* v_cache,
                         int B, int T, int Hq, int Hkv, int D, int S, int rope_len, float eps,
                         tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Skinny GEMM family, out[m][j] = epilogue(sum_k W[j][k] * x[m][k]), fp32
 * accumulation.  x: [M][K] (row stride ldx), W: [n_out][K], K % 8 == 0.
 * Picks the CUDA-core GEMV for small M and the tcgen05 path above it.
 *
 * tsds_linear:           out = bf16(acc)                         (qwen_model.py:108,153)
 * tsds_linear_residual:  out = bf16(res + bf16(acc))              (fused_qwen_decode.py:179-204,
 *                                                                  293-309; qwen_model.py:133-134,143-144)
 *                        out may alias res (in-place residual stream).
 * tsds_linear_swiglu:    W = [gate; up] ([2*n_out][K]);
 *                        out = bf16(bf16(silu(bf16(acc_g))) * bf16(acc_u))
 *                                                                 (fused_qwen_decode.py:242-265;
 *                                                                  qwen_model.py:139-142)
 */
/* Workspace: 0 bytes on the GEMV path; otherwise a status word (int32 at
 * offset 0: TSDS_E_TIMEOUT if a device wait gave up), tile counters that
 * must be zero before the first use (every launch leaves them zero) and
 * fp32 split-K partials.  Zero-fill a fresh workspace once. */
size_t tsds_linear_workspace_bytes(int M, int n_out, int K);
/* Leading bytes of a tcgen05 GEMM / LM-head workspace that hold the status
 * word and the tile counters.  A launch that gave up on a device wait
 * (status TSDS_E_TIMEOUT) may leave counters nonzero: zero these bytes
 * before the workspace is used again.  No counterpart in the reference
 * (its kernels have no device waits). */
size_t tsds_linear_workspace_header_bytes(void);
/* Limit of each bounded device wait of the tcgen05 GEMM and LM head, in
 * nanoseconds (default 2e9, clamped to 1..1e10).  Process-wide; read at
 * launch.  Lowering it makes every wait give up, which tests the timeout
 * recovery; no counterpart in the reference. */
void tsds_set_wait_limit_ns(unsigned long long ns);
unsigned long long tsds_get_wait_limit_ns(void);
/* Largest M served by the CUDA-core GEMV (0..8; above it the tcgen05 GEMM;
 * default 0: tcgen05 for every M).  Process-wide; read by the
 * *_workspace_bytes functions too. */
void tsds_set_gemv_max_rows(int rows);
int tsds_get_gemv_max_rows(void);
/* 1: the GEMV path runs its split-K variant - a CTA per few weight rows,
 * all its threads sweeping K, partials summed across the CTA's warps in a
 * fixed order - so even the narrowest projections cover every SM; 0
 * (default): one warp per weight rows.  Process-wide tuning switch. */
void tsds_set_gemv_splitk(int on);
int tsds_get_gemv_splitk(void);
/* Resident CTAs per SM of the tcgen05 GEMM (1..4, default 2; lowered
 * automatically when the accumulators would not fit in TMEM).  Tuning knob. */
void tsds_set_gemm_ctas_per_sm(int n);
/* Token rows M from which the tcgen05 GEMM runs on CTA pairs (two SMs per
 * 256-row weight tile, tcgen05 cta_group::2, each SM staging half of the
 * token rows; not the LM head); 0 (default): never.  Process-wide tuning
 * switch for large M. */
void tsds_set_gemm_pair_rows(int rows);
int tsds_get_gemm_pair_rows(void);
/* Token rows M from which a tcgen05 projection may run data-parallel -
 * min(tiles, CTAs) CTAs (or CTA pairs) take whole weight tiles, no split
 * tiles and so no fp32 partials exchanged at the end - instead of
 * stream-K; 0: always stream-K (default 128).  It is chosen where its makespan,
 * ceil(tiles / used CTAs) tiles, exceeds the ideal tiles / CTAs by at most
 * tsds_set_gemm_dp_slack percent (default 100; with fewer tiles than CTAs
 * that allows leaving CTAs idle).  Process-wide tuning switches for large
 * M.  The two schedules sum a split tile in a different order, so results
 * may differ in the last bit between them. */
void tsds_set_gemm_dp_rows(int rows);
int tsds_get_gemm_dp_rows(void);
void tsds_set_gemm_dp_slack(int percent);
int tsds_get_gemm_dp_slack(void);
/* The launch shape the tcgen05 GEMM would take for one projection of M
 * rows (epilogue code TSDS_EPI_STORE / _RESIDUAL / _SWIGLU / _STORE_F32, or
 * 3 for the LM head's argmax epilogue; n_out outputs, K inputs)
 * under the current switches: out[0..5] = weight tiles, k-blocks per tile,
 * CTAs, data-parallel (1) or stream-K (0), pipeline stages, CTAs per tile
 * (1, or 2 for a pair).  Host arithmetic only, except with CTA pairs (an
 * occupancy query); no counterpart in the reference (a tuning and test
 * aid). */
int tsds_tc_gemm_plan(int epi, int M, int n_out, int K, int32_t* out);
int tsds_linear(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out, int K,
                void* workspace, size_t workspace_bytes, tsds_stream_t stream);
int tsds_linear_residual(const void* x, int ldx, const void* W, const void* res, void* out, int ldo,
                         int M, int n_out, int K, void* workspace, size_t workspace_bytes,
                         tsds_stream_t stream);
/* tsds_linear_residual, then RMSNorm of its n_out-wide output rows with
 * weights norm_w into norm_out (row stride norm_ld), exactly as
 * tsds_rms_norm(out, norm_w, norm_out, M, n_out, ldo, norm_ld, eps) would
 * (bit for bit) - the residual add of a decoder layer followed by the next
 * RMSNorm (qwen_model.py:133-136 then the next layer's norm, norm.py:42-72).  On the
 * tcgen05 path (1 <= M <= 256) one launch: the first min(M, CTAs) CTAs
 * normalise the rows once every CTA of the GEMM has stored its part, so
 * the separate RMSNorm launch and its kernel boundary go away; uses two more
 * words of the workspace header.  n_out, ldo and norm_ld multiples of 8,
 * out / norm_w / norm_out 16-byte aligned. */
int tsds_linear_residual_norm(const void* x, int ldx, const void* W, const void* res, void* out, int ldo,
                              int M, int n_out, int K, const void* norm_w, void* norm_out, int norm_ld,
                              float eps, void* workspace, size_t workspace_bytes, tsds_stream_t stream);
int tsds_linear_swiglu(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out,
                       int K, void* workspace, size_t workspace_bytes, tsds_stream_t stream);
/* out[m][j] = acc as fp32 (no rounding): a tensor-parallel rank's partial of
 * a row-parallel projection, summed across ranks before the residual add. */
int tsds_linear_f32(const void* x, int ldx, const void* W, float* out, int ldo, int M, int n_out,
                    int K, void* workspace, size_t workspace_bytes, tsds_stream_t stream);
/* out = bf16(bf16(acc) + bias[j]): the EAGLE head's fc (eagle_head.py:80). */
int tsds_linear_bias(const void* x, int ldx, const void* W, const void* bias, void* out, int ldo,
                     int M, int n_out, int K, void* workspace, size_t workspace_bytes,
                     tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Verify / decode attention of T new tokens per sequence over the KV cache.
 * q: [B*T][Hq][D] (RoPE applied); k/v cache [B][Hkv][S][D] holding the new
 * tokens at rows starts[b]..starts[b]+T-1; out: [B*T][Hq][D] bf16.
 * Query t of sequence b sees the rows below starts[b]+T subject to a mask:
 *  - tree_mask NULL: causal - every row below starts[b], then new rows
 *    starts[b]+j for j <= t;
 *  - tree_mask given: bit i of tree_mask[b*T+t] admits row base+i, where
 *    base = starts[b] (mask_origin < 0, T <= 32) or base = mask_origin;
 *    rows below base are visible to every query, rows base+32.. to none.
 * fp32 online softmax, scale = softmax scale.
 * Keys are split into fixed chunks of split_keys rows (a multiple of 64);
 * the split boundaries depend only on the key index, so a query's result
 * does not depend on T or B.  max_kv bounds starts[b]+T (sizes the grid).
 * Replaces attention_gqa / _decode_attn_gqa_kernel (attention.py:236-318)
 * and the verify SDPA of qwen_model.py:121-131.  D = 128, T*Hq/Hkv <= 1024
 * (<= 65536 on the tcgen05 variant below), B*Hkv*S < 2^31.
 */
size_t tsds_attention_workspace_bytes(int B, int T, int Hq, int Hkv, int D, int max_kv,
                                      int split_keys);
int tsds_verify_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                          const int32_t* starts, const uint32_t* tree_mask, int mask_origin, int B,
                          int T, int Hq, int Hkv, int D, int S, int max_kv, int split_keys,
                          float scale, void* workspace, size_t workspace_bytes, int32_t* status,
                          tsds_stream_t stream);
/* The default kernel's launch shape for a call of tsds_verify_attention /
 * tsds_verify_attention_paged on num_sms SMs (0: the current device's):
 * out[0..5] = {row groups per CTA, key groups per split, row blocks, key
 * splits, ring stages, threads per CTA}.  The key-group count depends on
 * split_keys alone and divides the ring depth. */
int tsds_attention_plan(int B, int T, int Hq, int Hkv, int max_kv, int split_keys, int num_sms,
                        int32_t* out);
/* Process-wide switch (default 0): with 1, tsds_verify_attention runs its
 * tcgen05 variant (S = Q K^T and O = P V on the 5th-generation tensor cores,
 * TMEM accumulators, one softmax thread per query row, 128-key tiles) for
 * every call whose split_keys is a multiple of 128; other calls keep the
 * default kernel.  Same arguments, workspace and masking; results agree
 * within fp32 rounding of the products, not bit for bit.  With 2, calls of
 * 2 to 8 key splits also run each row block's splits as one thread-block
 * cluster that combines them through distributed shared memory instead of
 * a second launch (same bits as 1). */
void tsds_set_attention_tc(int mode);
int tsds_get_attention_tc(void);

/* ---------------------------------------------------------------------------
 * Paged KV: SGLang's token pool layout, the KV memory its spec worker runs on
 * (the reference's worker receives SGLang's ScheduleBatch, worker.py:3-4,
 * 59-61, whose requests own rows of a req_to_token table into per-layer
 * token_to_kv_pool buffers).  Per layer, k_pool / v_pool are
 * [pool_rows][Hkv][D] bf16; position p of sequence b lives at pool row
 * token_table[req(b) * table_ld + p], req(b) = req_rows[b] (the batch's
 * req_pool_indices) or b when req_rows is NULL.  page_size: when a multiple
 * of 64, every aligned run of 64 positions must occupy 64 consecutive pool
 * rows (paged allocators with such pages) and tiles are staged by TMA;
 * otherwise (1: one row per token) rows are gathered one by one.
 * A table entry outside [0, pool_rows) is never dereferenced: row 0 is read
 * instead and *status = TSDS_E_INDEX.
 *
 * tsds_verify_attention_paged: as tsds_verify_attention (same q / out /
 * starts / masks / splits / workspace and bit-identical results for the same
 * keys), the cache rows below starts[b]+T read through the table;
 * max_kv <= table_ld.
 */
int tsds_verify_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out,
                                const int32_t* starts, const uint32_t* tree_mask, int mask_origin,
                                const int32_t* token_table, int64_t table_ld, const int64_t* req_rows,
                                int64_t pool_rows, int page_size, int B, int T, int Hq, int Hkv, int D,
                                int max_kv, int split_keys, float scale, void* workspace,
                                size_t workspace_bytes, int32_t* status, tsds_stream_t stream);
/* tsds_qk_norm_rope_kv into the pools: as tsds_qk_norm_rope_kv for M token
 * rows, row m's K / V written to pool row out_loc[m] (SGLang's
 * out_cache_loc); q into q_out [M][Hq][D].  Replaces the cache write of
 * qwen_model.py:118-119 in the pool layout. */
int tsds_qk_norm_rope_kv_paged(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                               const void* cos, const void* sin, const int32_t* positions,
                               const int64_t* out_loc, void* q_out, void* k_pool, void* v_pool, int M,
                               int Hq, int Hkv, int D, int64_t pool_rows, int rope_len, float eps,
                               int32_t* status, tsds_stream_t stream);
/* The new tokens' pool rows: out_loc[b*T + t] = token_table[req(b) *
 * table_ld + starts[b] + t] (-1 past the table), the out_cache_loc of a
 * forward for engines that keep their own table. */
int tsds_table_rows(const int32_t* token_table, int64_t table_ld, const int64_t* req_rows,
                    const int32_t* starts, int B, int T, int64_t* out_loc, tsds_stream_t stream);
/* Tree commit in the pool layout: no K/V moves - the accepted nodes' pool
 * rows become the sequence's next positions.  With L = lengths[b] (the
 * tree's root at position L), a = accept_len[b] and path / accept_len as
 * tsds_accept_tree writes them (accepted non-root nodes, [B][depth+1]):
 * for j = 0 .. a-1 the entries at positions L + 1 + j and L + path[b][j] of
 * row req(b) of token_table are swapped (the table stays a permutation: the
 * rejected nodes' rows land past the new length, where the next forward
 * writes), then lengths[b] += a + 1.  kept_rows (optional, [B][depth+2], -1 padded)
 * receives the pool rows of positions L..L+a afterwards, so the caller can
 * free the tree's other rows.  root_feat (optional) gets the hidden state of
 * the last accepted node as tsds_tree_commit does (hidden [B][n_nodes+1][N]).
 * Replaces tsds_tree_commit's row moves for pooled caches (the reference
 * only advanced a length, qwen_model.py:190,206). */
int tsds_tree_commit_paged(int32_t* token_table, int64_t table_ld, const int64_t* req_rows,
                           int32_t* lengths, const int32_t* path, const int32_t* accept_len, int depth,
                           int64_t* kept_rows, const void* hidden, int n_nodes, int N, void* root_feat,
                           int B, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * tsds_verify_attention for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some callers may not cudaMalloc at all:
 * a plugin hosted by a serving framework that reserved the GPU's memory for
 * itself (SGLang sizes its KV pool to a fixed share of the device), or code
 * that must not allocate while a stream is being captured.  This variant
 * takes no workspace: its split-KV partials live in a built-in device array
 * of tsds_verify_attention_noalloc_limit() bytes (8 MiB, plus a 256-byte
 * status header), which every GPU that loads the library keeps until exit.
 * The caller still passes inputs and outputs; arguments as for
 * tsds_verify_attention.
 *  - The first call on a device looks the array's device address up (that
 *    device must be current) and keeps it with the current context; a call
 *    in another context (after cudaDeviceReset) looks it up again.  Make
 *    the first call on a device, and the first after a reset, before any
 *    stream capture.
 *  - All calls share the array and it keeps the last call's contents; the
 *    status word is cleared at every call.  Calls that overlap on the GPU
 *    race: order them on one stream.
 *  - Requests whose partials exceed the limit return TSDS_E_SCRATCH_LIMIT.
 * tsds_verify_attention_noalloc_status copies the status word of the last
 * call to the host (synchronous).
 */
size_t tsds_verify_attention_noalloc_limit(void);
int tsds_verify_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                                  const int32_t* starts, const uint32_t* tree_mask, int mask_origin,
                                  int B, int T, int Hq, int Hkv, int D, int S, int max_kv,
                                  int split_keys, float scale, tsds_stream_t stream);
int tsds_verify_attention_noalloc_status(int32_t* host_status);

/* ---------------------------------------------------------------------------
 * LM head + greedy pick: logits[m][v] = bf16(sum_k x[m][k] * W[v][k]);
 * argmax_out[m * argmax_stride] = lowest index of the largest bf16 logit
 * (torch.argmax semantics); argmax_val[m] (optional) = that logit.
 * x is the final-normed hidden state.  logits_out may be NULL.
 * Replaces the LM head + argmax of qwen_model.py:192,205 and
 * eagle_head.py:120-121.
 */
/* Workspace: per-row candidates, plus the tcgen05 workspace when M is above
 * the GEMV limit (zero-fill a fresh workspace once, as for tsds_linear). */
size_t tsds_lm_head_workspace_bytes(int M, int vocab);
int tsds_lm_head_argmax(const void* x, int ldx, const void* W, void* logits_out, int64_t* argmax_out,
                        int argmax_stride, float* argmax_val, int M, int vocab, int K,
                        void* workspace, size_t workspace_bytes, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Greedy acceptance + KV commit for one chain cycle (replaces the verify /
 * accept step that tri_sds/worker.py:66-68 leaves unimplemented).
 *   draft[B][K], target[B][K+1]  (argmax ids)
 *   n = longest prefix with draft[b][i] == target[b][i]
 *   accept_len[b] = n;  tokens[b][i] = target[b][i] for i <= n, else -1
 *   target_len[b] += n + 1               (commit: rows past it are stale)
 *   last[b] = token at position target_len-1 (cur if n == 0 else draft[n-1])
 *   cur[b]  = target[b][n]               (the bonus token)
 */
int tsds_accept_greedy(const int64_t* draft, const int64_t* target, int32_t* accept_len,
                       int64_t* tokens, int32_t* target_len, int64_t* last, int64_t* cur, int B,
                       int K, tsds_stream_t stream);

/* Build the verify input ids[b][0..K] = cur[b], draft[b][0..K-1]; and the
 * draft's first-step input ids2[b] = last[b], cur[b]. */
int tsds_gather_ids(const int64_t* cur, const int64_t* last, const int64_t* draft, int64_t* verify_ids,
                    int64_t* draft_ids2, int B, int K, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Tensor-parallel glue (one process per GPU; the collectives themselves are
 * NCCL's, issued by the host between these calls).
 * tsds_residual_add_f32: x = bf16(x + bf16(partial)) for the all-reduced
 *   fp32 partial of a row-parallel projection (qwen_model.py:133-134,143-144).
 * tsds_argmax_merge: per row, the best of tp per-rank (value, local index)
 *   candidates, index offset r * vocab_shard, ties -> lowest global index.
 * tsds_gather_shards: vocab-sharded logits [tp][M][vocab_shard] -> [M][V].
 */
int tsds_residual_add_f32(void* x, const float* partial, int M, int N, tsds_stream_t stream);
int tsds_argmax_merge(const float* vals, const int64_t* idx, int M, int tp, int64_t vocab_shard,
                      int64_t* out, int out_stride, tsds_stream_t stream);
int tsds_gather_shards(const void* src, void* dst, int tp, int M, int vocab_shard,
                       tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused layer: several dependent phases of decoder layers in ONE persistent launch
 * over the same M token rows, e.g. O (+residual) -> RMSNorm -> gate/up
 * (+SwiGLU) -> down (+residual) -> RMSNorm -> q/k/v (+QK-norm + RoPE + K/V
 * cache write).  GEMM phases are the tcgen05 skinny GEMM of tsds_linear*
 * (same tiles, same split-tile reduction, same rounding); RMSNorm phases are
 * tsds_rms_norm's arithmetic; the QKROPE epilogue is tsds_qk_norm_rope_kv's.
 * Phases are separated by an in-kernel grid barrier; weight tiles of the next
 * GEMM phase stream in while the previous phase finishes.  Replaces the
 * per-op launches of fused_qwen_decode.py:151-309 / qwen_model.py:104-144
 * (one launch instead of six) - no counterpart in the reference.
 *
 * Phase descriptors (host array, n_phases <= 8):
 *  GEMM: out[m][j] = epilogue(sum_k w[j][k] * x[m][k]) for m < M, j < n_out;
 *        epi TSDS_EPI_STORE (bf16), _RESIDUAL (bf16(res + bf16(acc)), res may
 *        be out), _SWIGLU (w = [gate; up], 2*n_out rows), _STORE_F32 (fp32),
 *        _QKROPE (n_out = (Hq + 2*Hkv) * 128; outputs as tsds_qk_norm_rope_kv
 *        with the parameters in *qr; out unused; at most one such phase).
 *  NORM: out[m][0:K] = RMSNorm(x[m][0:K]) * w, eps.
 *  PEER: tensor parallelism - out[m][0:K] (bf16, stride ldo) = bf16(out +
 *        bf16(sum over ranks 0..tp-1 of slot n_out (0 or 1) of their peer
 *        buffers, fp32 [M][K]))), the same on every rank; the preceding
 *        STORE_F32 phase writes this rank's partial into that slot (ldo = K).
 *        The peer buffers are those of tsds_peer_allreduce_residual (*peers);
 *        the cross-rank wait is per CTA index and bounded (1 s).  epi 0:
 *        one-shot (every rank reads every partial); epi 1: two-shot (each
 *        rank reduces 1/tp of the elements, publishes them in its buffer,
 *        and copies the others' after a second meeting) - same bits, a 1/tp
 *        of the remote reads.
 * Workspace: tsds_fused_layer_workspace_bytes(M) bytes, 16-byte aligned, zero-filled
 * once (every launch leaves its counters zero again); word 0 is the status
 * word (TSDS_E_TIMEOUT after a bounded device wait gave up).  M <= 256.
 */
enum { TSDS_PHASE_GEMM = 0, TSDS_PHASE_NORM = 1, TSDS_PHASE_PEER = 2 };
enum {
  TSDS_EPI_STORE = 0,
  TSDS_EPI_RESIDUAL = 1,
  TSDS_EPI_SWIGLU = 2,
  TSDS_EPI_STORE_F32 = 4,
  TSDS_EPI_QKROPE = 5
};
typedef struct {
  int kind;          /* TSDS_CHAIN_* */
  int epi;           /* GEMM: TSDS_EPI_* */
  const void* x;     /* GEMM: activations [M][K] bf16; NORM: input rows; PEER: unused */
  int ldx;           /* row stride of x (elements, multiple of 8) */
  int K;             /* GEMM: reduction length; NORM: row length */
  const void* w;     /* GEMM: weights [n_out][K] (SWIGLU [2*n_out][K]); NORM: gain [K] */
  int n_out;         /* GEMM output columns; PEER: the slot */
  int res_ld;        /* RESIDUAL: row stride of res */
  const void* res;   /* RESIDUAL: residual rows */
  void* out;         /* output rows (fp32 for STORE_F32); PEER: the residual, updated in place */
  int ldo;           /* row stride of out */
  float eps;         /* NORM */
} tsds_fused_phase;
typedef struct {
  const void* q_norm_w;          /* [128] bf16, or NULL: no QK-norm */
  const void* k_norm_w;
  const void* cos;               /* [rope_len][64] bf16 */
  const void* sin;
  const int32_t* positions;      /* [M] */
  const int32_t* starts;         /* [M / T] cache row of each sequence's first new token */
  void* q_out;                   /* [M][Hq][128] bf16 */
  void* k_cache;                 /* [M / T][Hkv][S][128] bf16 */
  void* v_cache;
  int T, Hq, Hkv, S, rope_len;
  float eps;
} tsds_qk_rope;
typedef struct {
  void* const* bufs;   /* host array [tp]: every rank's peer buffer as mapped here, bufs[rank] its own */
  int rank, tp;
  int max_elems;       /* the buffers' slot size (tsds_peer_buffer_bytes) */
} tsds_peer_group;
size_t tsds_fused_layer_workspace_bytes(int M);
/* Leading bytes of the fused-layer workspace holding the status word and
 * the phase counters: zero them after a TSDS_E_TIMEOUT before reuse. */
size_t tsds_fused_layer_workspace_header_bytes(void);
/* The grid tsds_fused_layer takes for M rows under the current switches:
 * out[0..3] = CTAs, CTAs per weight tile (2: pairs), pipeline stages, CTAs
 * per SM requested.  A tuning and test aid; no counterpart in the
 * reference. */
int tsds_fused_layer_grid(int M, int32_t* out);
int tsds_fused_layer(const tsds_fused_phase* phases, int n_phases, int M, const tsds_qk_rope* qr,
                     const tsds_peer_group* peers, void* workspace, size_t workspace_bytes,
                     tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Peer (NVLink) all-reduce of row-parallel partials, fused with the residual
 * add: the TP exchange after the O and down projections without NCCL.
 * Replaces the NCCL all-reduce + tsds_residual_add_f32 pair above.
 *
 * Each rank owns one peer buffer of tsds_peer_buffer_bytes(max_elems,
 * exchange_bytes) bytes
 * (tsds_peer_alloc: cudaMalloc, zero-filled), exports it with
 * tsds_peer_export (tsds_peer_handle_bytes() bytes, a CUDA IPC handle) and
 * maps every other rank's with tsds_peer_import (another process of the same
 * node; close with tsds_peer_close, free its own with tsds_peer_free).
 * Buffer layout: per-CTA call counters and flags in the first 32 KB, then two
 * slots of max_elems fp32 at tsds_peer_slot_offset(max_elems, 0 / 1), then
 * max_elems bf16 published by the fused kernel's two-shot all-reduce, then
 * exchange_bytes at tsds_peer_exchange_offset(max_elems) for
 * tsds_peer_lm_gather.
 *
 * tsds_peer_allreduce_residual: the partial [M][N] fp32 of every rank sits in
 * slot `slot` of that rank's buffer (written there by tsds_linear_f32);
 * x[M][N] bf16 = bf16(x + bf16(sum over ranks 0..tp-1 in order)), identical
 * on every rank.  bufs: host array of tp device pointers, bufs[rank] this
 * rank's own buffer, bufs[p] rank p's as mapped here.  Every rank must issue
 * the same sequence of calls with the same M, N, and successive calls must
 * alternate slots (a rank writes a slot again only two calls later).  The
 * cross-rank wait is bounded (1 s): on timeout *status = TSDS_E_TIMEOUT and
 * x is left unchanged.  tp <= 8, N % 4 == 0, M * N <= max_elems, x 8-byte
 * aligned, buffers 16-byte aligned.
 */
size_t tsds_peer_buffer_bytes(int max_elems, size_t exchange_bytes);
size_t tsds_peer_slot_offset(int max_elems, int slot);
size_t tsds_peer_exchange_offset(int max_elems);
size_t tsds_peer_handle_bytes(void);
int tsds_peer_alloc(size_t bytes, void** buf);
int tsds_peer_free(void* buf);
int tsds_peer_export(const void* buf, void* handle);
int tsds_peer_import(const void* handle, void** buf);
int tsds_peer_close(void* buf);
int tsds_peer_allreduce_residual(void* x, void* const* bufs, int rank, int tp, int slot, int M, int N,
                                 int max_elems, int* status, tsds_stream_t stream);
/* Vocab-parallel LM head without NCCL (replaces the all-gathers +
 * tsds_argmax_merge / tsds_gather_shards above): every rank's LM head has
 * written, into the exchange region of its own peer buffer, its shard's
 * argmax candidates - rows int64 local indices at offset 0 and rows fp32
 * values at val_off (tsds_lm_head_argmax's argmax_out / argmax_val) - and,
 * when logits_out is given, its logits shard [rows][vocab_shard] bf16 at
 * log_off.  Writes argmax_out[m * argmax_stride] (best value, ties to the
 * lowest global index) and logits_out [rows][tp * vocab_shard] on every rank.
 * Meets the other ranks before reading and again after, so a rank may
 * overwrite its region once this call has returned on its stream.  Bounded
 * waits (1 s) report TSDS_E_TIMEOUT in *status. */
int tsds_peer_lm_gather(void* const* bufs, int rank, int tp, int max_elems, size_t exchange_bytes, int rows,
                        int vocab_shard, int64_t val_off, int64_t log_off, int64_t* argmax_out,
                        int argmax_stride, void* logits_out, int* status, tsds_stream_t stream);

/* ---------------------------------------------------------------------------
 * Tree speculative decoding (EAGLE draft tree, verified in one target pass).
 * No counterpart in the reference: its chain draft (eagle_head.py:100-129)
 * stops at argmax tokens and tree drafting / acceptance / KV rollback live
 * in SGLang (worker.py:66-68 raises).  Semantics: oracle/eagle.py.
 *
 * tsds_logits_topk: per logits row (bf16, row stride ld): the k largest
 *   values (value desc, index asc) and log-sum-exp, fp32.  k in {1,2,4,8}.
 * tsds_tree_state_bytes: bytes of the per-sequence tree state (opaque).
 * tsds_tree_init: root = current token cur[b]; writes the root head pass's
 *   inputs (token, feature row -1 = root feature, position, head-cache mask,
 *   first head-cache row).
 * tsds_tree_step: after a head pass over T frontier nodes per sequence
 *   (their top-k at global rows row_base + b*T + t): add k children per
 *   node (score = parent + logit - lse), choose the next_T best new nodes
 *   as the next frontier (0: last pass) and write that pass's inputs.
 * tsds_tree_finalize: keep the n_nodes best nodes (score desc, depth asc,
 *   creation asc) and the root; write the verify ids / positions (L + depth)
 *   / ancestor masks / head rows / children lists, and starts = lengths.
 * tsds_accept_tree: walk the verified tree: U given -> rejection sampling
 *   at temperature 1 (accept child x if U*q(x) < p(x); else p <- norm(max(p -
 *   q, 0)), q <- q without x; bonus by inverse CDF); U NULL -> greedy
 *   (child == target argmax).  Writes path node indices, accept lengths,
 *   emitted tokens (accepted + bonus, -1 padded) and cur <- bonus.
 *   scratch: unused (nothing of vocabulary size is stored); may be NULL.
 *   The emitted token is distributed as p when the children were drawn
 *   from q without replacement.
 * tsds_accept_tree_rule: the same walk with the rule chosen per call:
 *   TSDS_ACCEPT_DRAFT (0) is tsds_accept_tree's; TSDS_ACCEPT_TARGET (1)
 *   takes the draft as deterministic (q one-hot on each child in turn):
 *   accept child x if U < p(x); else p <- p without x, renormalised; bonus
 *   by inverse CDF.  It is lossless for children chosen without looking at
 *   U - the tree's top-k expansion - and reads no head logits (may be NULL).
 * tsds_tree_commit: move the accepted nodes' K/V rows L + path[j] -> L+1+j
 *   in every layer, copy the last accepted node's hidden state to
 *   root_feat, then lengths += accept_len + 1.
 * tsds_eagle_inputs: the head pass input [feature | embedding(token)].
 */
int tsds_logits_topk(const void* logits, int ld, int M, int V, int k, float* vals, int32_t* idx,
                     float* lse, tsds_stream_t stream);
size_t tsds_tree_state_bytes(int B);
int tsds_tree_init(void* states, const int64_t* cur, const int32_t* lengths, int64_t* pass_tok,
                   int32_t* pass_featrow, int32_t* pass_pos, uint32_t* pass_mask, int32_t* pass_starts,
                   int B, tsds_stream_t stream);
int tsds_tree_step(void* states, const float* vals, const int32_t* idx, const float* lse, int row_base,
                   int T, int k, int next_T, const int32_t* lengths, int64_t* pass_tok,
                   int32_t* pass_featrow, int32_t* pass_pos, uint32_t* pass_mask, int32_t* pass_starts,
                   int B, tsds_stream_t stream);
int tsds_tree_finalize(const void* states, int n_nodes, int k, const int32_t* lengths, int64_t* ids,
                       int32_t* positions, uint32_t* masks, int32_t* hrow, int32_t* children,
                       int32_t* starts, int B, tsds_stream_t stream);
int tsds_accept_tree(const void* target_logits, const int64_t* target_argmax, const void* head_logits,
                     const int64_t* ids, const int32_t* hrow, const int32_t* children, const float* U,
                     float* scratch, int32_t* path, int32_t* accept_len, int64_t* tokens, int64_t* cur,
                     int B, int n_nodes, int V, int k, int depth, tsds_stream_t stream);
enum { TSDS_ACCEPT_DRAFT = 0, TSDS_ACCEPT_TARGET = 1 };
int tsds_accept_tree_rule(const void* target_logits, const int64_t* target_argmax, const void* head_logits,
                          const int64_t* ids, const int32_t* hrow, const int32_t* children, const float* U,
                          int rule, int32_t* path, int32_t* accept_len, int64_t* tokens, int64_t* cur, int B,
                          int n_nodes, int V, int k, int depth, tsds_stream_t stream);
int tsds_tree_commit(void* k_cache, void* v_cache, int layers, int B, int Hkv, int S, int D,
                     int32_t* lengths, const int32_t* path, const int32_t* accept_len, int depth,
                     const void* hidden, int n_nodes, int N, void* root_feat, tsds_stream_t stream);
int tsds_eagle_inputs(const void* root_feat, const void* head_feat, const int32_t* featrow,
                      const int64_t* tok, const void* embed, void* out, int B, int T, int N, int vocab,
                      tsds_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TSDS_H */
