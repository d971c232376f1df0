// Internal interface between the linear-layer ABI and its kernels.
#pragma once
#include "common.cuh"

enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_STORE_F32 = 4 };

// CUDA-core GEMV, any M (processed 8 rows per launch).
// res[m * res_ld + j] is the residual (res_ld = 0: a bias broadcast over rows).
int tsds_gemv_dispatch(int epi, const bf16* x, int ldx, const bf16* W, const bf16* res, int res_ld, bf16* out, int ldo,
                       int M, int n_out, int K, cudaStream_t stream);

// tcgen05 persistent GEMM, M <= 256.  epi also accepts EPI_ARGMAX (LM head:
// bf16 logits to `out` when non-null, per-tile candidates to cand_*).
enum { EPI_ARGMAX = 3 };
size_t tsds_tc_workspace_bytes(int M);
int tsds_tc_gemm(int epi, const bf16* x, int ldx, const bf16* W, int w_rows, const bf16* res, int res_ld, bf16* out,
                 int ldo, int M, int n_out, int K, void* workspace, size_t workspace_bytes, float* cand_val,
                 int* cand_idx, int ldc, cudaStream_t stream);

// The residual epilogue followed by RMSNorm of its output rows (weights
// norm_w, eps) into norm_out, in one launch; M <= 256.
int tsds_tc_gemm_residual_norm(const bf16* x, int ldx, const bf16* W, const bf16* res, int res_ld, bf16* out, int ldo,
                               int M, int n_out, int K, const bf16* norm_w, bf16* norm_out, int norm_ld, float eps,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream);

// Row count up to which the CUDA-core GEMV is used instead of tcgen05.
int tsds_gemv_rows_limit();

// Launch shape of the tcgen05 kernels: SMs of the current device, and the
// CTAs-per-SM setting (tsds_set_gemm_ctas_per_sm) before the TMEM cap.
int tsds_tc_num_sms();
int tsds_tc_ctas_setting();
// Token rows from which the tcgen05 kernels run on CTA pairs (0: never).
int tsds_tc_pair_rows();
// Units on which a tcgen05 projection of M rows and `tiles` weight tiles,
// given `units` CTAs (or pairs), runs data-parallel; 0: stream-K
// (tsds_set_gemm_dp_rows / _slack).
int tsds_tc_dp_units(int M, int tiles, int units);

// Fused-layer kernel only: q/k/v projection whose epilogue applies QK-norm + RoPE
// and writes q and the K/V cache rows (one 128-row tile = one head).
enum { EPI_QKROPE = 5 };
