// ABI entry points of the linear-layer family (tsds_linear*).
#include "linear.cuh"

namespace {

int check_linear(const void* x, int ldx, const void* W, const void* out, int ldo, int M, int n_out, int K) {
  TSDS_RETURN_IF(!x || !W || !out, TSDS_E_INVALID);
  TSDS_RETURN_IF(M <= 0 || n_out <= 0 || K <= 0 || (K % 8) != 0 || ldx < K || ldo < n_out, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(x) || !tsds_aligned16(W) || (ldx % 8) != 0, TSDS_E_ALIGN);
  return TSDS_OK;
}

// Measured on B200: the TMA-fed tcgen05 GEMM streams weights faster than the
// CUDA-core GEMV even at M = 1, so the GEMV is opt-in (tsds_set_gemv_max_rows).
std::atomic<int> g_gemv_max_rows{0};

int run_linear(int epi, const void* x, int ldx, const void* W, const void* res, int res_ld, void* out, int ldo, int M,
               int n_out, int K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (M <= g_gemv_max_rows)
    return tsds_gemv_dispatch(epi, (const bf16*)x, ldx, (const bf16*)W, (const bf16*)res, res_ld, (bf16*)out, ldo, M,
                              n_out, K, stream);
  const int w_rows = epi == EPI_SWIGLU ? 2 * n_out : n_out;
  for (int m0 = 0; m0 < M; m0 += 256) {  // rows beyond 256 (prefill-sized) in chunks
    const int mc = M - m0 < 256 ? M - m0 : 256;
    const bf16* res_c = res ? (const bf16*)res + (int64_t)m0 * res_ld : nullptr;
    bf16* out_c = epi == EPI_STORE_F32 ? reinterpret_cast<bf16*>((float*)out + (int64_t)m0 * ldo)
                                       : (bf16*)out + (int64_t)m0 * ldo;
    int st = tsds_tc_gemm(epi, (const bf16*)x + (int64_t)m0 * ldx, ldx, (const bf16*)W, w_rows, res_c, res_ld, out_c,
                          ldo, mc, n_out, K, workspace, workspace_bytes, nullptr, nullptr, 0, stream);
    if (st != TSDS_OK) return st;
  }
  return TSDS_OK;
}

}  // namespace

int tsds_gemv_rows_limit() { return g_gemv_max_rows; }

extern "C" int tsds_get_gemv_max_rows(void) { return g_gemv_max_rows; }

extern "C" void tsds_set_gemv_max_rows(int rows) { g_gemv_max_rows = rows < 0 ? 0 : (rows > 8 ? 8 : rows); }

extern "C" size_t tsds_linear_workspace_bytes(int M, int n_out, int K) {
  (void)n_out;
  (void)K;
  if (M <= g_gemv_max_rows) return 0;
  return tsds_tc_workspace_bytes(M < 256 ? M : 256);
}

extern "C" int tsds_linear(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out, int K,
                           void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  return run_linear(EPI_STORE, x, ldx, W, nullptr, 0, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_residual(const void* x, int ldx, const void* W, const void* res, void* out, int ldo, int M,
                                    int n_out, int K, void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  TSDS_RETURN_IF(!res, TSDS_E_INVALID);
  return run_linear(EPI_RESIDUAL, x, ldx, W, res, ldo, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_residual_norm(const void* x, int ldx, const void* W, const void* res, void* out, int ldo,
                                         int M, int n_out, int K, const void* norm_w, void* norm_out, int norm_ld,
                                         float eps, void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  TSDS_RETURN_IF(!res || !norm_w || !norm_out || (n_out % 8) != 0 || (ldo % 8) != 0 || (norm_ld % 8) != 0 ||
                     norm_ld < n_out,
                 TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(out) || !tsds_aligned16(norm_w) || !tsds_aligned16(norm_out), TSDS_E_ALIGN);
  if (M <= g_gemv_max_rows || M > 256 || n_out > 8192) {
    // the GEMV path, more rows than one launch takes, or rows wider than the
    // fused tail keeps in registers: the two steps apart
    st = run_linear(EPI_RESIDUAL, x, ldx, W, res, ldo, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
    if (st != TSDS_OK) return st;
    return tsds_rms_norm(out, norm_w, norm_out, M, n_out, ldo, norm_ld, eps, stream);
  }
  TSDS_RETURN_IF(workspace == nullptr, TSDS_E_WORKSPACE);
  return tsds_tc_gemm_residual_norm((const bf16*)x, ldx, (const bf16*)W, (const bf16*)res, ldo, (bf16*)out, ldo, M,
                                    n_out, K, (const bf16*)norm_w, (bf16*)norm_out, norm_ld, eps, workspace,
                                    workspace_bytes, stream);
}

extern "C" int tsds_linear_swiglu(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out, int K,
                                  void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  return run_linear(EPI_SWIGLU, x, ldx, W, nullptr, 0, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_f32(const void* x, int ldx, const void* W, float* out, int ldo, int M, int n_out, int K,
                               void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  return run_linear(EPI_STORE_F32, x, ldx, W, nullptr, 0, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_bias(const void* x, int ldx, const void* W, const void* bias, void* out, int ldo, int M,
                                int n_out, int K, void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  TSDS_RETURN_IF(!bias, TSDS_E_INVALID);
  return run_linear(EPI_RESIDUAL, x, ldx, W, bias, 0, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}
