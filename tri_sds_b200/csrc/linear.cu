// ABI entry points of the linear-layer family (tsds_linear*).
#include "linear.cuh"

namespace {

int check_linear(const void* x, int ldx, const void* W, const void* out, int ldo, int M, int n_out, int K) {
  TSDS_RETURN_IF(!x || !W || !out, TSDS_E_INVALID);
  TSDS_RETURN_IF(M <= 0 || n_out <= 0 || K <= 0 || (K % 8) != 0 || ldx < K || ldo < n_out, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(x) || !tsds_aligned16(W) || (ldx % 8) != 0, TSDS_E_ALIGN);
  return TSDS_OK;
}

int run_linear(int epi, const void* x, int ldx, const void* W, const void* res, void* out, int ldo, int M, int n_out,
               int K, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  return tsds_gemv_dispatch(epi, (const bf16*)x, ldx, (const bf16*)W, (const bf16*)res, (bf16*)out, ldo, M, n_out, K,
                            stream);
}

}  // namespace

extern "C" size_t tsds_linear_workspace_bytes(int M, int n_out, int K) {
  (void)M;
  (void)n_out;
  (void)K;
  return 0;
}

extern "C" int tsds_linear(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out, int K,
                           void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  return run_linear(EPI_STORE, x, ldx, W, nullptr, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_residual(const void* x, int ldx, const void* W, const void* res, void* out, int ldo, int M,
                                    int n_out, int K, void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  TSDS_RETURN_IF(!res, TSDS_E_INVALID);
  return run_linear(EPI_RESIDUAL, x, ldx, W, res, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}

extern "C" int tsds_linear_swiglu(const void* x, int ldx, const void* W, void* out, int ldo, int M, int n_out, int K,
                                  void* workspace, size_t workspace_bytes, tsds_stream_t stream) {
  int st = check_linear(x, ldx, W, out, ldo, M, n_out, K);
  if (st != TSDS_OK) return st;
  return run_linear(EPI_SWIGLU, x, ldx, W, nullptr, out, ldo, M, n_out, K, workspace, workspace_bytes, stream);
}
