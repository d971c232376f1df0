// Internal interface between the linear-layer ABI and its kernels.
#pragma once
#include "common.cuh"

enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2 };

// CUDA-core GEMV, any M (processed 8 rows per launch).
int tsds_gemv_dispatch(int epi, const bf16* x, int ldx, const bf16* W, const bf16* res, bf16* out, int ldo, int M,
                       int n_out, int K, cudaStream_t stream);
