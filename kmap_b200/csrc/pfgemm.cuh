// pfgemm.cuh -- the prefill TT-GEMM on the tensor cores (pfgemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kllm {

// Shapes the tensor-core path takes: K a multiple of 64, N of 128.
bool pf_gemm_applies(int K, int N);
// Wt[N][K] bf16 = codebook[idx[k][n]] transposed; every codebook entry must
// be a bf16 number (checked by the caller).
bool pf_build_wt(cudaStream_t s, const uint16_t *idx, const float *cb, int K, int N,
                 void *wt_bf16);
// xs[terms][n] bf16: the terms of the exact split of x[n] (terms 2 or 3).
bool pf_split(cudaStream_t s, const float *x, long long n, int terms, void *xs_bf16);
// y[R][N] fp32 = sum over the terms of xs[t] (R x K) . Wt^T (K x N).
bool pf_gemm_tc(cudaStream_t s, const void *xs_bf16, int terms, int R, int K, const void *wt_bf16,
                int N, float *y, int *status);

// Few rows (R <= 128, decode of many sequences): the weight on the MMA's
// 128-row side, K split over bd_gemm_splits(K, N) ranges whose partial
// tiles (part: that many x R x N floats; unused for one range) are summed
// in order into y -- or, with nz_out, left in part for the caller to sum
// (*nz_out ranges; one range writes y).
int bd_gemm_splits(int K, int N);
// Kernel attributes of every few-row instance set up front (before a graph
// capture of its launches).
bool bd_gemm_prepare();
bool bd_gemm_tc(cudaStream_t s, const void *xs_bf16, int terms, int R, int K, const void *wt_bf16,
                int N, float *y, float *part, int *status, int *nz_out = nullptr);

}  // namespace kllm
