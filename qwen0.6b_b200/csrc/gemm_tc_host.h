// Internal host interface of the tcgen05 GEMM (gemm_tc.cu), used by the
// batched decode step.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm_tc.cuh"
#include "launch.h"

// Tensor maps and shape of one GEMM C[M, N] = A[M, K] . B[N, K]^T.
struct GemmPlan {
  CUtensorMap ma, mb;
  int M, N, K, bn;
};

// Tile width (64 or 128 columns) used for an M x N output.
int qb200_gemm_bn(int M, int N);
// Builds the tensor maps (row pitches lda, ldb in elements).  0 or an error code.
int qb200_gemm_make_maps(GemmPlan *p, const void *a, const void *b, int M, int N, int K, int lda,
                         int ldb);
// Launches the GEMM with epilogue `epi` (qb200tc::Epilogue) on the first g.M
// rows (all planned rows when g.M is 0); g.N/K/n_tiles come from the plan.
int qb200_gemm_run(const GemmPlan &p, int epi, qb200tc::GemmArgs g, cudaStream_t st);
// Split-K: `splits` CTAs along K write fp32 partial slices into `partial`
// ([splits, M, N]); a reduction sums them in slice order and applies `epi`
// (EPI_F16, EPI_F32, EPI_F32_RES16 or EPI_F16_RES32) into g.out.
int qb200_gemm_run_splitk(const GemmPlan &p, int epi, qb200tc::GemmArgs g, int splits,
                          float *partial, cudaStream_t st);
// out[r] = argmax over the per-tile partials of an EPI_ARGMAX GEMM.
int qb200_argmax_reduce(const float *part_val, const int *part_idx, int n_tiles, int rows, int *out,
                        cudaStream_t st, bool pdl = false);
