// Internal host interface of the tcgen05 GEMM (gemm_tc.cu), used by the
// batched decode step.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm_tc.cuh"
#include "launch.h"

// Tensor maps and shape of one GEMM C[M, N] = A[M, K] . B[N, K]^T.
struct GemmPlan {
  CUtensorMap ma, mb, mb2;
  int M, N, K, bn;
  int bl = 0;  // qb200tc::BLayout of B
  const void *b_ptr = nullptr;  // B and its row pitch (K-major plans), to re-encode for another width
  int ldb = 0;
  int a_box = 128;  // rows per A copy (the A map's box height)
};

// Tile width (64 or 128 columns) used for an M x N output.
int qb200_gemm_bn(int M, int N);
// Builds the tensor maps (row pitches lda, ldb in elements).  0 or an error code.
int qb200_gemm_make_maps(GemmPlan *p, const void *a, const void *b, int M, int N, int K, int lda,
                         int ldb);
// Plan with an MN-major B ([K, N], N contiguous, the upstream Tools/swiglu
// weight layout): C[M, N] = A[M, K] . B.  With b2 (gate|up): the plan's N is
// 2 N, each 128-column tile holds 64 gate and 64 up columns of one output
// block, and the EPI_SWIGLU2 epilogue writes N outputs.  bn: 64 or 128.
// b_rows: rows of B when they are fewer than K (a GEMM whose A is [hi | lo]
// parts of one operand, with GemmArgs::b_kwrap = b_rows / BK); 0: K.
int qb200_gemm_make_maps_mn(GemmPlan *p, const void *a, const void *b, const void *b2, int M, int N,
                            int K, int lda, int ldb, int bn, int b_rows = 0);
// Re-plans a K-major GEMM for tile width bn (64, 128 or 256 columns).
int qb200_gemm_set_bn(GemmPlan *p, int bn);
// Launches the GEMM with epilogue `epi` (qb200tc::Epilogue) on the first g.M
// rows (all planned rows when g.M is 0); g.N/K/n_tiles come from the plan.
int qb200_gemm_run(const GemmPlan &p, int epi, qb200tc::GemmArgs g, cudaStream_t st);
// Row argmax partials (EPI_ARGMAX semantics) by the persistent lm_head kernel:
// one CTA per SM over all tiles, row tiles of a column tile adjacent.
int qb200_gemm_run_argmax(const GemmPlan &p, qb200tc::GemmArgs g, cudaStream_t st);
// Split-K: `splits` CTAs along K write fp32 partial slices into `partial`
// ([splits, M, N]); a reduction sums them in slice order and applies `epi`
// (EPI_F16, EPI_F32, EPI_F32_RES16 or EPI_F16_RES32) into g.out.
int qb200_gemm_run_splitk(const GemmPlan &p, int epi, qb200tc::GemmArgs g, int splits,
                          float *partial, cudaStream_t st);
// out[r] = argmax over the per-tile partials of an EPI_ARGMAX GEMM.
int qb200_argmax_reduce(const float *part_val, const int *part_idx, int n_tiles, int rows, int *out,
                        cudaStream_t st, bool pdl = false);
