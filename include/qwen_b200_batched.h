/*
 * qwen_b200_batched.h - C ABI of the batched decode path (many independent
 * sequences per GPU, each with its own fp16 KV cache) and of its tcgen05
 * tensor-core GEMM.  No upstream counterpart: upstream decodes one sequence
 * at a time (Tools/megakernel/megakernel.cu:1150-1314).  All calls are
 * asynchronous on `stream` (a cudaStream_t) and return 0, or a nonzero code
 * with a message from qwen_b200_last_error() (include/qwen_b200.h).
 */
#ifndef QWEN_B200_BATCHED_H
#define QWEN_B200_BATCHED_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * C[M, N] = A[M, K] . B[N, K]^T on the tensor cores (tcgen05, fp32
 * accumulation in tensor memory), A and B fp16 row-major with row pitch K,
 * followed by one fused epilogue:
 *   0  out fp16 [M, ldo]  = half(C)
 *   1  out fp32 [M, ldo]  = C
 *   2  out fp32 [M, ldo]  = C + float(res fp16 [M, ldo])
 *   3  out fp16 [M, N/2]  : columns (2i, 2i+1) are (gate_i, up_i),
 *                           out[r, i] = half(float(silu_half(half(gate))) * up)
 *                           with the upstream decode kernel's fp16 SiLU steps
 *   4  out fp16 [M, ldo]  = half(C + res fp32 [M, ldo])
 *   5  out int32 [M]      = column of the row maximum of C (lowest on ties);
 *                           workspace of qwen_b200_gemm_argmax_workspace bytes
 * Requirements: N a multiple of 16, K a multiple of 64, 16-byte aligned
 * pointers.
 */
int qwen_b200_gemm_f16(int epilogue, const void *a, const void *b, void *out, const void *res,
                       void *workspace, int M, int N, int K, int ldo, void *stream);
long long qwen_b200_gemm_argmax_workspace(int M, int N);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_BATCHED_H */
