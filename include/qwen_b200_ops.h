/*
 * qwen_b200_ops.h - C ABI of the standalone RMSNorm and SwiGLU operators
 * (B200 / sm_100a), the replacements of the upstream Tools/rmsnorm and
 * Tools/swiglu torch extensions.
 *
 * Upstream binds those kernels straight to torch (rmsnorm.cu:123-143,
 * swiglu_binding.cpp:5-31); this library puts a plain C ABI underneath the
 * same Python-facing modules (`rmsnorm`, `swiglu_fused`), so the operators are
 * callable without torch.  fp16 only.  Tensors are contiguous row-major;
 * `rows` is the product of all leading dimensions.  Every call is asynchronous
 * on `stream` (a cudaStream_t) and returns 0, or a nonzero code with a message
 * available from qwen_b200_last_error() (include/qwen_b200.h) and nothing
 * launched.
 *
 * Numerics follow the upstream kernels' fp16 rounding points:
 *  - RMSNorm: fp32 sum of squares, inv = rsqrtf(ss / cols + eps), rms = 1/inv;
 *    out = half((x * inv) * w) without residual, and with residual
 *    res = half(x + res) (written back), out = half(res * (inv * w))
 *    (rmsnorm.cuh:17-176).  The fp32 summation order differs from upstream's
 *    block tree, so an output can differ by one fp16 ulp where the fp32
 *    inverse differs in its last bit.
 *  - SwiGLU: every product and every partial sum is rounded to fp16 in
 *    ascending index order, starting from the bias (or 0), exactly as the
 *    upstream loops over c10::Half do (swiglu.cu:89-130, :267-310); results
 *    are bit-identical to upstream's for the same inputs.
 * Weights use the upstream layout: w_gate, w_up [hidden, inter];
 * w_down [inter, hidden].  Requirements: hidden and inter multiples of 8,
 * every pointer 16-byte aligned, hidden <= 8192, inter <= 65536.
 */
#ifndef QWEN_B200_OPS_H
#define QWEN_B200_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* RMSNorm over the last dimension.  residual == NULL selects the simple form
 * (rmsnorm_forward_simple, rmsnorm.cu:44-82); otherwise the fused add form
 * (rmsnorm_forward_fused, rmsnorm.cu:6-42), which updates residual in place.
 * rms receives one float per row.  Replaces rmsnorm_forward, rmsnorm.cu:123-133. */
int qwen_b200_rmsnorm_forward(void *out, float *rms, const void *input, const void *weight,
                              void *residual, long long rows, int cols, float eps, void *stream);

/* out[r, i] = half(silu(g) * u) with g = b_gate[i] + sum_h x[r,h] w_gate[h,i] and
 * u likewise (fp16 steps).  gate_cache / up_cache receive g and u (may be
 * NULL); b_gate / b_up may be NULL (start from 0).
 * Replaces swiglu_forward_cuda, swiglu.cu:316-361. */
int qwen_b200_swiglu_forward(const void *x, const void *w_gate, const void *w_up,
                             const void *b_gate, const void *b_up, void *out, void *gate_cache,
                             void *up_cache, long long rows, int hidden, int inter, void *stream);

/* Bytes of device workspace qwen_b200_swiglu_forward_down(_ex) needs: the
 * SwiGLU activations, rows x inter fp16 (the fp16 chains) or their hi and lo
 * fp16 parts (the tensor-core path), so 4 bytes per element, rounded up to 256,
 * then 12 bytes per element (rounded up to 256) for the tensor-core down
 * projection's fp32 K slices (8 slices while hidden <= 3 inter / 8, fewer
 * or a thread-block cluster reduction otherwise). */
long long qwen_b200_swiglu_forward_down_workspace(long long rows, int inter);

/* out[r, h] = b_down[h] + sum_i s[r,i] w_down[i,h] in fp16 steps, where s is
 * qwen_b200_swiglu_forward's output.  Upstream recomputes s for every output
 * element; the value is the same, so it is computed once here.
 * Replaces swiglu_down_forward_cuda, swiglu.cu:413-464. */
int qwen_b200_swiglu_forward_down(const void *x, const void *w_gate, const void *w_up,
                                  const void *w_down, const void *b_gate, const void *b_up,
                                  const void *b_down, void *out, void *workspace,
                                  long long rows, int hidden, int inter, void *stream);

/* Bytes of device workspace qwen_b200_rmsnorm_swiglu_down(_ex) needs: the
 * normed rows (rows x hidden fp16, rounded up to 256; used when `normed` is
 * NULL), then the activations and K slices as above. */
long long qwen_b200_rmsnorm_swiglu_down_workspace(long long rows, int hidden, int inter);

/* The config-3 chain in one call: normed = rmsnorm(x, norm_weight, eps,
 * residual) into `normed` (may be NULL: kept in the workspace), rms per row,
 * then out = swiglu_forward_down(normed, ...).  Same results as the two
 * separate calls.  No upstream counterpart as one call (upstream: rmsnorm.forward
 * followed by swiglu_fused.forward_down). */
int qwen_b200_rmsnorm_swiglu_down(const void *x, const void *norm_weight, void *residual,
                                  float eps, const void *w_gate, const void *w_up,
                                  const void *w_down, const void *b_gate, const void *b_up,
                                  const void *b_down, void *normed, float *rms, void *out,
                                  void *workspace, long long rows, int hidden, int inter,
                                  void *stream);

/* Dispatching forms of qwen_b200_swiglu_forward_down and
 * qwen_b200_rmsnorm_swiglu_down (same arguments and workspace, plus `mode`);
 * no upstream counterpart as entry points (upstream has only the fp16-chain
 * kernels, swiglu.cu:267-310, :413-464).
 *   mode 1   the fp16 chains above (bit-identical to upstream);
 *   mode 0   tensor cores: gate and up as one tcgen05 GEMM with fp32
 *            accumulation on the [hidden, inter] weights, s = half(g / (1 +
 *            exp(-g)) * u) with g, u in fp32 (biases added in fp32), then the
 *            down projection as a tcgen05 GEMM (fp32 accumulation, K split
 *            inside a thread-block cluster), out = half(acc + b_down).  Needs
 *            hidden and inter multiples of 64.  Closer to an fp32 evaluation
 *            than upstream's fp16 accumulation, not bit-identical to it;
 *   mode -1  tensor cores for rows >= 64 when the shape allows, else the chains. */
int qwen_b200_swiglu_forward_down_ex(const void *x, const void *w_gate, const void *w_up,
                                     const void *w_down, const void *b_gate, const void *b_up,
                                     const void *b_down, void *out, void *workspace,
                                     long long rows, int hidden, int inter, int mode, void *stream);
int qwen_b200_rmsnorm_swiglu_down_ex(const void *x, const void *norm_weight, void *residual,
                                     float eps, const void *w_gate, const void *w_up,
                                     const void *w_down, const void *b_gate, const void *b_up,
                                     const void *b_down, void *normed, float *rms, void *out,
                                     void *workspace, long long rows, int hidden, int inter, int mode,
                                     void *stream);

/* Synchronises the current device, then returns 0 if no operator kernel has
 * given up a bounded wait since the last call, else the code it recorded
 * (and the packed detail in *detail); the record is cleared. */
int qwen_b200_ops_status(uint64_t *detail);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_OPS_H */
