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
 * k_splits > 1 (epilogues 0, 1, 2, 4) cuts K into that many slices computed by
 * separate CTAs and summed in slice order before the epilogue: with a
 * workspace (k_splits * M * N * 4 bytes) through fp32 partials in global
 * memory and a reduction kernel; with workspace NULL (k_splits <= 8) inside a
 * thread-block cluster of the k_splits CTAs of a tile (partial tiles added
 * through distributed shared memory, one launch).  Both give the same bits.
 * Requirements: N a multiple of 16, K a multiple of 64, 16-byte aligned
 * pointers.
 */
int qwen_b200_gemm_f16(int epilogue, const void *a, const void *b, void *out, const void *res,
                       void *workspace, int M, int N, int K, int ldo, int k_splits, void *stream);
/* The same with the tile width chosen by the caller: bn = 64, 128 or 256
 * output columns per CTA (0: by output size, as qwen_b200_gemm_f16); the
 * argmax epilogue takes the default only.  No upstream counterpart. */
int qwen_b200_gemm_f16_tiled(int epilogue, const void *a, const void *b, void *out, const void *res,
                             void *workspace, int M, int N, int K, int ldo, int k_splits, int bn,
                             void *stream);
long long qwen_b200_gemm_argmax_workspace(int M, int N);

/*
 * Vocabulary-sharded tied lm_head (no upstream counterpart; upstream computes
 * the full 151,936-row lm_head on one GPU, megakernel.cu:1001-1144).
 * qwen_b200_lmhead_argmax: for hidden fp16 [rows, 1024] and this shard's rows
 * of the embedding, weight fp16 [vocab_rows, 1024], writes per row the largest
 * logit (fp32, tensor-core dot products with fp32 accumulation) and its index
 * + index_offset (lowest among equal values).  Workspace:
 * qwen_b200_lmhead_argmax_workspace bytes.  The dot product of one vocabulary
 * row does not depend on the shard it sits in, so shards picked together give
 * the single-GPU argmax exactly.
 * qwen_b200_argmax_pick: vals / idxs [world, rows] (every shard's pair, e.g.
 * after an all-gather) -> out[r], the largest value's index, lowest on ties.
 */
/*
 * Exchange of the shards' (max, index) pairs through peer memory instead of
 * an all-gather (no upstream counterpart).  Every rank owns a receive buffer
 * of qwen_b200_peer_buffer_bytes(world, rows) bytes made by
 * qwen_b200_peer_buffer_create (cudaMalloc'd, cleared, with its 64-byte CUDA
 * IPC handle written to ipc_handle); ranks share the handles (e.g. through
 * torch.distributed) and open each other's buffers with
 * qwen_b200_peer_buffer_open (a pointer valid on this device, peer access
 * enabled lazily); qwen_b200_peer_buffer_close releases an opened buffer
 * (opened = 1) or frees an own one (opened = 0) -- close the peers' mappings
 * of a buffer before it is freed.
 * qwen_b200_argmax_exchange: rank `rank` stores its pair of each row, tagged
 * with `epoch`, into every rank's buffer (peer_bufs[q]: rank q's buffer as
 * seen from this device, peer_bufs[rank] its own) with plain 8-byte stores at
 * system scope, then waits until every rank's pairs of this epoch are in its
 * own buffer and writes out[r] = the largest value's index (lowest among equal
 * values).  epoch: nonzero, one more per call, the same on every rank;
 * consecutive calls use the two halves of the buffers in turn.  Each wait is
 * bounded by timeout_ns (<= 0: 2 s): a rank whose pairs never come gives -1
 * and, when status is not NULL, (1 << 32 | rank << 24 | row) in *status.
 * world <= 8.
 */
long long qwen_b200_peer_buffer_bytes(int world, int rows);
int qwen_b200_peer_buffer_create(long long bytes, void **ptr, void *ipc_handle);
int qwen_b200_peer_buffer_open(const void *ipc_handle, void **ptr);
int qwen_b200_peer_buffer_close(void *ptr, int opened);
int qwen_b200_argmax_exchange(const float *val, const int *idx, void *const *peer_bufs, int world,
                              int rank, int rows, unsigned epoch, long long timeout_ns, int *out,
                              unsigned long long *status, void *stream);

long long qwen_b200_lmhead_argmax_workspace(int rows, int vocab_rows);
int qwen_b200_lmhead_argmax(const void *hidden, const void *weight, int rows, int vocab_rows,
                            long long index_offset, float *out_val, int *out_idx, void *workspace,
                            void *stream);
int qwen_b200_argmax_pick(const float *vals, const int *idxs, int world, int rows, int *out,
                          void *stream);

/* Weights of one layer for the batched path (all fp16, 16-byte aligned):
 * w_qkv [4096, 1024] = q_proj | k_proj | v_proj rows; w_gu [6144, 1024] with
 * rows 2i = gate_proj[i], 2i+1 = up_proj[i]; w_o [1024, 2048] and
 * w_down [1024, 3072] as in the checkpoint; norms [1024] / [128]. */
typedef struct QwenBatchedLayer {
  const void *input_norm, *w_qkv, *q_norm, *k_norm, *w_o, *post_norm, *w_gu, *w_down;
} QwenBatchedLayer;

/* Bytes of device workspace for up to max_rows rows per step. */
long long qwen_b200_batched_workspace(int max_rows, int max_seq);

/* Plans batched decode over `num_seqs` sequences: k_pool / v_pool are fp16
 * [num_seqs][num_layers][8][max_seq][128] (the upstream per-sequence cache
 * layout, Model/Qwen06B_architecture.py:233-237, stacked); embed is the tied
 * embedding / lm_head [151936, 1024]; cos/sin tables [max_seq, 128] fp16.
 * `layers` is a host array (copied).  Builds every tensor map once. */
int qwen_b200_batched_create(void **handle, const QwenBatchedLayer *layers, int num_layers,
                             const void *embed, const void *final_norm, const void *cos_table,
                             const void *sin_table, void *k_pool, void *v_pool, int num_seqs,
                             int max_seq, int max_rows, void *workspace,
                             long long workspace_bytes);

/* Paged KV pools (no upstream counterpart; upstream has one contiguous
 * 2048-token cache, Model/Qwen06B_architecture.py:21, :233-237): k_pool /
 * v_pool are fp16 [num_pages][num_layers][8][128][128], pages of 128 tokens
 * shared by all sequences; page_table is a device int32
 * [num_seqs][max_pages_per_seq] array owned and updated by the caller (entry
 * = the page holding positions [128 i, 128 i + 128) of that sequence, or -1).
 * A step reads the table when it runs: pages must be mapped before a step
 * touches their positions (an unmapped page is a recorded error, code 3, and
 * the access is skipped).  max_seq may exceed 2048 (up to 65536) as long as
 * max_pages_per_seq * 128 >= max_seq and the RoPE tables have max_seq rows.
 * Everything else as qwen_b200_batched_create. */
int qwen_b200_batched_create_paged(void **handle, const QwenBatchedLayer *layers, int num_layers,
                                   const void *embed, const void *final_norm, const void *cos_table,
                                   const void *sin_table, void *k_pool, void *v_pool, int num_pages,
                                   const int *page_table, int max_pages_per_seq, int num_seqs,
                                   int max_seq, int max_rows, void *workspace,
                                   long long workspace_bytes);

/* One greedy step for `rows` rows (device int32 arrays): row r is sequence
 * seq_ids[r] at position positions[r], fed token tokens_in[r]; K/V of that
 * position are appended to its cache, the argmax token is written to
 * tokens_out[r], and when norm_out is not NULL the final RMSNorm output
 * (fp32 [rows, 1024], the logits tap) as well.  (sequence, position) pairs
 * must be distinct within a step; one sequence may occupy several rows at
 * consecutive positions (parallel prefill): every row's K/V is appended
 * before the step's attention, so the row at position p attends to positions
 * 0..p including those written by the same step.  max_position must be >=
 * every positions[r] and < max_seq (it sizes the attention grid).  No host
 * synchronisation and no allocation. */
int qwen_b200_batched_step(void *handle, int rows, const int *seq_ids, const int *positions,
                           const int *tokens_in, int *tokens_out, float *norm_out,
                           int max_position, float attn_scale, void *stream);

/* The step above, with the tied lm_head's fp32 logits written to
 * logits[r * ld + v] (ld >= 151936 and a multiple of 4, 16-byte aligned)
 * instead of the fused argmax; feeds the sampler of qwen_b200_sample.h.  No
 * upstream counterpart (upstream decodes greedily only). */
int qwen_b200_batched_step_logits(void *handle, int rows, const int *seq_ids, const int *positions,
                                  const int *tokens_in, float *logits, long long ld, float *norm_out,
                                  int max_position, float attn_scale, void *stream);

/* Synchronises the device; returns 0 if no batched kernel has recorded an
 * error since the last call, else its code (1: a bounded wait gave up, 2: a
 * token id outside the vocabulary, 3: a sequence id or position outside the
 * caches; the offending row's access was skipped), and clears the record. */
int qwen_b200_batched_status(void *handle, uint64_t *detail);
void qwen_b200_batched_destroy(void *handle);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_BATCHED_H */
