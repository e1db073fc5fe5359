/*
 * qwen_b200.h - C ABI of the B200-native Qwen3-0.6B fp16 greedy-decode engine.
 *
 * Plain C types only: raw device pointers, sizes, a cudaStream_t passed as
 * void*.  No torch types.  The two decode launchers keep the exact symbol
 * names and parameter order of the upstream launchers they replace, so an
 * existing binding (Tools/megakernel/qwen_ops.cpp:9-27) links against this
 * library unchanged.
 *
 * All device pointers must be 16-byte aligned (the weights are streamed with
 * bulk async copies).  All launchers are asynchronous on `stream`; argument
 * errors found on the host are reported through qwen_b200_last_error(), and
 * errors found on the device (a bounded wait that ran out, a misaligned weight
 * pointer in the packed table) through qwen_b200_device_status() and a -1 in
 * the token output.
 *
 * Calls that share a device must not overlap in time: they share one
 * per-device workspace (as the upstream launchers share their static device
 * state, megakernel.cu:714-737).
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-layer weight table, 12 pointers = 96 bytes, 16-byte aligned.
 * Same field order as the upstream struct (megakernel.cu:87-100) and the
 * upstream packer (Model/Qwen06B_architecture.py:177-202). */
typedef struct __attribute__((aligned(16))) LDGLayerWeight {
  const void *input_layernorm_weight;     /* [1024]        */
  const void *q_proj_weight;              /* [2048, 1024]  */
  const void *k_proj_weight;              /* [1024, 1024]  */
  const void *v_proj_weight;              /* [1024, 1024]  */
  const void *q_norm_weight;              /* [128]         */
  const void *k_norm_weight;              /* [128]         */
  const void *o_proj_weight;              /* [1024, 2048]  */
  const void *post_attn_layernorm_weight; /* [1024]        */
  const void *gate_proj_weight;           /* [3072, 1024]  */
  const void *up_proj_weight;             /* [3072, 1024]  */
  const void *down_proj_weight;           /* [1024, 3072]  */
  const void *padding;                    /* zero          */
} LDGLayerWeight;

/* ABI version of the packed table + launcher signatures
 * (Tools/megakernel/qwen_ops.cpp:30-32; Model/Qwen06B_architecture.py:12). */
#define QWEN_B200_ABI_VERSION 2
int qwen_b200_abi_version(void);

/*
 * One greedy decode step: embed(input_token_id) -> num_layers layers at
 * `position` (writes K/V at that position) -> final RMSNorm (fp32 into
 * g_normalized) -> tied lm_head -> argmax into *output_token_id (device int).
 * Replaces launch_ldg_decode_direct, Tools/megakernel/megakernel.cu:1150-1196
 * (same name, same parameters).  Scratch buffers keep the upstream dtypes and
 * sizes (Model/Qwen06B_architecture.py:240-255); after the call g_normalized
 * holds the final normalised hidden (fp32[1024]) and hidden_buffer the last
 * layer's output (fp16[1024]).  stream is a cudaStream_t.
 */
void launch_ldg_decode_direct(
    int input_token_id, int *output_token_id, const void *embed_weight,
    const LDGLayerWeight *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table, void *k_cache,
    void *v_cache, void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
    void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate, void *g_normalized,
    void *block_max_vals, void *block_max_idxs, int num_layers, int position, int max_seq_len,
    float attn_scale, void *stream);

/*
 * num_steps greedy steps from first_token_id at start_position, the produced
 * token fed back on the device; output_log[s] = token produced at step s.
 * One kernel launch for all steps, no host round trip.
 * Replaces launch_ldg_generate_nosync, Tools/megakernel/megakernel.cu:1247-1314
 * (same name, same parameters).
 */
void launch_ldg_generate_nosync(
    int first_token_id, int num_steps, const void *embed_weight,
    const LDGLayerWeight *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table, void *k_cache,
    void *v_cache, void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
    void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate, void *g_normalized,
    void *block_max_vals, void *block_max_idxs, int *output_log, int num_layers,
    int start_position, int max_seq_len, float attn_scale, void *stream);

/*
 * launch_ldg_generate_nosync_static_ws has no counterpart in the reference.
 * Same parameters and results as launch_ldg_generate_nosync, but it never
 * allocates device memory: the kernel's scratch (stage handoff words, attention
 * split partials, per-CTA argmax, status word) is a fixed 618,752-byte array
 * compiled into this library, one copy per device.  It is for callers that
 * cannot have a library allocate behind their back: a server that hands all of
 * HBM to its own pool up front (a cudaMalloc at call time would fail or
 * fragment it), or a latency-critical loop where cudaMalloc's implicit device
 * synchronisation is not acceptable.
 * - The first call on each device does a one-time set-up with that device
 *   current: it looks the array up (cudaGetSymbolAddress, which may load this
 *   library's kernels on the device), clears it (cudaMemset) and waits for the
 *   device (cudaDeviceSynchronize), so that the clear cannot land during the
 *   first launch on a non-blocking stream.  Make that first call before any
 *   stream capture.
 * - The array is sized for at most 256 SMs and 32 attention splits per KV
 *   head; it does not grow with sequence length, steps or layers.  A device
 *   that would need more is rejected with an error; so are the arguments
 *   launch_ldg_generate_nosync rejects.
 * - Calls on one device share the array: calls that overlap in time (other
 *   streams, other host threads without ordering) race and corrupt each other.
 *   Order them, e.g. on one stream.
 * - Device-side failures show as -1 tokens in output_log, and
 *   qwen_b200_device_status() reports their code and detail word.
 * Returns 0 when the launch was issued, else the qwen_b200_last_error() code.
 */
int launch_ldg_generate_nosync_static_ws(
    int first_token_id, int num_steps, const void *embed_weight,
    const LDGLayerWeight *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table, void *k_cache,
    void *v_cache, void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
    void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate, void *g_normalized,
    void *block_max_vals, void *block_max_idxs, int *output_log, int num_layers,
    int start_position, int max_seq_len, float attn_scale, void *stream);

/*
 * qwen_b200_decode_step_dev has no counterpart in the reference (upstream
 * decodes greedily only).  One decode step like launch_ldg_decode_direct,
 * except that the input token is read from device memory (*input_token, int32)
 * when the kernel starts, and, when logits_out is not NULL, the fp32 logits of
 * the step (norm_out @ lm_head^T, [151936]) are written there.  The greedy
 * token still goes to *output_token.  With the sampler of qwen_b200_sample.h
 * writing the next step's *input_token, sampled generation runs without a host
 * round trip per token.  An input token outside [0, 151936) is a device-side
 * error (status code 6, output -1).  Returns 0 when the launch was issued,
 * else the qwen_b200_last_error() code.
 */
int qwen_b200_decode_step_dev(
    const int *input_token, int *output_token, float *logits_out, const void *embed_weight,
    const LDGLayerWeight *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table, void *k_cache,
    void *v_cache, void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
    void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate, void *g_normalized,
    void *block_max_vals, void *block_max_idxs, int num_layers, int position, int max_seq_len,
    float attn_scale, void *stream);

/* Error reporting (no upstream counterpart: the upstream megakernel launchers
 * return void and check no CUDA errors, qwen_ops.cpp:34-165).
 * qwen_b200_last_error: 0 if the calling thread's last launcher call was
 * accepted, else a nonzero code; a message is copied into msg (may be NULL).
 * qwen_b200_device_status: synchronises the device's work submitted so far,
 * then returns the device-side status of the last decode launch on `device`
 * of each workspace (the allocating launchers' and the static one of
 * launch_ldg_generate_nosync_static_ws): 0 = ok, else the first failure's
 * code, with its word ((code, where, CTA) packed as described in the source)
 * in *detail.
 * qwen_b200_workspace_info: whether each of the two per-device workspaces has
 * been set up on `device` (1) or not (0); host-side only, no device call. */
int qwen_b200_last_error(char *msg, int msg_len);
int qwen_b200_device_status(int device, uint64_t *detail);
int qwen_b200_workspace_info(int device, int *alloc_ready, int *static_ready);

/* Wall-clock limit for every bounded wait inside the decode kernel,
 * nanoseconds (default 2e9).  Applies to later launches on all devices. */
void qwen_b200_set_wait_timeout_ns(long long ns);

/* Stage timeline for profiling (no upstream counterpart).  When a device
 * buffer is registered, later decode launches write %globaltimer stamps into
 * it: u64 [cta][step][layer 0..num_layers][40] for as many leading steps as
 * fit in `bytes`.  Events per layer: stage A/B/C/D/E entry, after-wait and
 * warp-0 end at 0..14; producer issue start / cumulative stall ns / issue end
 * at 15..17; CTA-wide end of A/B/C/D/E at 18..22; cumulative ns consumer
 * thread 0 waited for ring data at 23; inside stage B: first K/V pieces
 * landed, scores done, P.V done, split partials stored, combiner's (m, l)
 * gathered at 24..28; SM clock (clock64) in stage E after its wait, after
 * the k loop and at its end at 29..31, and in stage B after the scores, the
 * softmax, the P.V loop and the ring release at 32..35; stage A: ring pieces
 * landed (warp 0) and hidden words gathered (thread 0) at 36..37; producer
 * issue of the layer's last stage-A piece at 38.  Row num_layers: final
 * norm + lm_head
 * entry, after-wait, end, argmax after-wait, end at 0..4.  Tracing adds one
 * barrier per stage.  Pass NULL to turn it off.  The buffer must outlive the
 * launches that use it. */
void qwen_b200_set_trace(void *device_buffer, long long bytes);

/* Failure-detection self test: launches one tiny kernel whose thread waits,
 * with the decode kernel's own bounded-wait routine, on a handoff word that
 * nothing writes.  Returns the status code that wait produced (the timeout
 * code when the bound works).  Synchronous. */
int qwen_b200_selftest_wait_timeout(long long timeout_ns, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_H */
