/* Token sampling on logits rows: temperature, top-k, top-p (B200, sm_100a).
 *
 * No upstream counterpart: upstream decodes greedily only (README.md:691-692,
 * Tools/megakernel/megakernel.cu:1114-1144).  The filtering follows the
 * Hugging Face logits warpers that upstream's benchmark drives through
 * generate() (transformers TemperatureLogitsWarper, TopKLogitsWarper,
 * TopPLogitsWarper, applied in that order):
 *   z = logits / temperature;
 *   top-k: drop every z below the k-th largest z (ties with it are kept);
 *   top-p: over the softmax of the surviving z, drop every token whose
 *          strictly larger tokens already hold at least top_p of the mass
 *          (the largest token is always kept).  Equal values are kept or
 *          dropped together; transformers cuts inside a group of equal values
 *          in the order of an unstable sort.
 * The token is then drawn from the softmax of the surviving z with the
 * Gumbel-max rule, argmax(z_i - log(-log u_i)), u_i from a Philox-4x32-10
 * counter stream keyed by (seed, offset, row, i): the same arguments give the
 * same tokens.  temperature == 0 or top_k == 1 gives the greedy argmax
 * (lowest index among equal maxima).
 *
 * Thresholds are exact: radix selection on the order-preserving 32-bit key of
 * each z (count histograms for top-k, softmax-mass histograms for top-p), one
 * CTA per row.
 */
#ifndef QWEN_B200_SAMPLE_H
#define QWEN_B200_SAMPLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* logits: fp32 [rows][ld] (device), the first `vocab` columns used; ld >= vocab.
 * temperature >= 0; top_k >= 0 (0 = off); 0 < top_p <= 1 (1 = off).
 * Random stream of row r: counter (element group, row_seq[r], offset +
 * row_pos[r]) under key `seed`; row_seq / row_pos are optional device int32
 * [rows] (NULL: r and 0), so a batched caller can key each draw by (sequence,
 * position) and get the same draw whatever the batch composition.
 * out_tokens: int32 [rows] (device).  kept_min (optional, may be NULL): float
 * [rows], the smallest z kept by the filters (z = logits / temperature); the
 * kept set is {i : z_i >= kept_min[row]}.  stream is a cudaStream_t.
 * Returns 0 when the launch was issued, else a code with the message in
 * qwen_b200_last_error(). */
int qwen_b200_sample(const float *logits, long long ld, int rows, int vocab, float temperature,
                     int top_k, float top_p, unsigned long long seed, unsigned long long offset,
                     const int *row_seq, const int *row_pos, int *out_tokens, float *kept_min,
                     void *stream);

/* Path choice: with the default (1), calls of at most 96 rows of at most
 * 8 x 19,200 logits hold each row in the shared memory of a cluster of 8 CTAs
 * (read once, the selection run on the elements of a window that provably
 * contains the kept set); other calls use one CTA per row; 0 forces one CTA
 * per row.  Both give the same kept set and
 * the same draws.  Process-wide; for tests and measurements. */
void qwen_b200_sample_set_cluster(int enable);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_SAMPLE_H */
