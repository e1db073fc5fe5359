/*
 * CPU oracle for the Qwen3-0.6B fp16 greedy-decode path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm may load this library, and only
 * as the checker (or as the timed CPU restatement of the reference).  The
 * product path never calls it.
 *
 * This is a plain-C restatement of the upstream project's algorithm, with the
 * upstream fp16 rounding points reproduced exactly.  Citations are to files of
 * the upstream project (emmanuelalo52/QWEN0.6B):
 *
 *   decode step ........ Tools/megakernel/megakernel.cu:763-920 (body),
 *                        :1001-1144 (lm_head + argmax)
 *   RMSNorm operator ... Tools/rmsnorm/rmsnorm.cuh:17-176
 *   SwiGLU operator .... Tools/swiglu/swiglu.cu:60-130, :267-310
 *
 * What is and is not reproduced bit for bit:
 *   - every fp32 -> fp16 rounding (RNE) the upstream code performs, and the
 *     association of every elementwise fp32 product, is reproduced;
 *   - half-precision arithmetic (__hadd, __hmul, c10::Half operators) is
 *     emulated as fp32 arithmetic rounded to fp16, which is exact because
 *     binary32 has at least 2*11+2 significand bits;
 *   - the *order* of fp32 summations in dot products differs from the GPU's
 *     lane-strided warp trees, and rsqrtf/expf/exp2f come from the C library
 *     instead of CUDA's.  Results therefore agree with the upstream kernels to
 *     fp32 rounding, not bit for bit (except the fp16-accumulating SwiGLU
 *     operator, whose sequential loop order is reproduced exactly).
 *
 * Compiled with -ffp-contract=off so that each written expression is evaluated
 * exactly as IEEE single-precision operations; dot products use explicit
 * fmaf() in 16 independent partial sums.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define H 1024
#define I_SZ 3072
#define NQ 16
#define NKV 8
#define HD 128
#define QS (NQ * HD)
#define KVS (NKV * HD)
#define VOCAB 151936
#define EPS 1e-6f

typedef uint16_t half_t;

static inline float h2f(half_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}
static inline half_t f2h(float f) {
  _Float16 x = (_Float16)f;
  half_t h;
  memcpy(&h, &x, 2);
  return h;
}
static inline float rh(float f) { return (float)(_Float16)f; }

static void set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* fp32 dot of an fp16 row with an fp32 vector (16 partial sums, then a fixed
 * pairwise tree).  Stands in for the warp-level reductions of
 * megakernel.cu:270-290, :593-606, :651-667, :689-702, :1034-1070. */
static float dot_h_f(const half_t *w, const float *x, int n) {
  float acc[16];
  for (int j = 0; j < 16; j++) acc[j] = 0.f;
  for (int k = 0; k < n; k += 16) {
    float wf[16];
    for (int j = 0; j < 16; j++) wf[j] = h2f(w[k + j]);
    for (int j = 0; j < 16; j++) acc[j] = fmaf(wf[j], x[k + j], acc[j]);
  }
  for (int s = 8; s > 0; s >>= 1)
    for (int j = 0; j < s; j++) acc[j] += acc[j + s];
  return acc[0];
}

static void gemv(const half_t *W, const float *x, float *y, int rows, int k) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < rows; m++) y[m] = dot_h_f(W + (size_t)m * k, x, k);
}

static float sumsq(const float *x, int n) {
  float acc[16];
  for (int j = 0; j < 16; j++) acc[j] = 0.f;
  for (int k = 0; k < n; k += 16)
    for (int j = 0; j < 16; j++) acc[j] = fmaf(x[k + j], x[k + j], acc[j]);
  for (int s = 8; s > 0; s >>= 1)
    for (int j = 0; j < s; j++) acc[j] += acc[j + s];
  return acc[0];
}

static float rsqrt_ref(float x) { return 1.0f / sqrtf(x); }

/* Half-precision SiLU of megakernel.cu:141-154: every step is an fp16 op. */
float oracle_silu_half(float xf) {
  float x = rh(xf);
  float log2e = rh(1.44269504088896340736f);
  float t = rh(-x * log2e);          /* __hmul(__hneg(x), LOG2E_HALF)      */
  float e = rh(exp2f(t));            /* ptx_hexp2: half(exp2f(float(x)))    */
  float d = rh(1.0f + e);            /* __hadd(1, e)                        */
  float r = rh(1.0f / d);            /* ptx_hrcp: half(1.0f / float(x))     */
  return rh(x * r);                  /* __hmul(x, r)                        */
}

/* q/k head RMSNorm + rotate-half RoPE with fp16 tables, megakernel.cu:345-390
 * (K) and :395-434 (Q).  `out` receives the fp16-rounded rotated head. */
static void norm_rope_head(const half_t *src, const half_t *nw, const half_t *cosp,
                           const half_t *sinp, half_t *out) {
  float v[HD], ss = 0.f;
  for (int i = 0; i < HD; i++) {
    float f = h2f(src[i]);
    ss = fmaf(f, f, ss);
  }
  float inv = rsqrt_ref(ss / (float)HD + 1e-6f);
  for (int i = 0; i < HD; i++) v[i] = h2f(src[i]) * inv * h2f(nw[i]); /* (x*inv)*w */
  for (int i = 0; i < HD; i++) {
    int ri = i < HD / 2 ? i : i - HD / 2;
    float c = h2f(cosp[ri]), s = h2f(sinp[ri]);
    float r;
    if (i < HD / 2) r = v[i] * c - v[i + HD / 2] * s;
    else r = v[i - HD / 2] * s + v[i] * c;
    out[i] = f2h(r);
  }
}

/*
 * One greedy decode step (megakernel.cu:763-920 then :1001-1144).
 *
 * layer_ptrs: num_layers*11 host pointers in LDGLayerWeight order
 * (megakernel.cu:87-100): in_norm, q, k, v, q_norm, k_norm, o, post_norm,
 * gate, up, down.  k_cache/v_cache: [num_layers][8][max_seq_len][128] fp16,
 * updated in place at `position`.  Optional outputs (may be NULL):
 * hidden_out fp16[1024], norm_out f32[1024], logits f32[151936],
 * attn_dbg fp16[num_layers*2048] (per-layer attention output),
 * qkv_dbg fp16[num_layers*4096] (per-layer rotated q | rotated k | raw v).
 * Returns the argmax token (lowest index among equal maxima), or -1 on a bad
 * argument.
 */
int oracle_decode_step(int token, int position, const half_t *embed,
                       const half_t *const *layer_ptrs, int num_layers,
                       const half_t *final_norm, const half_t *lm_head,
                       const half_t *cos_table, const half_t *sin_table,
                       half_t *k_cache, half_t *v_cache, int max_seq_len, float attn_scale,
                       half_t *hidden_out, float *norm_out, float *logits,
                       half_t *attn_dbg, half_t *qkv_dbg, int nthreads) {
  if (token < 0 || token >= VOCAB || position < 0 || position >= max_seq_len || num_layers < 1)
    return -1;
  set_threads(nthreads);
  half_t hidden[H];
  memcpy(hidden, embed + (size_t)token * H, sizeof(hidden));    /* :790-796 */

  float xf[QS > I_SZ ? QS : I_SZ];
  float qkv[QS + 2 * KVS];
  half_t qh[QS], kh[KVS], vh[KVS], attn[QS];
  float act[H], tmp[I_SZ], gate[I_SZ], up[I_SZ];
  const half_t *cosp = cos_table + (size_t)position * HD;
  const half_t *sinp = sin_table + (size_t)position * HD;
  const size_t layer_stride = (size_t)NKV * max_seq_len * HD;

  for (int l = 0; l < num_layers; l++) {
    const half_t *const *w = layer_ptrs + (size_t)l * 11;
    /* Input RMSNorm, :806-847: s_norm = half(h * (inv * w)). */
    for (int i = 0; i < H; i++) tmp[i] = h2f(hidden[i]);
    float inv = rsqrt_ref(sumsq(tmp, H) / (float)H + EPS);
    for (int i = 0; i < H; i++) xf[i] = rh(tmp[i] * (inv * h2f(w[0][i])));
    /* Fused QKV GEMV, :242-291: outputs rounded to fp16. */
    gemv(w[1], xf, qkv, QS, H);
    gemv(w[2], xf, qkv + QS, KVS, H);
    gemv(w[3], xf, qkv + QS + KVS, KVS, H);
    for (int i = 0; i < QS; i++) qh[i] = f2h(qkv[i]);
    for (int i = 0; i < KVS; i++) kh[i] = f2h(qkv[QS + i]);
    for (int i = 0; i < KVS; i++) vh[i] = f2h(qkv[QS + KVS + i]);

    /* K norm + RoPE into the cache, V copied raw, :339-390. */
    half_t *lkc = k_cache + (size_t)l * layer_stride;
    half_t *lvc = v_cache + (size_t)l * layer_stride;
    half_t krot[KVS], qrot[QS];
    for (int h = 0; h < NKV; h++) {
      norm_rope_head(kh + h * HD, w[5], cosp, sinp, krot + h * HD);
      memcpy(lkc + (size_t)h * max_seq_len * HD + (size_t)position * HD, krot + h * HD, HD * 2);
      memcpy(lvc + (size_t)h * max_seq_len * HD + (size_t)position * HD, vh + h * HD, HD * 2);
    }
    /* Q norm + RoPE, :395-434. */
    for (int h = 0; h < NQ; h++) norm_rope_head(qh + h * HD, w[4], cosp, sinp, qrot + h * HD);
    if (qkv_dbg) {
      half_t *d = qkv_dbg + (size_t)l * (QS + 2 * KVS);
      memcpy(d, qrot, QS * 2);
      memcpy(d + QS, krot, KVS * 2);
      memcpy(d + QS + KVS, vh, KVS * 2);
    }

    /* Decode attention over cache_len = position+1 tokens, :457-552:
     * fp32 scores * attn_scale, softmax with expf, out = half(acc * (1/sum)). */
    int clen = position + 1;
#pragma omp parallel for schedule(static)
    for (int qhd = 0; qhd < NQ; qhd++) {
      int g = qhd / (NQ / NKV);
      const half_t *kc = lkc + (size_t)g * max_seq_len * HD;
      const half_t *vc = lvc + (size_t)g * max_seq_len * HD;
      float qf[HD], acc[HD];
      float *sc = (float *)malloc(sizeof(float) * (size_t)clen);
      for (int i = 0; i < HD; i++) qf[i] = h2f(qrot[qhd * HD + i]);
      float mx = -INFINITY;
      for (int t = 0; t < clen; t++) {
        float s = dot_h_f(kc + (size_t)t * HD, qf, HD) * attn_scale;
        sc[t] = s;
        if (s > mx) mx = s;
      }
      float sum = 0.f;
      for (int i = 0; i < HD; i++) acc[i] = 0.f;
      for (int t = 0; t < clen; t++) {
        float p = expf(sc[t] - mx);
        sum += p;
        const half_t *vr = vc + (size_t)t * HD;
        for (int i = 0; i < HD; i++) acc[i] = fmaf(p, h2f(vr[i]), acc[i]);
      }
      float invs = sum > 0.f ? 1.0f / sum : 0.f;
      for (int i = 0; i < HD; i++) attn[qhd * HD + i] = f2h(acc[i] * invs);
      free(sc);
    }
    if (attn_dbg) memcpy(attn_dbg + (size_t)l * QS, attn, QS * 2);

    /* o_proj + fp32 residual (not rounded), :585-610 and :868-872. */
    for (int i = 0; i < QS; i++) xf[i] = h2f(attn[i]);
    gemv(w[6], xf, act, H, QS);
    for (int i = 0; i < H; i++) act[i] = act[i] + h2f(hidden[i]);

    /* Post-attention RMSNorm from fp32 act, :614-638:
     * s_act = half(float(half(act)) * rstd * w). */
    float rstd = rsqrt_ref(sumsq(act, H) / (float)H + EPS);
    for (int i = 0; i < H; i++) xf[i] = rh(rh(act[i]) * rstd * h2f(w[7][i]));

    /* gate/up + half SiLU * up (fp32 product, stored fp32), :640-675. */
    gemv(w[8], xf, gate, I_SZ, H);
    gemv(w[9], xf, up, I_SZ, H);
    for (int i = 0; i < I_SZ; i++) tmp[i] = rh(oracle_silu_half(gate[i]) * up[i]);
    /* down + residual, rounded to fp16 hidden, :679-707.  tmp holds
     * half(inter) because the kernel rounds inter when staging it in smem. */
    float dn[H];
    gemv(w[10], tmp, dn, H, I_SZ);
    for (int i = 0; i < H; i++) hidden[i] = f2h(dn[i] + act[i]);
  }

  /* Final RMSNorm to fp32, :890-919: norm = (h * inv) * w. */
  float hf[H], nrm[H];
  for (int i = 0; i < H; i++) hf[i] = h2f(hidden[i]);
  float inv = rsqrt_ref(sumsq(hf, H) / (float)H + EPS);
  for (int i = 0; i < H; i++) nrm[i] = hf[i] * inv * h2f(final_norm[i]);
  if (hidden_out) memcpy(hidden_out, hidden, sizeof(hidden));
  if (norm_out) memcpy(norm_out, nrm, sizeof(nrm));

  /* Tied lm_head GEMV + argmax, :1001-1144. */
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * VOCAB);
  gemv(lm_head, nrm, lg, VOCAB, H);
  int best = 0;
  for (int r = 1; r < VOCAB; r++)
    if (lg[r] > lg[best]) best = r;
  if (!logits) free(lg);
  return best;
}

/* fp32 tied-lm_head logits + argmax of fp16 hidden rows (vocab-sharded
 * lm_head check): logits[b][r] = sum_k float(E[r,k]) * float(x[b,k]).
 * rows [row0,row1) of E only; out_idx[b] is a global row index. */
void oracle_lm_head_argmax(const half_t *x, int batch, const half_t *E, int row0, int row1,
                           float *out_val, int *out_idx, int nthreads) {
  set_threads(nthreads);
  for (int b = 0; b < batch; b++) {
    float xf[H];
    for (int k = 0; k < H; k++) xf[k] = h2f(x[(size_t)b * H + k]);
    float bv = -INFINITY;
    int bi = -1;
#pragma omp parallel
    {
      float lv = -INFINITY;
      int li = -1;
#pragma omp for schedule(static)
      for (int r = row0; r < row1; r++) {
        float v = dot_h_f(E + (size_t)r * H, xf, H);
        if (v > lv || li < 0) { lv = v; li = r; }
      }
#pragma omp critical
      {
        if (li >= 0 && (lv > bv || (lv == bv && li < bi) || bi < 0)) { bv = lv; bi = li; }
      }
    }
    out_val[b] = bv;
    out_idx[b] = bi;
  }
}

/*
 * RMSNorm operator, Tools/rmsnorm/rmsnorm.cuh:17-119 (fused add, residual
 * updated in place with half adds) and :125-176 (simple).  residual == NULL
 * selects the simple kernel, as rmsnorm.cu:123-133 does.  rms_out[row] gets
 * 1/inv_rms.
 */
void oracle_rmsnorm(const half_t *input, const half_t *weight, half_t *residual, half_t *out,
                    float *rms_out, int rows, int cols, float eps) {
  for (int r = 0; r < rows; r++) {
    const half_t *x = input + (size_t)r * cols;
    half_t *o = out + (size_t)r * cols;
    float ss = 0.f;
    if (residual) {
      /* Elements below (cols/4)*4 take the vector path (rmsnorm.cuh:47-62,
       * :82-93), the rest the scalar remainder path (:64-69, :95-99), which
       * squares the unrounded sum and normalises as (res*inv)*w. */
      const int vec_end = (cols / 4) * 4;
      half_t *res = residual + (size_t)r * cols;
      for (int i = 0; i < cols; i++) {
        const float sum = h2f(x[i]) + h2f(res[i]);
        res[i] = f2h(sum);                                  /* __hadd2 / static_cast<T> */
        const float f = i < vec_end ? h2f(res[i]) : sum;
        ss = fmaf(f, f, ss);
      }
      float inv = rsqrt_ref(ss / (float)cols + eps);
      rms_out[r] = 1.0f / inv;
      for (int i = 0; i < cols; i++)
        o[i] = i < vec_end ? f2h(h2f(res[i]) * (inv * h2f(weight[i])))
                           : f2h(h2f(res[i]) * inv * h2f(weight[i]));
    } else {
      for (int i = 0; i < cols; i++) {
        float f = h2f(x[i]);
        ss = fmaf(f, f, ss);
      }
      float inv = rsqrt_ref(ss / (float)cols + eps);
      rms_out[r] = 1.0f / inv;
      for (int i = 0; i < cols; i++) o[i] = f2h(h2f(x[i]) * inv * h2f(weight[i]));
    }
  }
}

/* c10::Half arithmetic: every operator rounds its fp32 result to fp16. */
static inline float hadd_c10(float a, float b) { return rh(a + b); }
static inline float hmul_c10(float a, float b) { return rh(a * b); }
/* swiglu.cu:60-63 instantiated for c10::Half: x / (1 + expf(-x)) in fp32,
 * rounded to fp16 on return. */
static inline float silu_c10(float x) { return rh(x / (1.0f + expf(-x))); }

/*
 * SwiGLU forward, Tools/swiglu/swiglu.cu:89-130 with T = c10::Half:
 * out[row, i] = silu(x.Wg[:,i]) * (x.Wu[:,i]), fp16 accumulation in h order
 * starting from the bias (swiglu.cu:111-112; 0 when bg / bu are NULL).
 * Weights use the upstream [H, I] layout.  gate_cache / up_cache may be NULL.
 */
void oracle_swiglu_forward(const half_t *x, const half_t *wg, const half_t *wu, const half_t *bg,
                           const half_t *bu, int rows, int hidden, int inter, half_t *out,
                           half_t *gate_cache, half_t *up_cache, int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static) collapse(2)
  for (int r = 0; r < rows; r++) {
    for (int i = 0; i < inter; i++) {
      float g = bg ? h2f(bg[i]) : 0.f, u = bu ? h2f(bu[i]) : 0.f;
      for (int h = 0; h < hidden; h++) {
        float xv = h2f(x[(size_t)r * hidden + h]);
        g = hadd_c10(g, hmul_c10(xv, h2f(wg[(size_t)h * inter + i])));
        u = hadd_c10(u, hmul_c10(xv, h2f(wu[(size_t)h * inter + i])));
      }
      size_t o = (size_t)r * inter + i;
      out[o] = f2h(hmul_c10(silu_c10(g), u));
      if (gate_cache) gate_cache[o] = f2h(g);
      if (up_cache) up_cache[o] = f2h(u);
    }
  }
}

/*
 * Fused SwiGLU + down, Tools/swiglu/swiglu.cu:267-310 with T = c10::Half:
 * out[row, h] = sum_i half(silu(g_i) * u_i) * Wd[i, h], all in fp16 steps.
 * The gate/up values do not depend on the output column, so they are
 * computed once per row here; the arithmetic is the same sequence of fp16
 * operations the upstream kernel repeats per column.
 */
void oracle_swiglu_forward_down(const half_t *x, const half_t *wg, const half_t *wu,
                                const half_t *wd, const half_t *bg, const half_t *bu,
                                const half_t *bd, int rows, int hidden, int inter, half_t *out,
                                int nthreads) {
  set_threads(nthreads);
  float *so = (float *)malloc(sizeof(float) * (size_t)rows * inter);
#pragma omp parallel for schedule(static) collapse(2)
  for (int r = 0; r < rows; r++) {
    for (int i = 0; i < inter; i++) {
      float g = bg ? h2f(bg[i]) : 0.f, u = bu ? h2f(bu[i]) : 0.f;
      for (int h = 0; h < hidden; h++) {
        float xv = h2f(x[(size_t)r * hidden + h]);
        g = hadd_c10(g, hmul_c10(xv, h2f(wg[(size_t)h * inter + i])));
        u = hadd_c10(u, hmul_c10(xv, h2f(wu[(size_t)h * inter + i])));
      }
      so[(size_t)r * inter + i] = hmul_c10(silu_c10(g), u);
    }
  }
#pragma omp parallel for schedule(static) collapse(2)
  for (int r = 0; r < rows; r++) {
    for (int h = 0; h < hidden; h++) {
      float acc = bd ? h2f(bd[h]) : 0.f;
      for (int i = 0; i < inter; i++)
        acc = hadd_c10(acc, hmul_c10(so[(size_t)r * inter + i], h2f(wd[(size_t)i * hidden + h])));
      out[(size_t)r * hidden + h] = f2h(acc);
    }
  }
  free(so);
}
