// Persistent batch-1 greedy decode kernel for Qwen3-0.6B on B200 (sm_100a),
// plus the C-ABI launchers that replace the upstream
// launch_ldg_decode_direct / launch_ldg_generate_nosync
// (Tools/megakernel/megakernel.cu:1150-1196, :1247-1314).
//
// Design (one CTA per SM, cooperative launch so all CTAs are co-resident):
//
//  * A producer warp streams this CTA's slice of every weight matrix (and of
//    the KV cache for its attention work) into a 16-slot shared-memory ring
//    with bulk async copies (cp.async.bulk, completion on mbarriers, L2
//    evict-first).  Weights do not depend on activations, so the producer runs
//    ahead across stage boundaries, layers and decode steps; HBM keeps
//    streaming while the consumer warps wait for the previous stage.
//  * 16 consumer warps compute each stage on the bytes already in shared
//    memory.  Per layer: A input RMSNorm + QKV GEMV, B q/k RMSNorm + RoPE +
//    split-KV GQA attention (2 q heads share one K/V read), C o_proj +
//    residual, D post-attention RMSNorm + gate/up GEMV + SiLU*mul, E down GEMV
//    + residual.  After the last layer: F final RMSNorm + tied lm_head GEMV +
//    per-CTA argmax, G global argmax; the token is fed back on the device.
//  * Stages hand activations to each other through 8-byte words that carry
//    their own epoch (payload 32 bits | epoch 32 bits).  A reader polls the
//    words it needs; there is no separate grid barrier, no fence and no
//    counter on the critical path.
//  * Every wait is bounded (wall clock via %globaltimer) and any failure is
//    reported in a device status word and a -1 token; exits are decided
//    uniformly per CTA with bar.red.or so no named barrier is left short.
//
// The upstream fp16 rounding points are reproduced exactly (RMSNorm outputs,
// q/k/v, rotated q/k, attention output, hidden rounded to fp16; act,
// mlp_inter, norm_out kept fp32; half-precision SiLU); only the order of fp32
// summations differs from the upstream warp trees.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "ptx.cuh"
#include "qwen_b200.h"

namespace qb200 {

constexpr int H = 1024, IM = 3072, NQ = 16, NKV = 8, HD = 128;
constexpr int QS = NQ * HD, KVS = NKV * HD, QKV_ROWS = QS + 2 * KVS;
constexpr int VOCAB = 151936;
constexpr float RMS_EPS = 1e-6f;

constexpr int NCW = 16;               // consumer warps
constexpr int NCT = NCW * 32;         // consumer threads
constexpr int NTHREADS = NCT + 32;    // + one producer warp
constexpr int SLOT_BYTES = 12288;     // 6 rows of K=1024, 3 of 2048, 2 of 3072, 48 KV tokens
constexpr int NSLOTS = 16;
constexpr int BATCH_MAX = 8;          // pieces per consumer batch (<= NSLOTS/2)
constexpr int KV_ROW_BYTES = HD * 2;
constexpr int KV_TOK_PER_PIECE = SLOT_BYTES / KV_ROW_BYTES;  // 48
constexpr int SC_PAIRS = 3;                                  // K/V piece pairs per super-chunk
constexpr int SC_TOK = SC_PAIRS * KV_TOK_PER_PIECE;          // 144
constexpr int SPLIT_MIN_TOK = 64;
constexpr int MAX_SPLITS = 32;
constexpr int MIN_CTAS = 64, MAX_CTAS = 512;  // stage G gathers one CTA per consumer thread
constexpr int MAX_OWN = 64;           // rows per CTA of o_proj/down/gate-up (C >= 64)
constexpr uint32_t BAR_ID = 1;

enum Status : uint32_t {
  ST_OK = 0,
  ST_TIMEOUT_LL = 1,
  ST_TIMEOUT_FULL = 2,
  ST_TIMEOUT_EMPTY = 3,
  ST_TIMEOUT_KV = 4,
  ST_MISALIGNED = 5,
};
enum Where : uint32_t { W_A = 1, W_B, W_C, W_D, W_E, W_F, W_G, W_PROD, W_SELFTEST };

struct Workspace {
  uint64_t *hidden;  // [H]        fp16 payload
  uint64_t *qkv;     // [QKV_ROWS] fp16 payload (q | k | v rows)
  uint64_t *attn;    // [QS/2]     2 x fp16 payload
  uint64_t *act;     // [H]        fp32 payload
  uint64_t *inter;   // [IM]       fp16 payload (half(mlp_inter))
  uint64_t *part;    // [NKV][MAX_SPLITS][2][HD+2] fp32 payload (acc | m | l)
  uint64_t *amax;    // [2][MAX_CTAS] per-CTA argmax value / index
  uint32_t *kv_ready;
  unsigned long long *err;
};

struct DecodeArgs {
  const __half *embed;
  const LDGLayerWeight *layers;
  const __half *final_norm;
  const __half *lm_head;
  const __half *cos_t;
  const __half *sin_t;
  __half *k_cache;
  __half *v_cache;
  __half *hidden;
  float *act;
  float *res;
  __half *q;
  __half *k;
  __half *v;
  __half *attn_out;
  float *inter;
  float *norm_out;
  float *bmax_vals;
  int *bmax_idxs;
  int *out_tokens;
  int num_layers, start_pos, max_seq, num_steps, first_token;
  float attn_scale;
  uint32_t epoch_base;
  long long timeout_ns;
  Workspace ws;
};

struct __align__(128) Smem {
  uint8_t ring[NSLOTS][SLOT_BYTES];
  uint64_t full[NSLOTS];
  uint64_t empty[NSLOTS];
  __half xa[H];          // activation vector for K=1024 GEMVs (stages A, D)
  __half xb[IM];         // activation vector for K=2048/3072 GEMVs (stages C, E)
  float xf[H];           // fp32 final-normed hidden (stage F)
  float red[NCW];
  float g_out[MAX_OWN], u_out[MAX_OWN], act_own[MAX_OWN];
  __half hid_own[MAX_OWN];
  __half qkv_raw[4 * HD];  // q head 2g, q head 2g+1, k head g, v head g
  float q_rot[2][HD];
  __half k_fresh[HD];
  float sc[2][SC_TOK + 1];
  float att_m[2], att_l[2], att_alpha[2];
  float accbuf[NCT];
  float wmax_val[NCW];
  int wmax_idx[NCW];
  float gmax_val[NCW];
  int gmax_idx[NCW];
  volatile uint32_t abort;
};

// B200: 227 KB of dynamic shared memory per block (1 KB kept for alignment).
static_assert(sizeof(Smem) + 1024 <= 232448, "decode kernel shared memory exceeds 227 KB");

// ------------------------------------------------------------------ waits
struct WaitCtx {
  volatile uint32_t *abort;  // CTA-local
  unsigned long long *err;   // kernel-wide status word
  uint32_t tag;              // epoch base of this launch
  long long timeout_ns;
};

__device__ __forceinline__ bool peer_failed(const WaitCtx &w) {
  const uint64_t e = ld_relaxed_u64(reinterpret_cast<const uint64_t *>(w.err));
  return static_cast<uint32_t>(e >> 32) == w.tag && (e & 0xffffffffull) != 0;
}

// Records (tag | code | where | cta) unless this launch already recorded one.
__device__ __noinline__ void set_error(const WaitCtx &w, uint32_t code, uint32_t where) {
  const unsigned long long mine = (static_cast<unsigned long long>(w.tag) << 32) |
                                  (static_cast<unsigned long long>(code & 0xff) << 24) |
                                  (static_cast<unsigned long long>(where & 0xff) << 16) |
                                  (blockIdx.x & 0xffff);
  unsigned long long cur = atomicAdd(w.err, 0ull);
  while (static_cast<uint32_t>(cur >> 32) != w.tag) {
    const unsigned long long prev = atomicCAS(w.err, cur, mine);
    if (prev == cur) break;
    cur = prev;
  }
  *w.abort = 1;
}

// Slow path of a failed poll: returns false (and marks the CTA aborted) when
// the CTA or another CTA aborted, or when the wall-clock bound ran out.
__device__ __forceinline__ bool wait_ok(const WaitCtx &w, uint64_t t0, uint32_t code,
                                        uint32_t where) {
  if (*w.abort) return false;
  if (peer_failed(w)) {
    *w.abort = 1;
    return false;
  }
  if (static_cast<long long>(globaltimer_ns() - t0) > w.timeout_ns) {
    set_error(w, code, where);
    return false;
  }
  return true;
}

__device__ __forceinline__ bool wait_mbar(const WaitCtx &w, uint64_t *bar, uint32_t parity,
                                          uint32_t code, uint32_t where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15) == 0 && !wait_ok(w, t0, code, where)) return false;
  }
}

// Loads N handoff words (addresses from addr(i)) until all carry `epoch`;
// payloads go to out[].  Loads are issued together, so a ready set costs one
// L2 round trip.
template <int N, class AddrFn>
__device__ __forceinline__ bool ll_gather(const WaitCtx &w, AddrFn addr, uint32_t epoch,
                                          uint32_t (&out)[N], uint32_t where) {
  uint64_t v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = ll_load(addr(i));
  bool done = true;
#pragma unroll
  for (int i = 0; i < N; ++i) done &= (static_cast<uint32_t>(v[i] >> 32) == epoch);
  bool ok = true;
  if (!done) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      done = true;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (static_cast<uint32_t>(v[i] >> 32) != epoch) {
          v[i] = ll_load(addr(i));
          done &= (static_cast<uint32_t>(v[i] >> 32) == epoch);
        }
      }
      if (done) break;
      if ((it & 7) == 0 && !wait_ok(w, t0, ST_TIMEOUT_LL, where)) {
        ok = false;
        break;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = static_cast<uint32_t>(v[i]);
  return ok;
}

// ------------------------------------------------------------ work layout
__device__ __forceinline__ int part_lo(int n, int C, int c) {
  return static_cast<int>((static_cast<long long>(n) * c) / C);
}

struct Piece {
  const char *src;
  uint32_t bytes;
  int row0;   // first matrix row (or first token) in the piece
  int nrows;
  int kind;   // QKV: 0 q 1 k 2 v; gate/up: 0 gate 1 up; KV: 0 K 1 V
};

__device__ __forceinline__ int npieces(int nrows, int row_bytes) {
  const int rpp = SLOT_BYTES / row_bytes;
  return (nrows + rpp - 1) / rpp;
}

__device__ __forceinline__ Piece seg_piece(const void *base, int row_bytes, int row0, int nrows,
                                           int i, int kind) {
  const int rpp = SLOT_BYTES / row_bytes;
  Piece P;
  const int r = i * rpp;
  P.row0 = row0 + r;
  P.nrows = min(rpp, nrows - r);
  P.kind = kind;
  P.src = static_cast<const char *>(base) + static_cast<size_t>(P.row0) * row_bytes;
  P.bytes = static_cast<uint32_t>(P.nrows * row_bytes);
  return P;
}

struct LayerPtrs {
  const __half *w[11];
};

__device__ __forceinline__ LayerPtrs load_layer(const LDGLayerWeight *t, int l) {
  const unsigned long long *p = reinterpret_cast<const unsigned long long *>(t + l);
  LayerPtrs L;
#pragma unroll
  for (int i = 0; i < 11; ++i) L.w[i] = reinterpret_cast<const __half *>(__ldg(p + i));
  return L;
}

struct QkvGeom {
  int s_lo[3], s_n[3], np[3], total;
};

__device__ __forceinline__ QkvGeom qkv_geom(int C, int c) {
  QkvGeom g;
  const int lo = part_lo(QKV_ROWS, C, c), hi = part_lo(QKV_ROWS, C, c + 1);
  const int b[4] = {0, QS, QS + KVS, QKV_ROWS};
  g.total = 0;
#pragma unroll
  for (int m = 0; m < 3; ++m) {
    const int a0 = max(lo, b[m]), e0 = min(hi, b[m + 1]);
    g.s_lo[m] = a0 - b[m];
    g.s_n[m] = max(0, e0 - a0);
    g.np[m] = npieces(g.s_n[m], 2 * H);
    g.total += g.np[m];
  }
  return g;
}

__device__ __forceinline__ Piece qkv_piece(const QkvGeom &g, const LayerPtrs &L, int i) {
#pragma unroll
  for (int m = 0; m < 3; ++m) {
    if (i < g.np[m]) return seg_piece(L.w[1 + m], 2 * H, g.s_lo[m], g.s_n[m], i, m);
    i -= g.np[m];
  }
  return seg_piece(L.w[3], 2 * H, g.s_lo[2], g.s_n[2], 0, 2);  // not reached
}

struct AttnGeom {
  int S, has, g, j, t0, t1, last, npairs, nsc;
};

// Split-KV work for position p: the p cached tokens of each KV head are cut
// into S splits of >= SPLIT_MIN_TOK tokens (S <= min(MAX_SPLITS, C/8)); work
// item w = g*S + j runs on CTA w.  The new token (position p) goes to the
// last split of its head.
__device__ __forceinline__ AttnGeom attn_geom(int p, int C, int c) {
  AttnGeom a;
  const int n_old = p;
  const int smax = min(MAX_SPLITS, C / NKV);
  a.S = n_old < SPLIT_MIN_TOK ? 1 : min(smax, (n_old + SPLIT_MIN_TOK - 1) / SPLIT_MIN_TOK);
  a.has = c < NKV * a.S;
  a.g = c / a.S;
  a.j = c % a.S;
  const int per = (n_old + a.S - 1) / a.S;
  a.t0 = min(n_old, a.j * per);
  a.t1 = min(n_old, a.t0 + per);
  a.last = (a.j == a.S - 1);
  a.npairs = (a.t1 - a.t0 + KV_TOK_PER_PIECE - 1) / KV_TOK_PER_PIECE;
  a.nsc = max(1, (a.npairs + SC_PAIRS - 1) / SC_PAIRS);
  return a;
}

__device__ __forceinline__ Piece kv_piece(const DecodeArgs &a, const AttnGeom &ag, int l, int i) {
  const int pair = i >> 1, kind = i & 1;
  const int tok0 = ag.t0 + pair * KV_TOK_PER_PIECE;
  const __half *base = (kind ? a.v_cache : a.k_cache) +
                       (static_cast<size_t>(l) * NKV + ag.g) * static_cast<size_t>(a.max_seq) * HD;
  return seg_piece(base, KV_ROW_BYTES, tok0, min(KV_TOK_PER_PIECE, ag.t1 - tok0), 0, kind);
}

__device__ __forceinline__ WaitCtx make_wait(const DecodeArgs &a, Smem &sm) {
  WaitCtx w;
  w.abort = &sm.abort;
  w.err = a.ws.err;
  w.tag = a.epoch_base;
  w.timeout_ns = a.timeout_ns;
  return w;
}

// ------------------------------------------------------------- producer
__device__ __noinline__ void producer(const DecodeArgs &a, Smem &sm) {
  const int C = gridDim.x, c = blockIdx.x, L = a.num_layers;
  const WaitCtx w = make_wait(a, sm);
  const uint64_t pol = policy_evict_first();
  uint32_t n = 0;
  bool ok = true;

  auto issue = [&](const Piece &P) -> bool {
    const int slot = n % NSLOTS;
    const uint32_t round = n / NSLOTS;
    if (round > 0 && !wait_mbar(w, &sm.empty[slot], (round - 1) & 1, ST_TIMEOUT_EMPTY, W_PROD))
      return false;
    if ((reinterpret_cast<uintptr_t>(P.src) & 15u) || (P.bytes & 15u) || P.bytes == 0 ||
        P.bytes > static_cast<uint32_t>(SLOT_BYTES)) {
      set_error(w, ST_MISALIGNED, W_PROD);
      return false;
    }
    mbar_arrive_expect_tx(&sm.full[slot], P.bytes);
    bulk_g2s(sm.ring[slot], P.src, P.bytes, &sm.full[slot], pol);
    ++n;
    return true;
  };

  const QkvGeom qg = qkv_geom(C, c);
  const int o_lo = part_lo(H, C, c), o_n = part_lo(H, C, c + 1) - o_lo;
  const int gu_lo = part_lo(IM, C, c), gu_n = part_lo(IM, C, c + 1) - gu_lo;
  const int lm_lo = part_lo(VOCAB, C, c), lm_n = part_lo(VOCAB, C, c + 1) - lm_lo;
  const int o_np = npieces(o_n, 2 * QS), gu_np = npieces(gu_n, 2 * H);
  const int d_np = npieces(o_n, 2 * IM), lm_np = npieces(lm_n, 2 * H);

  for (int s = 0; s < a.num_steps && ok; ++s) {
    const int p = a.start_pos + s;
    const AttnGeom ag = attn_geom(p, C, c);
    for (int l = 0; l < L && ok; ++l) {
      const LayerPtrs lp = load_layer(a.layers, l);
      for (int i = 0; i < qg.total && ok; ++i) ok = issue(qkv_piece(qg, lp, i));
      if (ok && ag.has && ag.npairs > 0) {
        // Cached tokens written earlier in this launch must be visible to the
        // bulk-copy engine: wait for every KV write of the previous steps.
        if (s > 0 && ag.t1 > a.start_pos) {
          const uint32_t target = static_cast<uint32_t>(s) * L * NKV;
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t it = 1; ld_acquire_u32(a.ws.kv_ready) < target; ++it) {
            if (!wait_ok(w, t0, ST_TIMEOUT_KV, W_PROD)) {
              ok = false;
              break;
            }
          }
          fence_proxy_async_global();
        }
        for (int i = 0; i < 2 * ag.npairs && ok; ++i) ok = issue(kv_piece(a, ag, l, i));
      }
      for (int i = 0; i < o_np && ok; ++i) ok = issue(seg_piece(lp.w[6], 2 * QS, o_lo, o_n, i, 0));
      for (int i = 0; i < 2 * gu_np && ok; ++i)
        ok = issue(seg_piece((i & 1) ? lp.w[9] : lp.w[8], 2 * H, gu_lo, gu_n, i >> 1, i & 1));
      for (int i = 0; i < d_np && ok; ++i) ok = issue(seg_piece(lp.w[10], 2 * IM, o_lo, o_n, i, 0));
    }
    for (int i = 0; i < lm_np && ok; ++i) ok = issue(seg_piece(a.lm_head, 2 * H, lm_lo, lm_n, i, 0));
  }

  if (!ok) {
    // Let every copy already issued land before the CTA exits.
    *w.abort = 1;
    for (int k = 0; k < NSLOTS; ++k) {
      if (n <= static_cast<uint32_t>(k)) break;
      const uint32_t last = k + NSLOTS * ((n - 1 - k) / NSLOTS);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.full[k], (last / NSLOTS) & 1)) {
        if (static_cast<long long>(globaltimer_ns() - t0) > w.timeout_ns) break;
      }
    }
  }
}

// -------------------------------------------------------------- consumers
// Consumes `count` ring pieces of fp16 rows of length K (pieces from
// get_piece(i)), batch by batch; row j of a batch goes to warp j % NCW.  The
// activation vector x (fp16[K]) is read from shared memory.
// epi(piece, matrix_row, dot) runs on every lane of the owning warp.
template <int K, class GetPiece, class Epi>
__device__ __forceinline__ bool gemv_pieces(Smem &sm, const WaitCtx &w, uint32_t &n, int count,
                                            GetPiece get_piece, const __half *x, Epi epi,
                                            uint32_t where) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool ok = true;
  for (int b0 = 0; b0 < count; b0 += BATCH_MAX) {
    const int nb = min(BATCH_MAX, count - b0);
    int j0 = 0;
    for (int i = 0; i < nb; ++i) {
      const Piece P = get_piece(b0 + i);
      const uint32_t pn = n + i;
      const int slot = pn % NSLOTS;
      int r = (warp - j0) % NCW;
      if (r < 0) r += NCW;
      if (r < P.nrows) ok &= wait_mbar(w, &sm.full[slot], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, where);
      for (; r < P.nrows; r += NCW) {
        const __half *row = reinterpret_cast<const __half *>(sm.ring[slot] + r * (K * 2));
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int jj = 0; jj < K / 256; jj += 2) {
          const int o0 = lane * 8 + 256 * jj;
          acc0 = dot8_hh(*reinterpret_cast<const uint4 *>(row + o0),
                         *reinterpret_cast<const uint4 *>(x + o0), acc0);
          acc1 = dot8_hh(*reinterpret_cast<const uint4 *>(row + o0 + 256),
                         *reinterpret_cast<const uint4 *>(x + o0 + 256), acc1);
        }
        epi(P, P.row0 + r, warp_sum(acc0 + acc1));
      }
      j0 += P.nrows;
    }
    __syncwarp();
    if (lane == 0)
      for (int i = 0; i < nb; ++i) mbar_arrive(&sm.empty[(n + i) % NSLOTS]);
    n += nb;
  }
  return ok;
}

__device__ __forceinline__ __half silu_half(float g) {
  // megakernel.cu:141-154: every step in fp16 (exp2f / reciprocal in fp32,
  // rounded to fp16).
  const __half x = __float2half(g);
  const __half t = __hmul(__hneg(x), __float2half(1.44269504088896340736f));
  const __half e = __float2half(exp2f(__half2float(t)));
  const __half d = __hadd(__float2half(1.0f), e);
  const __half r = __float2half(1.0f / __half2float(d));
  return __hmul(x, r);
}

// Stage B.  Returns true when the CTA must abort (uniform across consumers).
__device__ __noinline__ bool attention(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                          const AttnGeom &ag, int l, int p, uint32_t ep, const LayerPtrs &lp,
                          bool &fail) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = ag.g;
  {
    const int word = tid < 256 ? (256 * g + tid)
                               : (tid < 384 ? (QS + 128 * g + tid - 256) : (QS + KVS + 128 * g + tid - 384));
    uint32_t u[1];
    fail |= !ll_gather<1>(w, [&](int) { return a.ws.qkv + word; }, ep, u, W_B);
    sm.qkv_raw[tid] = u2h(u[0]);
    if (tid < 2) {
      sm.att_m[tid] = -INFINITY;
      sm.att_l[tid] = 0.f;
    }
  }
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;

  // q/k RMSNorm (eps 1e-6) + rotate-half RoPE, megakernel.cu:345-434.
  if (warp < 2 || (ag.last && warp == 2)) {
    const __half *src = sm.qkv_raw + warp * HD;
    const __half *nw = warp < 2 ? lp.w[4] : lp.w[5];
    const __half *cosp = a.cos_t + static_cast<size_t>(p) * HD;
    const __half *sinp = a.sin_t + static_cast<size_t>(p) * HD;
    float xv[4], ss = 0.f;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      xv[it] = __half2float(src[lane + 32 * it]);
      ss = fmaf(xv[it], xv[it], ss);
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / static_cast<float>(HD) + 1e-6f);
    float vals[4];
#pragma unroll
    for (int it = 0; it < 4; ++it)
      vals[it] = __fmul_rn(__fmul_rn(xv[it], inv), __half2float(__ldg(nw + lane + 32 * it)));
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int i = lane + 32 * it;
      const int ri = it < 2 ? i : i - HD / 2;
      const float cs = __half2float(__ldg(cosp + ri)), sn = __half2float(__ldg(sinp + ri));
      const float r = it < 2 ? __fsub_rn(__fmul_rn(vals[it], cs), __fmul_rn(vals[it + 2], sn))
                             : __fadd_rn(__fmul_rn(vals[it - 2], sn), __fmul_rn(vals[it], cs));
      const __half hr = __float2half(r);
      if (warp < 2) sm.q_rot[warp][i] = __half2float(hr);
      else sm.k_fresh[i] = hr;
    }
  }
  named_bar_sync(BAR_ID, NCT);

  if (ag.last) {
    // New token's K (rotated) and V (raw) into the cache at position p.
    const size_t off = ((static_cast<size_t>(l) * NKV + g) * a.max_seq + p) * HD;
    if (tid < HD) a.k_cache[off + tid] = sm.k_fresh[tid];
    else if (tid < 2 * HD) a.v_cache[off + tid - HD] = sm.qkv_raw[3 * HD + tid - HD];
    if (tid < 2 * HD) {
      fence_proxy_async_global();
      __threadfence();
    }
    named_bar_sync(BAR_ID, NCT);
    if (tid == 0) red_release_add_u32(a.ws.kv_ready, 1);
  }

  const int pair = tid & 255, hh = pair >> 7, dd = pair & 127, par = tid >> 8;
  float acc = 0.f;
  const int total_old = ag.t1 - ag.t0;
  for (int sc = 0; sc < ag.nsc; ++sc) {
    const int pair0 = sc * SC_PAIRS;
    const int npair = max(0, min(SC_PAIRS, ag.npairs - pair0));
    const int n_old = max(0, min(SC_TOK, total_old - pair0 * KV_TOK_PER_PIECE));
    const bool fresh = ag.last && (sc == ag.nsc - 1);
    const int ntok = n_old + (fresh ? 1 : 0);
    // Scores: one warp per token, lanes over 4 dims each.
    for (int tt = warp; tt < ntok; tt += NCW) {
      const __half *krow;
      if (tt < n_old) {
        const uint32_t pn = n + 2 * (tt / KV_TOK_PER_PIECE);
        fail |= !wait_mbar(w, &sm.full[pn % NSLOTS], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, W_B);
        krow = reinterpret_cast<const __half *>(sm.ring[pn % NSLOTS] + (tt % KV_TOK_PER_PIECE) * KV_ROW_BYTES);
      } else {
        krow = sm.k_fresh;
      }
      const uint2 kv = *reinterpret_cast<const uint2 *>(krow + 4 * lane);
      const float2 k01 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.x));
      const float2 k23 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.y));
      const float4 q0 = *reinterpret_cast<const float4 *>(&sm.q_rot[0][4 * lane]);
      const float4 q1 = *reinterpret_cast<const float4 *>(&sm.q_rot[1][4 * lane]);
      float d0 = q0.x * k01.x;
      d0 = fmaf(q0.y, k01.y, d0);
      d0 = fmaf(q0.z, k23.x, d0);
      d0 = fmaf(q0.w, k23.y, d0);
      float d1 = q1.x * k01.x;
      d1 = fmaf(q1.y, k01.y, d1);
      d1 = fmaf(q1.z, k23.x, d1);
      d1 = fmaf(q1.w, k23.y, d1);
      d0 = warp_sum(d0);
      d1 = warp_sum(d1);
      if (lane == 0) {
        sm.sc[0][tt] = d0 * a.attn_scale;
        sm.sc[1][tt] = d1 * a.attn_scale;
      }
    }
    named_bar_sync(BAR_ID, NCT);
    // Online softmax update per head (expf as upstream, :490-494).
    if (warp < 2 && ntok > 0) {
      float mx = -INFINITY;
      for (int tt = lane; tt < ntok; tt += 32) mx = fmaxf(mx, sm.sc[warp][tt]);
      mx = warp_max(mx);
      const float m_old = sm.att_m[warp];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int tt = lane; tt < ntok; tt += 32) {
        const float pr = expf(sm.sc[warp][tt] - m_new);
        sm.sc[warp][tt] = pr;
        sum += pr;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sm.att_alpha[warp] = alpha;
        sm.att_l[warp] = sm.att_l[warp] * alpha + sum;
        sm.att_m[warp] = m_new;
      }
    } else if (warp < 2 && lane == 0) {
      sm.att_alpha[warp] = 1.f;
    }
    named_bar_sync(BAR_ID, NCT);
    // P.V: thread (head hh, dim dd) over tokens of parity `par`.
    acc *= sm.att_alpha[hh];
    for (int tt = par; tt < ntok; tt += 2) {
      __half vv;
      if (tt < n_old) {
        const uint32_t pn = n + 2 * (tt / KV_TOK_PER_PIECE) + 1;
        if ((tt % KV_TOK_PER_PIECE) < 2)
          fail |= !wait_mbar(w, &sm.full[pn % NSLOTS], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, W_B);
        vv = reinterpret_cast<const __half *>(sm.ring[pn % NSLOTS] +
                                              (tt % KV_TOK_PER_PIECE) * KV_ROW_BYTES)[dd];
      } else {
        vv = sm.qkv_raw[3 * HD + dd];
      }
      acc = fmaf(sm.sc[hh][tt], __half2float(vv), acc);
    }
    named_bar_sync(BAR_ID, NCT);
    if (lane == 0)
      for (int i = 0; i < 2 * npair; ++i) mbar_arrive(&sm.empty[(n + i) % NSLOTS]);
    n += 2 * npair;
  }

  sm.accbuf[tid] = acc;
  named_bar_sync(BAR_ID, NCT);
  if (tid < 256) {
    const int h = tid >> 7, d = tid & 127;
    float val = sm.accbuf[tid] + sm.accbuf[tid + 256];
    float m = sm.att_m[h], lsum = sm.att_l[h];
    bool write_out = false;
    if (ag.S > 1 && ag.j != 0) {
      uint64_t *pp = a.ws.part + ((static_cast<size_t>(g) * MAX_SPLITS + ag.j) * 2 + h) * (HD + 2);
      ll_store(pp + d, __float_as_uint(val), ep);
      if (d < 2) ll_store(pp + HD + d, __float_as_uint(d == 0 ? m : lsum), ep);
    } else if (ag.S > 1) {
      // Combiner (split 0): merge the other splits' (m, l, acc), 8 at a time.
      for (int j0 = 1; j0 < ag.S; j0 += 4) {
        uint32_t u[12];
        const int jn = min(4, ag.S - j0);
        fail |= !ll_gather<12>(
            w,
            [&](int i) {
              const int jj = j0 + min(i / 3, jn - 1);
              const uint64_t *pp =
                  a.ws.part + ((static_cast<size_t>(g) * MAX_SPLITS + jj) * 2 + h) * (HD + 2);
              const int k = i % 3;
              return pp + (k == 0 ? d : HD + k - 1);
            },
            ep, u, W_B);
        for (int q = 0; q < jn; ++q) {
          const float aj = __uint_as_float(u[3 * q]), mj = __uint_as_float(u[3 * q + 1]),
                      lj = __uint_as_float(u[3 * q + 2]);
          if (mj == -INFINITY) continue;
          if (m == -INFINITY) {
            m = mj;
            lsum = lj;
            val = aj;
            continue;
          }
          const float mn = fmaxf(m, mj);
          const float f0 = expf(m - mn), f1 = expf(mj - mn);
          val = val * f0 + aj * f1;
          lsum = lsum * f0 + lj * f1;
          m = mn;
        }
      }
      write_out = true;
    } else {
      write_out = true;
    }
    if (write_out) {
      const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
      const __half o = __float2half(val * inv);
      const int col = (2 * g + h) * HD + d;
      a.attn_out[col] = o;
      const uint32_t other = __shfl_down_sync(0xffffffffu, h2u(o), 1);
      if ((d & 1) == 0) ll_store(a.ws.attn + col / 2, h2u(o) | (other << 16), ep);
    }
  }
  return false;
}

// Per-CTA row ranges of the stage GEMVs (same split for o_proj and down, so
// a CTA owns the same hidden rows in stages C and E).
struct Rows {
  int lo, n;
};
__device__ __forceinline__ Rows rows_of(int total, int C, int c) {
  Rows r;
  r.lo = part_lo(total, C, c);
  r.n = part_lo(total, C, c + 1) - r.lo;
  return r;
}

__device__ __forceinline__ const __half *layer_ptr(const LDGLayerWeight *t, int l, int idx) {
  return reinterpret_cast<const __half *>(
      __ldg(reinterpret_cast<const unsigned long long *>(t + l) + idx));
}

// Stage A: input RMSNorm (megakernel.cu:806-847) + fused QKV GEMV (:242-291).
// Returns true when the CTA must abort (uniform across consumer threads).
__device__ __noinline__ bool stage_a(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                                     bool &fail, int l, int token, uint32_t ep) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = gridDim.x, c = blockIdx.x;
  float h0, h1;
  if (l == 0) {
    const __half *emb = a.embed + static_cast<size_t>(token) * H;
    h0 = __half2float(__ldg(emb + tid));
    h1 = __half2float(__ldg(emb + tid + NCT));
    const Rows o = rows_of(H, C, c);
    if (tid < o.n) sm.hid_own[tid] = __ldg(emb + o.lo + tid);
  } else {
    uint32_t u[2];
    fail |= !ll_gather<2>(w, [&](int i) { return a.ws.hidden + tid + i * NCT; }, ep - 1, u, W_A);
    h0 = __half2float(u2h(u[0]));
    h1 = __half2float(u2h(u[1]));
  }
  const float ss = warp_sum(fmaf(h0, h0, h1 * h1));
  if (lane == 0) sm.red[warp] = ss;
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
  {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) tot += sm.red[i];
    const float inv = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
    const __half *nw = layer_ptr(a.layers, l, 0);
    sm.xa[tid] = __float2half(h0 * (inv * __half2float(__ldg(nw + tid))));
    sm.xa[tid + NCT] = __float2half(h1 * (inv * __half2float(__ldg(nw + tid + NCT))));
  }
  named_bar_sync(BAR_ID, NCT);
  const QkvGeom qg = qkv_geom(C, c);
  const LayerPtrs lp{};  // consumers only need row ranges, not addresses
  fail |= !gemv_pieces<H>(
      sm, w, n, qg.total, [&](int i) { return qkv_piece(qg, lp, i); }, sm.xa,
      [&](const Piece &P, int row, float dot) {
        if (lane == 0) {
          const __half hv = __float2half(dot);
          const int vrow = (P.kind == 0 ? 0 : (P.kind == 1 ? QS : QS + KVS)) + row;
          ll_store(a.ws.qkv + vrow, h2u(hv), ep);
          __half *dst = P.kind == 0 ? a.q : (P.kind == 1 ? a.k : a.v);
          dst[row] = hv;
        }
      },
      W_A);
  return false;
}

// Stage C: o_proj GEMV + fp32 residual (megakernel.cu:585-610, :868-872).
__device__ __noinline__ bool stage_c(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                                     bool &fail, uint32_t ep) {
  const int tid = threadIdx.x, lane = tid & 31;
  {
    uint32_t u[2];
    fail |= !ll_gather<2>(w, [&](int i) { return a.ws.attn + tid + i * NCT; }, ep, u, W_C);
    reinterpret_cast<uint32_t *>(sm.xb)[tid] = u[0];
    reinterpret_cast<uint32_t *>(sm.xb)[tid + NCT] = u[1];
  }
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
  const Rows o = rows_of(H, gridDim.x, blockIdx.x);
  fail |= !gemv_pieces<QS>(
      sm, w, n, npieces(o.n, 2 * QS), [&](int i) { return seg_piece(nullptr, 2 * QS, o.lo, o.n, i, 0); },
      sm.xb,
      [&](const Piece &, int row, float dot) {
        if (lane == 0) {
          const float resid = __half2float(sm.hid_own[row - o.lo]);
          const float act = dot + resid;
          ll_store(a.ws.act + row, __float_as_uint(act), ep);
          a.act[row] = act;
          a.res[row] = resid;
          sm.act_own[row - o.lo] = act;
        }
      },
      W_C);
  return false;
}

// Stage D: post-attention RMSNorm from fp32 act (megakernel.cu:614-638) +
// gate/up GEMV + half SiLU * up (:640-675).
__device__ __noinline__ bool stage_d(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                                     bool &fail, int l, uint32_t ep) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float h0, h1;
  {
    uint32_t u[2];
    fail |= !ll_gather<2>(w, [&](int i) { return a.ws.act + tid + i * NCT; }, ep, u, W_D);
    h0 = __uint_as_float(u[0]);
    h1 = __uint_as_float(u[1]);
    const float ss = warp_sum(fmaf(h0, h0, h1 * h1));
    if (lane == 0) sm.red[warp] = ss;
  }
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
  {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) tot += sm.red[i];
    const float rstd = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
    const __half *nw = layer_ptr(a.layers, l, 7);
    sm.xa[tid] = __float2half(__half2float(__float2half(h0)) * rstd * __half2float(__ldg(nw + tid)));
    sm.xa[tid + NCT] =
        __float2half(__half2float(__float2half(h1)) * rstd * __half2float(__ldg(nw + tid + NCT)));
  }
  named_bar_sync(BAR_ID, NCT);
  const Rows gu = rows_of(IM, gridDim.x, blockIdx.x);
  fail |= !gemv_pieces<H>(
      sm, w, n, 2 * npieces(gu.n, 2 * H),
      [&](int i) { return seg_piece(nullptr, 2 * H, gu.lo, gu.n, i >> 1, i & 1); }, sm.xa,
      [&](const Piece &P, int row, float dot) {
        if (lane == 0) (P.kind == 0 ? sm.g_out : sm.u_out)[row - gu.lo] = dot;
      },
      W_D);
  named_bar_sync(BAR_ID, NCT);
  if (tid < gu.n) {
    const float act = __half2float(silu_half(sm.g_out[tid])) * sm.u_out[tid];
    const int row = gu.lo + tid;
    ll_store(a.ws.inter + row, h2u(__float2half(act)), ep);
    a.inter[row] = act;
  }
  return false;
}

// Stage E: down GEMV on half(mlp_inter) + residual, rounded to fp16
// (megakernel.cu:679-707).
__device__ __noinline__ bool stage_e(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                                     bool &fail, uint32_t ep) {
  const int tid = threadIdx.x, lane = tid & 31;
  {
    uint32_t u[IM / NCT];
    fail |= !ll_gather<IM / NCT>(w, [&](int i) { return a.ws.inter + tid + i * NCT; }, ep, u, W_E);
#pragma unroll
    for (int i = 0; i < IM / NCT; ++i) sm.xb[tid + i * NCT] = u2h(u[i]);
  }
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
  const Rows o = rows_of(H, gridDim.x, blockIdx.x);
  fail |= !gemv_pieces<IM>(
      sm, w, n, npieces(o.n, 2 * IM), [&](int i) { return seg_piece(nullptr, 2 * IM, o.lo, o.n, i, 0); },
      sm.xb,
      [&](const Piece &, int row, float dot) {
        if (lane == 0) {
          const __half hv = __float2half(dot + sm.act_own[row - o.lo]);
          ll_store(a.ws.hidden + row, h2u(hv), ep);
          a.hidden[row] = hv;
          sm.hid_own[row - o.lo] = hv;
        }
      },
      W_E);
  return false;
}

// Stage F: final RMSNorm to fp32 (megakernel.cu:890-919), tied lm_head GEMV
// and this CTA's argmax (:1001-1109; lowest index among equal maxima).
__device__ __noinline__ bool stage_f(Smem &sm, const DecodeArgs &a, const WaitCtx &w, uint32_t &n,
                                     bool &fail, int s, uint32_t ep_last) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  {
    uint32_t u[2];
    fail |= !ll_gather<2>(w, [&](int i) { return a.ws.hidden + tid + i * NCT; }, ep_last, u, W_F);
    const float f0 = __half2float(u2h(u[0])), f1 = __half2float(u2h(u[1]));
    const float ssum = warp_sum(fmaf(f0, f0, f1 * f1));
    if (lane == 0) sm.red[warp] = ssum;
    if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) tot += sm.red[i];
    const float inv = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
    const float n0 = f0 * inv * __half2float(__ldg(a.final_norm + tid));
    const float n1 = f1 * inv * __half2float(__ldg(a.final_norm + tid + NCT));
    sm.xf[tid] = n0;
    sm.xf[tid + NCT] = n1;
    if (c == 0) {
      a.norm_out[tid] = n0;
      a.norm_out[tid + NCT] = n1;
    }
  }
  named_bar_sync(BAR_ID, NCT);
  const Rows lm = rows_of(VOCAB, gridDim.x, c);
  const int lm_np = npieces(lm.n, 2 * H);
  float4 xr[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    xr[2 * j] = *reinterpret_cast<const float4 *>(sm.xf + lane * 8 + 256 * j);
    xr[2 * j + 1] = *reinterpret_cast<const float4 *>(sm.xf + lane * 8 + 256 * j + 4);
  }
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int b0 = 0; b0 < lm_np; b0 += BATCH_MAX) {
    const int nb = min(BATCH_MAX, lm_np - b0);
    int j0 = 0;
    for (int i = 0; i < nb; ++i) {
      const Piece P = seg_piece(nullptr, 2 * H, lm.lo, lm.n, b0 + i, 0);
      const uint32_t pn = n + i;
      const int slot = pn % NSLOTS;
      int r = (warp - j0) % NCW;
      if (r < 0) r += NCW;
      if (r < P.nrows) fail |= !wait_mbar(w, &sm.full[slot], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, W_F);
      for (; r < P.nrows; r += NCW) {
        const __half *row = reinterpret_cast<const __half *>(sm.ring[slot] + r * (2 * H));
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          acc0 = dot8_hf(*reinterpret_cast<const uint4 *>(row + lane * 8 + 256 * j), xr[2 * j],
                         xr[2 * j + 1], acc0);
          acc1 = dot8_hf(*reinterpret_cast<const uint4 *>(row + lane * 8 + 256 * (j + 1)),
                         xr[2 * j + 2], xr[2 * j + 3], acc1);
        }
        const float v = warp_sum(acc0 + acc1);
        const int idx = P.row0 + r;
        if (v > best || (v == best && idx < bidx)) {
          best = v;
          bidx = idx;
        }
      }
      j0 += P.nrows;
    }
    __syncwarp();
    if (lane == 0)
      for (int i = 0; i < nb; ++i) mbar_arrive(&sm.empty[(n + i) % NSLOTS]);
    n += nb;
  }
  if (lane == 0) {
    sm.wmax_val[warp] = best;
    sm.wmax_idx[warp] = bidx;
  }
  named_bar_sync(BAR_ID, NCT);
  if (tid == 0) {
    float bv = sm.wmax_val[0];
    int bi = sm.wmax_idx[0];
    for (int i = 1; i < NCW; ++i) {
      const float v = sm.wmax_val[i];
      const int id = sm.wmax_idx[i];
      if (v > bv || (v == bv && id < bi)) {
        bv = v;
        bi = id;
      }
    }
    const uint32_t eps_ = a.epoch_base + static_cast<uint32_t>(s);
    ll_store(a.ws.amax + c, __float_as_uint(bv), eps_);
    ll_store(a.ws.amax + MAX_CTAS + c, static_cast<uint32_t>(bi), eps_);
    a.bmax_vals[c] = bv;
    a.bmax_idxs[c] = bi;
  }
  return false;
}

// Stage G: global argmax over the per-CTA results (megakernel.cu:1114-1144),
// lowest index among equal maxima.  Sets *token_out (uniform).
__device__ __noinline__ bool stage_g(Smem &sm, const DecodeArgs &a, const WaitCtx &w, bool &fail,
                                     int s, int *token_out) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = gridDim.x;
  float v = -INFINITY;
  int id = 0x7fffffff;
  if (tid < C) {
    uint32_t u[2];
    const uint32_t eps_ = a.epoch_base + static_cast<uint32_t>(s);
    fail |= !ll_gather<2>(w, [&](int i) { return a.ws.amax + i * MAX_CTAS + tid; }, eps_, u, W_G);
    v = __uint_as_float(u[0]);
    id = static_cast<int>(u[1]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (ov > v || (ov == v && oi < id)) {
      v = ov;
      id = oi;
    }
  }
  if (lane == 0) {
    sm.gmax_val[warp] = v;
    sm.gmax_idx[warp] = id;
  }
  if (named_bar_or(BAR_ID, NCT, fail || sm.abort)) return true;
  float bv = sm.gmax_val[0];
  int bi = sm.gmax_idx[0];
  for (int i = 1; i < NCW; ++i) {
    const float vv = sm.gmax_val[i];
    const int ii = sm.gmax_idx[i];
    if (vv > bv || (vv == bv && ii < bi)) {
      bv = vv;
      bi = ii;
    }
  }
  if (blockIdx.x == 0 && tid == 0) a.out_tokens[s] = bi;
  *token_out = (bi >= 0 && bi < VOCAB) ? bi : 0;
  return false;
}

__device__ void consumer(const DecodeArgs &a, Smem &sm) {
  const int C = gridDim.x, c = blockIdx.x, L = a.num_layers;
  const WaitCtx w = make_wait(a, sm);
  uint32_t n = 0;
  int token = a.first_token;
  bool fail = false;
  int s = 0;
  for (s = 0; s < a.num_steps; ++s) {
    const int p = a.start_pos + s;
    for (int l = 0; l < L; ++l) {
      const uint32_t ep = a.epoch_base + static_cast<uint32_t>(s * L + l);
      if (stage_a(sm, a, w, n, fail, l, token, ep)) goto out;
      const AttnGeom ag = attn_geom(p, C, c);
      if (ag.has) {
        const LayerPtrs lp = load_layer(a.layers, l);
        if (attention(sm, a, w, n, ag, l, p, ep, lp, fail)) goto out;
      }
      if (stage_c(sm, a, w, n, fail, ep)) goto out;
      if (stage_d(sm, a, w, n, fail, l, ep)) goto out;
      if (stage_e(sm, a, w, n, fail, ep)) goto out;
    }
    if (stage_f(sm, a, w, n, fail, s, a.epoch_base + static_cast<uint32_t>(s * L + L - 1))) goto out;
    if (stage_g(sm, a, w, fail, s, &token)) goto out;
  }
  return;
out:
  if (c == 0 && threadIdx.x == 0)
    for (int s2 = s; s2 < a.num_steps; ++s2) a.out_tokens[s2] = -1;
}

__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < NSLOTS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], NCW);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (tid >= NCT) {
    if (tid == NCT) producer(a, sm);
    return;
  }
  consumer(a, sm);
}

// Failure-detection self test: waits on a handoff word nothing writes.
__global__ void selftest_wait_kernel(uint64_t *word, unsigned long long *err, long long timeout_ns,
                                     uint32_t tag) {
  __shared__ volatile uint32_t abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  if (threadIdx.x != 0) return;
  WaitCtx w;
  w.abort = &abort_flag;
  w.err = err;
  w.tag = tag;
  w.timeout_ns = timeout_ns;
  uint32_t u[1];
  ll_gather<1>(w, [&](int) { return word; }, 0xfffffff0u, u, W_SELFTEST);
}

}  // namespace qb200

// ====================================================================== host
using namespace qb200;

namespace {

struct DevState {
  bool ready = false;
  int num_sms = 0;
  Workspace ws{};
  void *mem = nullptr;
  size_t ll_bytes = 0;
  uint32_t epoch = 1;
  uint32_t last_tag = 0;
};

std::mutex g_mu;
DevState g_dev[64];
long long g_timeout_ns = 2000000000LL;
thread_local int t_err = 0;
thread_local char t_msg[512] = {0};

int fail_msg(int code, const char *fmt, ...) {
  t_err = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return code;
}

size_t smem_bytes() { return sizeof(Smem) + 1024; }

DevState *get_dev(int *dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail_msg(2, "cudaGetDevice failed");
    return nullptr;
  }
  *dev_out = dev;
  DevState &d = g_dev[dev];
  if (d.ready) return &d;
  int sms = 0, coop = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop) {
    fail_msg(3, "device %d does not support cooperative launch", dev);
    return nullptr;
  }
  if (sms < MIN_CTAS || sms > MAX_CTAS) {
    fail_msg(3, "device %d has %d SMs; this kernel needs %d..%d", dev, sms, MIN_CTAS, MAX_CTAS);
    return nullptr;
  }
  cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem_bytes()));
  if (e != cudaSuccess) {
    fail_msg(4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return nullptr;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, NTHREADS, smem_bytes());
  if (per_sm < 1) {
    fail_msg(4, "decode kernel does not fit on an SM (%zu B shared memory)", smem_bytes());
    return nullptr;
  }
  const size_t words = H + QKV_ROWS + QS / 2 + H + IM +
                       static_cast<size_t>(NKV) * MAX_SPLITS * 2 * (HD + 2) + 2 * MAX_CTAS;
  const size_t ll_bytes = words * sizeof(uint64_t);
  const size_t total = ll_bytes + 256;
  void *mem = nullptr;
  e = cudaMalloc(&mem, total);
  if (e != cudaSuccess) {
    fail_msg(5, "cudaMalloc(%zu) for the decode workspace: %s", total, cudaGetErrorString(e));
    return nullptr;
  }
  cudaMemset(mem, 0, total);
  uint64_t *p = static_cast<uint64_t *>(mem);
  d.ws.hidden = p; p += H;
  d.ws.qkv = p; p += QKV_ROWS;
  d.ws.attn = p; p += QS / 2;
  d.ws.act = p; p += H;
  d.ws.inter = p; p += IM;
  d.ws.part = p; p += static_cast<size_t>(NKV) * MAX_SPLITS * 2 * (HD + 2);
  d.ws.amax = p; p += 2 * MAX_CTAS;
  d.ws.kv_ready = reinterpret_cast<uint32_t *>(p);
  d.ws.err = reinterpret_cast<unsigned long long *>(p) + 4;
  d.mem = mem;
  d.ll_bytes = ll_bytes;
  d.num_sms = sms;
  d.epoch = 1;
  d.ready = true;
  return &d;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_decode(DecodeArgs &a, cudaStream_t st) {
  t_err = 0;
  t_msg[0] = 0;
  if (a.num_layers < 1 || a.num_layers > 4096)
    return fail_msg(10, "num_layers=%d out of range", a.num_layers);
  if (a.num_steps < 1) return fail_msg(10, "num_steps=%d must be >= 1", a.num_steps);
  if (a.max_seq < 1 || a.max_seq > (1 << 20)) return fail_msg(10, "max_seq_len=%d out of range", a.max_seq);
  if (a.start_pos < 0 || static_cast<long long>(a.start_pos) + a.num_steps > a.max_seq)
    return fail_msg(11,
                    "positions %d..%d exceed max_seq_len=%d (the KV cache has no slot for them)",
                    a.start_pos, a.start_pos + a.num_steps - 1, a.max_seq);
  if (a.first_token < 0 || a.first_token >= VOCAB)
    return fail_msg(12, "token id %d outside [0, %d)", a.first_token, VOCAB);
  const void *ptrs[] = {a.embed, a.layers, a.final_norm, a.lm_head, a.cos_t, a.sin_t, a.k_cache,
                        a.v_cache, a.hidden, a.act, a.res, a.q, a.k, a.v, a.attn_out, a.inter,
                        a.norm_out, a.bmax_vals, a.bmax_idxs, a.out_tokens};
  for (const void *q : ptrs) {
    if (!q) return fail_msg(13, "null pointer argument");
  }
  for (const void *q : {static_cast<const void *>(a.embed), static_cast<const void *>(a.layers),
                        static_cast<const void *>(a.lm_head), static_cast<const void *>(a.k_cache),
                        static_cast<const void *>(a.v_cache)}) {
    if (!aligned16(q))
      return fail_msg(14, "layer_weights_packed / weights / KV cache must be 16-byte aligned");
  }
  std::lock_guard<std::mutex> lk(g_mu);
  int dev = 0;
  DevState *d = get_dev(&dev);
  if (!d) return t_err;
  if (d->num_sms > MAX_CTAS) return fail_msg(3, "too many SMs");
  const uint64_t need = static_cast<uint64_t>(a.num_steps) * (a.num_layers + 1) + 2;
  if (static_cast<uint64_t>(d->epoch) + need >= 0xfffffff0ull) {
    cudaMemsetAsync(d->mem, 0, d->ll_bytes, st);
    d->epoch = 1;
  }
  a.epoch_base = d->epoch;
  d->epoch += static_cast<uint32_t>(need);
  d->last_tag = a.epoch_base;
  a.timeout_ns = g_timeout_ns;
  a.ws = d->ws;
  if (a.num_steps > 1) cudaMemsetAsync(d->ws.kv_ready, 0, sizeof(uint32_t), st);
  void *args[] = {&a};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<void *>(decode_kernel),
                                              dim3(d->num_sms), dim3(NTHREADS), args, smem_bytes(), st);
  if (e != cudaSuccess) return fail_msg(20, "decode kernel launch: %s", cudaGetErrorString(e));
  return 0;
}

}  // namespace

extern "C" {

int qwen_b200_abi_version(void) { return QWEN_B200_ABI_VERSION; }

int qwen_b200_last_error(char *msg, int msg_len) {
  if (msg && msg_len > 0) {
    strncpy(msg, t_msg, msg_len - 1);
    msg[msg_len - 1] = 0;
  }
  return t_err;
}

void qwen_b200_set_wait_timeout_ns(long long ns) { g_timeout_ns = ns > 0 ? ns : 2000000000LL; }

int qwen_b200_device_status(int device, uint64_t *detail) {
  if (device < 0 || device >= 64) return -1;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int rc = 0;
  uint64_t word = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DevState &d = g_dev[device];
    if (d.ready) {
      cudaDeviceSynchronize();
      if (cudaMemcpy(&word, d.ws.err, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess) rc = -2;
      else if (static_cast<uint32_t>(word >> 32) == d.last_tag && (word & 0xffffffffull))
        rc = static_cast<int>((word >> 24) & 0xff);
    }
  }
  if (detail) *detail = word;
  cudaSetDevice(prev);
  return rc;
}

void launch_ldg_decode_direct(int input_token_id, int *output_token_id, const void *embed_weight,
                              const LDGLayerWeight *layer_weights, const void *final_norm_weight,
                              const void *lm_head_weight, const void *cos_table,
                              const void *sin_table, void *k_cache, void *v_cache,
                              void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
                              void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate,
                              void *g_normalized, void *block_max_vals, void *block_max_idxs,
                              int num_layers, int position, int max_seq_len, float attn_scale,
                              void *stream) {
  DecodeArgs a{};
  a.embed = static_cast<const __half *>(embed_weight);
  a.layers = layer_weights;
  a.final_norm = static_cast<const __half *>(final_norm_weight);
  a.lm_head = static_cast<const __half *>(lm_head_weight);
  a.cos_t = static_cast<const __half *>(cos_table);
  a.sin_t = static_cast<const __half *>(sin_table);
  a.k_cache = static_cast<__half *>(k_cache);
  a.v_cache = static_cast<__half *>(v_cache);
  a.hidden = static_cast<__half *>(hidden_buffer);
  a.act = static_cast<float *>(g_activations);
  a.res = static_cast<float *>(g_residual);
  a.q = static_cast<__half *>(g_q);
  a.k = static_cast<__half *>(g_k);
  a.v = static_cast<__half *>(g_v);
  a.attn_out = static_cast<__half *>(g_attn_out);
  a.inter = static_cast<float *>(g_mlp_intermediate);
  a.norm_out = static_cast<float *>(g_normalized);
  a.bmax_vals = static_cast<float *>(block_max_vals);
  a.bmax_idxs = static_cast<int *>(block_max_idxs);
  a.out_tokens = output_token_id;
  a.num_layers = num_layers;
  a.start_pos = position;
  a.max_seq = max_seq_len;
  a.num_steps = 1;
  a.first_token = input_token_id;
  a.attn_scale = attn_scale;
  launch_decode(a, static_cast<cudaStream_t>(stream));
}

void launch_ldg_generate_nosync(int first_token_id, int num_steps, const void *embed_weight,
                                const LDGLayerWeight *layer_weights, const void *final_norm_weight,
                                const void *lm_head_weight, const void *cos_table,
                                const void *sin_table, void *k_cache, void *v_cache,
                                void *hidden_buffer, void *g_activations, void *g_residual,
                                void *g_q, void *g_k, void *g_v, void *g_attn_out,
                                void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
                                void *block_max_idxs, int *output_log, int num_layers,
                                int start_position, int max_seq_len, float attn_scale,
                                void *stream) {
  DecodeArgs a{};
  a.embed = static_cast<const __half *>(embed_weight);
  a.layers = layer_weights;
  a.final_norm = static_cast<const __half *>(final_norm_weight);
  a.lm_head = static_cast<const __half *>(lm_head_weight);
  a.cos_t = static_cast<const __half *>(cos_table);
  a.sin_t = static_cast<const __half *>(sin_table);
  a.k_cache = static_cast<__half *>(k_cache);
  a.v_cache = static_cast<__half *>(v_cache);
  a.hidden = static_cast<__half *>(hidden_buffer);
  a.act = static_cast<float *>(g_activations);
  a.res = static_cast<float *>(g_residual);
  a.q = static_cast<__half *>(g_q);
  a.k = static_cast<__half *>(g_k);
  a.v = static_cast<__half *>(g_v);
  a.attn_out = static_cast<__half *>(g_attn_out);
  a.inter = static_cast<float *>(g_mlp_intermediate);
  a.norm_out = static_cast<float *>(g_normalized);
  a.bmax_vals = static_cast<float *>(block_max_vals);
  a.bmax_idxs = static_cast<int *>(block_max_idxs);
  a.out_tokens = output_log;
  a.num_layers = num_layers;
  a.start_pos = start_position;
  a.max_seq = max_seq_len;
  a.num_steps = num_steps;
  a.first_token = first_token_id;
  a.attn_scale = attn_scale;
  launch_decode(a, static_cast<cudaStream_t>(stream));
}

int qwen_b200_selftest_wait_timeout(long long timeout_ns, void *stream) {
  t_err = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *mem = nullptr;
  if (cudaMalloc(&mem, 64) != cudaSuccess) return -1;
  cudaMemsetAsync(mem, 0, 64, st);
  uint64_t *word = static_cast<uint64_t *>(mem);
  unsigned long long *err = reinterpret_cast<unsigned long long *>(word + 4);
  const uint32_t tag = 0x5e1f7e57u;
  selftest_wait_kernel<<<1, 32, 0, st>>>(word, err, timeout_ns, tag);
  cudaError_t e = cudaStreamSynchronize(st);
  unsigned long long v = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost);
  cudaFree(mem);
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (static_cast<uint32_t>(v >> 32) != tag) return 0;
  return static_cast<int>((v >> 24) & 0xff);
}

}  // extern "C"
