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
//  * 8 consumer warps compute each stage on the bytes already in shared
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
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "ptx.cuh"
#include "qwen_b200.h"

namespace qb200 {

constexpr int H = 1024, IM = 3072, NQ = 16, NKV = 8, HD = 128;
constexpr int QS = NQ * HD, KVS = NKV * HD, QKV_ROWS = QS + 2 * KVS;
constexpr int VOCAB = 151936;
constexpr float RMS_EPS = 1e-6f;

constexpr int NCW = 8;                // consumer warps
constexpr int NCT = NCW * 32;         // consumer threads
constexpr int NTHREADS = NCT + 32;    // + one producer warp
// A ring piece carries up to PIECE_BYTES of payload: 6 weight rows of
// K=1024, 3 of 2048, 2 of 3072, 48 KV-cache rows or 6 lm_head rows, stored
// densely (one bulk copy per piece).
constexpr int PIECE_BYTES = 12288;
constexpr int SLOT_BYTES = PIECE_BYTES;
constexpr int NSLOTS = 16;
constexpr int BATCH_MAX = 8;          // pieces per consumer batch (<= NSLOTS/2)
// Bulk copies in flight per CTA (issued, not yet landed).  The ring may hold
// up to NSLOTS landed pieces, but more bytes in flight than bandwidth x
// latency only queue in the memory system and delay every other access on
// the critical path (handoff words, norm weights).
#ifndef QB200_INFLIGHT
#define QB200_INFLIGHT 8
#endif
constexpr int INFLIGHT = QB200_INFLIGHT;
constexpr int KV_ROW_BYTES = HD * 2;
constexpr int KV_TOK_PER_PIECE = PIECE_BYTES / KV_ROW_BYTES;  // 48
constexpr int SC_PAIRS = 3;                                  // K/V piece pairs per super-chunk
constexpr int SC_TOK = SC_PAIRS * KV_TOK_PER_PIECE;          // 144
constexpr int SPLIT_MIN_TOK = 64;
constexpr int MAX_SPLITS = 32;
// Splits the combine gathers in one round: C / NKV for a 148-SM B200.
constexpr int MAX_SPLITS_B200 = 18;
constexpr int MIN_CTAS = 128, MAX_CTAS = 256;  // stage G gathers one CTA per consumer thread
constexpr int MAX_OWN = 64;           // rows per CTA of o_proj/down/gate-up
constexpr int MAX_STAGE_ROWS = 48;    // GEMV rows per CTA and stage (C >= 128: QKV 32, gate+up 48)
constexpr int MAX_TILES = MAX_STAGE_ROWS / 16;
constexpr uint32_t BAR_ID = 1;
// Layers whose norm-weight pointers the consumers keep in shared memory (read
// once per launch instead of a dependent global load at every stage start).
constexpr int NTAB_LAYERS = 32;

enum Status : uint32_t {
  ST_OK = 0,
  ST_TIMEOUT_LL = 1,
  ST_TIMEOUT_FULL = 2,
  ST_TIMEOUT_EMPTY = 3,
  ST_TIMEOUT_KV = 4,
  ST_MISALIGNED = 5,
  ST_BAD_TOKEN = 6,
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
  uint64_t *token;   // [1] the step's token, published by CTA 0
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
  const int *first_token_dev;  // when set: the first token is read from device memory
  float *logits_out;           // when set: fp32 [VOCAB] logits of the last step
  float attn_scale;
  uint32_t epoch_base;
  long long timeout_ns;
  Workspace ws;
  // Optional stage timeline (null = off): [cta][step < trace_steps][layer 0..L][TR_N]
  // %globaltimer stamps written by consumer thread 0 and the producer thread.
  unsigned long long *trace;
  int trace_steps;
};

enum TraceEv : int {
  TR_A0 = 0, TR_A1, TR_A2, TR_B0, TR_B1, TR_B2, TR_C0, TR_C1, TR_C2, TR_D0, TR_D1, TR_D2,
  TR_E0, TR_E1, TR_E2, TR_P_START, TR_P_STALL, TR_P_END,
  TR_A3, TR_B3, TR_C3, TR_D3, TR_E3,   // CTA-wide stage end (after a consumer barrier)
  TR_FW,                               // cumulative ns thread 0 waited on ring data
  TR_B_KV, TR_B_SC, TR_B_PV, TR_B_PART, TR_B_CMB,  // stage B: K/V landed, scores, P.V, partials out, (m, l) in
  TR_E_CYC0, TR_E_CYC1, TR_E_CYC2,     // stage E SM clock (clock64): after wait, after the k loop, end
  TR_B_CYC0, TR_B_CYC1, TR_B_CYC2, TR_B_CYC3,  // stage B SM clock: scores done, softmax, P.V loop, ring release
  TR_A_PIECES, TR_A_GATHER,            // stage A: warp 0 saw all ring pieces, thread 0 gathered the hidden words
  TR_P_A_LAST,                         // producer: issue of this layer's last stage-A piece
  TR_N = 40
};
// Row l == num_layers holds the final stages: F entry / F after its wait /
// F end / G after its wait / G end at events 0..4.

__device__ __forceinline__ unsigned long long *trace_row(const DecodeArgs &a, int s, int l) {
  if (a.trace == nullptr || s >= a.trace_steps) return nullptr;
  return a.trace + ((static_cast<size_t>(blockIdx.x) * a.trace_steps + s) * (a.num_layers + 1) + l) * TR_N;
}

__device__ __forceinline__ void trace_mark(unsigned long long *row, int ev) {
  if (row != nullptr && threadIdx.x == 0) row[ev] = globaltimer_ns();
}

__device__ __forceinline__ void trace_clock(unsigned long long *row, int ev) {
  if (row != nullptr && threadIdx.x == 0) row[ev] = clock64();
}

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
  __half q_rot[2][HD];     // rotated q of the two heads (fp16, as upstream rounds it)
  float wred[NCW][2];      // per-warp score max per head
  float wsum[NCW];         // per-warp softmax sum
  __align__(16) float pvp[NCW][2][HD];  // P.V partials of the eight token slices [slice][head][dim]
  __align__(16) __half k_fresh[HD];
  __align__(16) float sc[SC_TOK + 1][2];  // scores, then softmax weights [token][head]
  float att_m[2], att_l[2], att_alpha[2];
  float cmb_m[2][MAX_SPLITS], cmb_l[2][MAX_SPLITS];  // split (max, sum) per head
  float cmb_f[2][MAX_SPLITS];                        // split rescale factor exp(m_j - M) per head
  uint32_t rowaddr[MAX_TILES * 16];  // smem address of each GEMV stage row (padding rows -> row 0)
  int rowinfo[MAX_TILES * 16];       // matrix row | kind << 24
  // Stage A's row plan (made once per launch, see plan_rows_a):
  uint32_t plan_po[MAX_TILES * 16];  // stage row -> piece << 16 | byte offset in the piece (~0: padding)
  int plan_info[MAX_TILES * 16];     // stage row -> matrix row | kind << 24 (-1: padding)
  int plan_np, plan_total;           // stage A's pieces and rows
  int plan_o_lo, plan_o_n;           // this CTA's o_proj / down rows (layer 0 copies their embedding)
  const __half *ntab[NTAB_LAYERS][4];  // norm weights of the first layers: input, q, k, post
  float mred[NCW][MAX_TILES * 16];   // per-warp partial dot products
  unsigned long long trace_fullwait;
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
  unsigned long long *fullwait;  // tracing only: ns thread 0 spent waiting on ring data
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
__device__ __noinline__ void set_error_word(unsigned long long *err, volatile uint32_t *abort_flag,
                                            uint32_t tag, uint32_t code, uint32_t where) {
  const unsigned long long mine = (static_cast<unsigned long long>(tag) << 32) |
                                  (static_cast<unsigned long long>(code & 0xff) << 24) |
                                  (static_cast<unsigned long long>(where & 0xff) << 16) |
                                  (blockIdx.x & 0xffff);
  unsigned long long cur = atomicAdd(err, 0ull);
  while (static_cast<uint32_t>(cur >> 32) != tag) {
    const unsigned long long prev = atomicCAS(err, cur, mine);
    if (prev == cur) break;
    cur = prev;
  }
  *abort_flag = 1;
}

__device__ __forceinline__ void set_error(const WaitCtx &w, uint32_t code, uint32_t where) {
  set_error_word(w.err, w.abort, w.tag, code, where);
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

// backoff: sleep between polls (the producer's wait for a free ring slot,
// which is off the critical path; a hot poll would take issue slots from the
// consumer warps on its SM sub-partition).
__device__ __noinline__ bool wait_mbar_slow(WaitCtx w, uint64_t *bar, uint32_t parity,
                                            uint32_t code, uint32_t where, bool backoff = false) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) {
      if (w.fullwait != nullptr && threadIdx.x == 0) *w.fullwait += globaltimer_ns() - t0;
      return true;
    }
    if (backoff) __nanosleep(200);
    if ((it & 63) == 0 && !wait_ok(w, t0, code, where)) return false;
  }
}

__device__ __forceinline__ bool wait_mbar(const WaitCtx &w, uint64_t *bar, uint32_t parity,
                                          uint32_t code, uint32_t where) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_mbar_slow(w, bar, parity, code, where);
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
#pragma unroll 1
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
      if ((it & 31) == 0 && !wait_ok(w, t0, ST_TIMEOUT_LL, where)) {
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
// n * c < 2^31 for every partition here (n <= 151936, c <= 512).
__device__ __forceinline__ int part_lo(int n, int C, int c) { return (n * c) / C; }

struct Piece {
  const char *src;
  uint32_t bytes;
  int row0;   // first matrix row (or first token) in the piece
  int nrows;
  int kind;   // QKV: 0 q 1 k 2 v; gate/up: 0 gate 1 up; KV: 0 K 1 V
};

__device__ __forceinline__ int npieces(int nrows, int row_bytes) {
  const int rpp = PIECE_BYTES / row_bytes;
  return (nrows + rpp - 1) / rpp;
}


__device__ __forceinline__ Piece seg_piece(const void *base, int row_bytes, int row0, int nrows,
                                           int i, int kind) {
  const int rpp = PIECE_BYTES / row_bytes;
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
  const int smax = min(MAX_SPLITS_B200, C / NKV);
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
  w.fullwait = a.trace != nullptr ? &sm.trace_fullwait : nullptr;
  w.abort = &sm.abort;
  w.err = a.ws.err;
  w.tag = a.epoch_base;
  w.timeout_ns = a.timeout_ns;
  return w;
}

// ------------------------------------------------------------- producer
// Issues ring piece n (one bulk copy) after its slot was released and piece
// n-INFLIGHT landed.  One copy per piece, never one per weight row: the copy
// engine's per-copy cost caps a CTA at about 24 GB/s with 2 KB copies
// against about 47 GB/s with 12 KB copies (measured on B200).
__device__ __noinline__ bool issue_piece(Smem &sm, WaitCtx w, uint32_t n, const char *src,
                                         uint32_t bytes, uint64_t pol, unsigned long long *stall_ns) {
  const int slot = n % NSLOTS;
  const uint32_t round = n / NSLOTS;
  if (round > 0 && !mbar_try_wait(&sm.empty[slot], (round - 1) & 1)) {
    const uint64_t t0 = stall_ns ? globaltimer_ns() : 0;
    if (!wait_mbar_slow(w, &sm.empty[slot], (round - 1) & 1, ST_TIMEOUT_EMPTY, W_PROD, true)) return false;
    if (stall_ns) *stall_ns += globaltimer_ns() - t0;
  }
  if (n >= static_cast<uint32_t>(INFLIGHT)) {
    // Piece n-INFLIGHT must have landed; its slot is reused only by piece
    // n-INFLIGHT+NSLOTS > n, so this phase cannot have been overtaken.
    const uint32_t m = n - INFLIGHT;
    if (!wait_mbar(w, &sm.full[m % NSLOTS], (m / NSLOTS) & 1, ST_TIMEOUT_FULL, W_PROD)) return false;
  }
  if ((reinterpret_cast<uintptr_t>(src) & 15u) || (bytes & 15u) || bytes == 0 ||
      bytes > static_cast<uint32_t>(PIECE_BYTES)) {
    set_error(w, ST_MISALIGNED, W_PROD);
    return false;
  }
  mbar_arrive_expect_tx(&sm.full[slot], bytes);
  bulk_g2s(sm.ring[slot], src, bytes, &sm.full[slot], pol);
  return true;
}

__device__ __forceinline__ void producer(const DecodeArgs &a, Smem &sm) {
  const int C = gridDim.x, c = blockIdx.x, L = a.num_layers;
  const WaitCtx w = make_wait(a, sm);
  const uint64_t pol = policy_evict_first();
  uint32_t n = 0;
  bool ok = true;

  unsigned long long stall_ns = 0;
  const bool tracing = a.trace != nullptr;
  auto prefetch = [&](const Piece &P) {
    if (!((reinterpret_cast<uintptr_t>(P.src) & 15u) || (P.bytes & 15u) || P.bytes == 0))
      bulk_prefetch_l2(P.src, P.bytes);
  };
  auto issue = [&](const Piece &P) -> bool {
    const bool ok = issue_piece(sm, w, n, P.src, P.bytes, pol, tracing ? &stall_ns : nullptr);
    ++n;
    return ok;
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
      unsigned long long *tr = trace_row(a, s, l);
      if (tr) {
        tr[TR_P_START] = globaltimer_ns();
        tr[TR_P_STALL] = stall_ns;
      }
      for (int i = 0; i < qg.total && ok; ++i) ok = issue(qkv_piece(qg, lp, i));
      if (tr) tr[TR_P_A_LAST] = globaltimer_ns();
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
      // The next layer's q|k|v pieces get ring slots only when stage D
      // releases its pieces, a few microseconds before stage A needs them:
      // start pulling them into L2 now, so those copies are served from L2.
      // (Prefetching the other stages' pieces too was slower: every prefetch
      // is one more operation for the SM's copy engine.)
      if (l + 1 < L) {
        const LayerPtrs nx = load_layer(a.layers, l + 1);
        for (int i = 0; i < qg.total; ++i) prefetch(qkv_piece(qg, nx, i));
      }
      if (tr) tr[TR_P_END] = globaltimer_ns();
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
// Row table of a GEMV stage whose `count` pieces start at ring piece n:
// thread j (< MAX_TILES*16) records the smem address of stage row j, and its
// matrix row and kind.  Rows past the end point at row 0 (their results are
// ignored).  Each thread writes and later reads only its own entry, so no
// barrier is needed between one stage's epilogue and the next table.
template <int K, class GetPiece>
__device__ __forceinline__ int prep_rows(Smem &sm, uint32_t n, int count, GetPiece get_piece) {
  constexpr int PITCH = 2 * K;
  const int j = threadIdx.x;
  int total = 0;
  uint32_t addr0 = 0, my_addr = 0;
  int my_info = 0;
  bool found = false;
  for (int i = 0; i < count; ++i) {
    const Piece P = get_piece(i);
    const uint32_t base = smem_u32(sm.ring[(n + i) % NSLOTS]);
    if (i == 0) addr0 = base;
    if (!found && j < total + P.nrows) {
      my_addr = base + (j - total) * PITCH;
      my_info = (P.row0 + (j - total)) | (P.kind << 24);
      found = true;
    }
    total += P.nrows;
  }
  if (j < MAX_TILES * 16) {
    sm.rowaddr[j] = found ? my_addr : addr0;
    sm.rowinfo[j] = found ? my_info : -1;
  }
  return total;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// s0 += lo(w) * lo(x) and s1 += hi(w) * hi(x) for two fp16 pairs packed in
// 32-bit words, as sm_100's mixed-precision fma: the fp16 operands widen to
// fp32 exactly, their product is exact in fp32 and each sum is rounded once,
// which is fmaf on the widened values (the same bits), without separate
// conversion instructions.
__device__ __forceinline__ void fma_h2(float &s0, float &s1, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "mov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.f16 %1, wh, xh, %1;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "r"(w), "r"(x));
}
// s += lo(w) * lo(x), then s += hi(w) * hi(x) (one chain, same rounding).
__device__ __forceinline__ void fma_h2_chain(float &s, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
      : "+f"(s)
      : "r"(w), "r"(x));
}

// Batch-1 GEMV of a stage with up to RMAX rows (QKV: <= 32, gate/up: <= 48
// per CTA) on the CUDA cores: y[j] = W[j,:] . x for the `total` rows of the
// row table (pieces n .. n+count-1, all landed before use).  Warp w takes
// stage rows w, w + 8, ...; its lanes split K into 16-byte chunks (x's chunks
// kept in registers), so each weight byte is read from
// shared memory once, by consecutive lanes (no bank conflict, no row
// padding).  Products use the mixed-precision fma (fma_h2); each lane keeps two
// fp32 chains, then a fixed-order warp sum: results are deterministic.
// epi(kind, matrix_row, dot) runs on thread j for stage row j < total.
template <int K, int RMAX, class Epi>
__device__ __forceinline__ void gemv_wr(Smem &sm, uint32_t &n, int count, int total,
                                        const __half *x, Epi epi) {
  constexpr int CH = K / 8 / 32;       // 16-byte chunks per lane
  constexpr int RPW = RMAX / NCW;      // rows per warp
  static_assert(K % 256 == 0 && RMAX % NCW == 0 && RMAX <= MAX_TILES * 16, "gemv_wr shape");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint4 xw[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) xw[i] = *reinterpret_cast<const uint4 *>(x + 8 * (lane + 32 * i));
  float res[RPW];
#pragma unroll
  for (int q = 0; q < RPW; ++q) {
    // Rows >= total are padding entries pointing at row 0 (results unused).
    const uint32_t row = sm.rowaddr[warp + NCW * q];
    uint4 wv[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) wv[i] = lds_u4(row + 16u * (lane + 32 * i));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      fma_h2(s0, s1, wv[i].x, xw[i].x);
      fma_h2(s0, s1, wv[i].y, xw[i].y);
      fma_h2(s0, s1, wv[i].z, xw[i].z);
      fma_h2(s0, s1, wv[i].w, xw[i].w);
    }
    res[q] = s0 + s1;
  }
#pragma unroll
  for (int q = 0; q < RPW; ++q) res[q] = warp_sum(res[q]);
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < RPW; ++q) sm.mred[0][warp + NCW * q] = res[q];
  }
  named_bar_sync(BAR_ID, NCT);
  // Release the pieces: every warp arrives once per piece (lane i on piece i).
  if (lane < count) mbar_arrive(&sm.empty[(n + lane) % NSLOTS]);
  n += count;
  if (tid < total) {
    const int info = sm.rowinfo[tid];
    epi(info >> 24, info & 0xffffff, sm.mred[0][tid]);
  }
}

__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// GEMV of a stage with at most 8 rows (o_proj, down: 1024 rows over >= 128
// CTAs) on the CUDA cores.  A tensor-core tile would waste 15 of its 16 rows
// and read the padding from shared memory; here every weight byte is read
// once: thread t takes the 4-element chunks t, t + 256, ... of every row (x's
// chunks stay in registers), products are exact in fp32 and summed in fp32.
// The per-row partials are reduce-scattered across the warp (lanes 4r..4r+3
// end with row r), then added over the warps in a fixed order, so results
// are deterministic.  epi(kind, matrix_row, dot) runs on thread j < total.
template <int K, class Epi>
__device__ __forceinline__ void gemv_cc(Smem &sm, uint32_t &n, int count, int total, const __half *x,
                                        Epi epi, unsigned long long *tr = nullptr) {
  constexpr int CH = K / 4 / NCT;  // chunks per thread
  static_assert(K % (4 * NCT) == 0, "K must split into 4-element chunks over the consumer threads");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint2 xw[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) xw[i] = *reinterpret_cast<const uint2 *>(x + 4 * (tid + NCT * i));
  // All loads first, with no branch between them (rows >= total are
  // padding entries that point at row 0: valid memory, results unused).
  uint2 wv[8][CH];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const uint32_t row = sm.rowaddr[r];
#pragma unroll
    for (int i = 0; i < CH; ++i) wv[r][i] = lds_u2(row + 8u * (tid + NCT * i));
  }
  float acc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      fma_h2_chain(s, wv[r][i].x, xw[i].x);
      fma_h2_chain(s, wv[r][i].y, xw[i].y);
    }
    acc[r] = s;
  }
  trace_clock(tr, TR_E_CYC1);
  // Reduce-scatter over the warp: offsets 16, 8, 4 halve the rows a lane
  // keeps; offsets 2, 1 finish the sum of the four lanes sharing a row.
  float v4[4], v2[2];
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float keep = b16 ? acc[j + 4] : acc[j], send = b16 ? acc[j] : acc[j + 4];
    v4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float keep = b8 ? v4[j + 2] : v4[j], send = b8 ? v4[j] : v4[j + 2];
    v2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float v;
  {
    const float keep = b4 ? v2[1] : v2[0], send = b4 ? v2[0] : v2[1];
    v = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  if ((lane & 3) == 0) sm.mred[warp][(b16 ? 4 : 0) + (b8 ? 2 : 0) + (b4 ? 1 : 0)] = v;
  named_bar_sync(BAR_ID, NCT);
  // Release the pieces: every warp arrives once per piece (lane i on piece i).
  if (lane < count) mbar_arrive(&sm.empty[(n + lane) % NSLOTS]);
  n += count;
  if (tid < total) {
    float dot = 0.f;
#pragma unroll
    for (int ww = 0; ww < NCW; ++ww) dot += sm.mred[ww][tid];
    const int info = sm.rowinfo[tid];
    epi(info >> 24, info & 0xffffff, dot);
  }
}

// Waits until the `count` (<= 32) ring pieces from n on have landed: lane i
// of warp 0 waits on piece i, so the waits overlap.  Called before a stage's
// first barrier, which then orders the pieces' shared memory before every
// consumer thread's reads.
__device__ __forceinline__ bool wait_pieces(Smem &sm, const WaitCtx &w, uint32_t n, int count,
                                            uint32_t where) {
  const int tid = threadIdx.x;
  if (tid >= count) return true;
  const uint32_t pn = n + tid;
  return wait_mbar(w, &sm.full[pn % NSLOTS], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, where);
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

// ======================================================================
// Consumer warps (NCW = 8, all stages inlined into the kernel: no calls, no
// stack, kernel parameters read straight from the parameter space).
// ======================================================================

struct St {
  uint32_t n;  // ring pieces consumed so far
  bool fail;   // this thread saw a failed wait
};

__device__ __forceinline__ const __half *layer_ptr(const LDGLayerWeight *t, int l, int idx) {
  return reinterpret_cast<const __half *>(
      __ldg(reinterpret_cast<const unsigned long long *>(t + l) + idx));
}

// Norm weights k (0 input, 1 q, 2 k, 3 post-attention) of layer l: the table
// entry packed at LDGLayerWeight slot 0 / 4 / 5 / 7.
__device__ __forceinline__ int norm_slot(int k) { return k == 0 ? 0 : (k == 1 ? 4 : (k == 2 ? 5 : 7)); }
__device__ __forceinline__ const __half *norm_ptr(const Smem &sm, const DecodeArgs &a, int l, int k) {
  return l < NTAB_LAYERS ? sm.ntab[l][k] : layer_ptr(a.layers, l, norm_slot(k));
}

struct Rows {
  int lo, n;
};
__device__ __forceinline__ Rows rows_of(int total, int C, int c) {
  Rows r;
  r.lo = part_lo(total, C, c);
  r.n = part_lo(total, C, c + 1) - r.lo;
  return r;
}

// Sum of a per-thread float over the consumer threads: warp reduce, one
// named barrier that also ORs the abort predicate (returned in *abort), then
// every thread adds the NCW warp sums in the same order.
__device__ __forceinline__ float block_sum(Smem &sm, float v, bool pred, bool *abort) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sm.red[threadIdx.x >> 5] = v;
  *abort = named_bar_or(BAR_ID, NCT, pred);
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NCW; ++i) t += sm.red[i];
  return t;
}

// Stage A's row table, planned once per launch.  Its input (the hidden words
// of the previous layer's stage E) is ready a few hundred ns after the stage
// starts, so walking the pieces there (qkv_geom + prep_rows, ~0.7 us measured
// on B200) sat on the critical path.  The other GEMV stages start well before
// their inputs arrive and keep prep_rows: planning them too made the kernel
// slower (3-5 %), their handoff polls then starting earlier and loading the
// memory system while the producing stage still ran.
// Thread j (< MAX_TILES*16) records which piece holds stage row j, the row's
// byte offset in it, and its matrix row and kind (padding: row 0 of piece 0).
__device__ __forceinline__ void plan_rows_a(Smem &sm, int C, int c) {
  const QkvGeom qg = qkv_geom(C, c);
  const LayerPtrs lp{};  // consumers only need row ranges, not addresses
  const int j = threadIdx.x;
  int total = 0;
  uint32_t po = ~0u;
  int info = -1;
  for (int i = 0; i < qg.total; ++i) {
    const Piece P = qkv_piece(qg, lp, i);
    if (po == ~0u && j < total + P.nrows) {
      po = (static_cast<uint32_t>(i) << 16) | static_cast<uint32_t>((j - total) * 2 * H);
      info = (P.row0 + (j - total)) | (P.kind << 24);
    }
    total += P.nrows;
  }
  if (j < MAX_TILES * 16) {
    sm.plan_po[j] = po;
    sm.plan_info[j] = info;
  }
  if (j == 0) {
    const Rows o = rows_of(H, C, c);
    sm.plan_np = qg.total;
    sm.plan_total = total;
    sm.plan_o_lo = o.lo;
    sm.plan_o_n = o.n;
  }
}

// prep_rows for stage A from its plan, pieces starting at ring piece n.
__device__ __forceinline__ int prep_rows_a(Smem &sm, uint32_t n) {
  const int j = threadIdx.x;
  if (j < MAX_TILES * 16) {
    const uint32_t po = sm.plan_po[j];
    const uint32_t piece = po == ~0u ? 0u : (po >> 16), off = po == ~0u ? 0u : (po & 0xffffu);
    sm.rowaddr[j] = smem_u32(sm.ring[0]) + ((n + piece) % NSLOTS) * SLOT_BYTES + off;
    sm.rowinfo[j] = sm.plan_info[j];
  }
  return sm.plan_total;
}

// ---------------------------------------------------------------- stage A
// Input RMSNorm (megakernel.cu:806-847) + fused QKV GEMV (:242-291).
__device__ __forceinline__ bool stage_a(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        int l, int token, uint32_t ep, unsigned long long *tr) {
  const int tid = threadIdx.x;
  trace_mark(tr, TR_A0);
  const int np = sm.plan_np;
  const int total = prep_rows_a(sm, st.n);
  // Norm weights: loaded now, converted only where they are used (after the
  // hidden-vector gather), so their latency hides behind the gather.
  const __half *nw = norm_ptr(sm, a, l, 0);
  __half wr[4];
  float h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wr[i] = __ldg(nw + tid + NCT * i);
  st.fail |= !wait_pieces(sm, w, st.n, np, W_A);
  if (tr != nullptr) {
    __syncwarp();
    trace_mark(tr, TR_A_PIECES);
  }
  if (l == 0) {
    const __half *emb = a.embed + static_cast<size_t>(token) * H;
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __half2float(__ldg(emb + tid + NCT * i));
    if (tid < sm.plan_o_n) sm.hid_own[tid] = __ldg(emb + sm.plan_o_lo + tid);
  } else {
    uint32_t u[4];
    st.fail |= !ll_gather<4>(w, [&](int i) { return a.ws.hidden + tid + NCT * i; }, ep - 1, u, W_A);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __half2float(u2h(u[i]));
    trace_mark(tr, TR_A_GATHER);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(h[i], h[i], ss);
  bool abort;
  const float tot = block_sum(sm, ss, st.fail || sm.abort, &abort);
  if (abort) return true;
  trace_mark(tr, TR_A1);
  const float inv = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
#pragma unroll
  for (int i = 0; i < 4; ++i) sm.xa[tid + NCT * i] = __float2half(h[i] * (inv * __half2float(wr[i])));
  named_bar_sync(BAR_ID, NCT);
  gemv_wr<H, 32>(
      sm, st.n, np, total, sm.xa,
      [&](int kind, int row, float dot) {
        const __half hv = __float2half(dot);
        const int vrow = (kind == 0 ? 0 : (kind == 1 ? QS : QS + KVS)) + row;
        ll_store(a.ws.qkv + vrow, h2u(hv), ep);
        __half *dst = kind == 0 ? a.q : (kind == 1 ? a.k : a.v);
        dst[row] = hv;
      });
  trace_mark(tr, TR_A2);
  return false;
}

// ---------------------------------------------------------------- stage B
// q/k RMSNorm + RoPE, KV-cache write, split-KV GQA attention over the cache
// and the combine of the splits (megakernel.cu:308-553).
__device__ __forceinline__ bool stage_b(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        const AttnGeom &ag, int l, int p, uint32_t ep,
                                        unsigned long long *tr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = ag.g;
  trace_mark(tr, TR_B0);
  // Loads that do not depend on this layer's activations go first.
  const bool rope_warp = warp < 2 || (ag.last && warp == 2);
  __half nwv[4], csv[4], snv[4];  // converted where used, after the q|k|v gather
  if (rope_warp) {
    const __half *nw = norm_ptr(sm, a, l, warp < 2 ? 1 : 2);
    const __half *cosp = a.cos_t + static_cast<size_t>(p) * HD;
    const __half *sinp = a.sin_t + static_cast<size_t>(p) * HD;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int i = lane + 32 * it;
      const int ri = it < 2 ? i : i - HD / 2;
      nwv[it] = __ldg(nw + i);
      csv[it] = __ldg(cosp + ri);
      snv[it] = __ldg(sinp + ri);
    }
  }
  // Warp 0 / 1 gathers q head 2g / 2g+1 and rotates it right away; on the
  // split that holds the new token, warp 2 also takes k head g (rotated into
  // k_fresh) and warp 3 v head g (raw).  Other splits read no k / v words.
  if (tid < 2) {
    sm.att_m[tid] = -INFINITY;
    sm.att_l[tid] = 0.f;
  }
  if (warp < 2 || (ag.last && warp < 4)) {
    const int word0 = warp < 2 ? HD * (2 * g + warp) : (warp == 2 ? QS + HD * g : QS + KVS + HD * g);
    uint32_t u[4];
    st.fail |= !ll_gather<4>(w, [&](int it) { return a.ws.qkv + word0 + lane + 32 * it; }, ep, u, W_B);
    if (warp == 3) {
#pragma unroll
      for (int it = 0; it < 4; ++it) sm.qkv_raw[3 * HD + lane + 32 * it] = u2h(u[it]);
    } else {
      // q/k RMSNorm (eps 1e-6) + rotate-half RoPE, megakernel.cu:345-434.
      float xv[4], ss = 0.f;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        xv[it] = __half2float(u2h(u[it]));
        ss = fmaf(xv[it], xv[it], ss);
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / static_cast<float>(HD) + 1e-6f);
      float vals[4];
#pragma unroll
      for (int it = 0; it < 4; ++it) vals[it] = __fmul_rn(__fmul_rn(xv[it], inv), __half2float(nwv[it]));
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int i = lane + 32 * it;
        const float c = __half2float(csv[it]), sn = __half2float(snv[it]);
        const float r = it < 2 ? __fsub_rn(__fmul_rn(vals[it], c), __fmul_rn(vals[it + 2], sn))
                               : __fadd_rn(__fmul_rn(vals[it - 2], sn), __fmul_rn(vals[it], c));
        const __half hr = __float2half(r);
        if (warp < 2) sm.q_rot[warp][i] = hr;
        else sm.k_fresh[i] = hr;
      }
    }
  }
  if (named_bar_or(BAR_ID, NCT, st.fail || sm.abort)) return true;
  trace_mark(tr, TR_B1);

  // A fragments of q (m16n8k16, rows 0/1 = the two q heads, other rows 0).
  // The k order of the MMAs is a permutation of the 128 dims that matches the
  // 16-byte K loads below: in 32-dim block b, lane (row, c = lane & 3) holds
  // dims 32b + 8c + 4s + {0,1} (low k half) and 32b + 8c + 4s + {2,3} (high k
  // half) for k step 2b + s.  A dot product does not depend on the order of
  // its terms' k steps; every product is exact and sums are fp32.
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int dim = 32 * (kk >> 1) + 8 * (lane & 3) + 4 * (kk & 1);
    qa[kk][0] = lane < 8 ? *reinterpret_cast<const uint32_t *>(&sm.q_rot[lane >> 2][dim]) : 0u;
    qa[kk][1] = lane < 8 ? *reinterpret_cast<const uint32_t *>(&sm.q_rot[lane >> 2][dim + 2]) : 0u;
  }
  const int hh = tid >> 7;                      // head of this thread in the softmax
  const int dq = lane, ts = warp;               // P.V: dims 4*dq..+3 of both heads, tokens = ts mod 8
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // [head][dim]
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // every thread tracks both heads
  const int total_old = ag.t1 - ag.t0;
  uint32_t n = st.n;
#pragma unroll 1
  for (int sc = 0; sc < ag.nsc; ++sc) {
    const int pair0 = sc * SC_PAIRS;
    const int npair = max(0, min(SC_PAIRS, ag.npairs - pair0));
    const int n_old = max(0, min(SC_TOK, total_old - pair0 * KV_TOK_PER_PIECE));
    const bool fresh = ag.last && (sc == ag.nsc - 1);
    const int ntok = n_old + (fresh ? 1 : 0);
    // This super-chunk's K/V pieces: warp 0 waits, the barrier publishes.
    st.fail |= !wait_pieces(sm, w, n, 2 * npair, W_B);
    named_bar_sync(BAR_ID, NCT);
    if (sc == 0) trace_mark(tr, TR_B_KV);
    // Scores S[h][t] = q_h . k_t on the tensor cores (fp16 inputs, exact
    // products, fp32 accumulation), 8 tokens per tile, tiles over warps.
    float wmax = -INFINITY;  // lanes 0..3: head 0, lanes 4..7: head 1
    const int ntile = (ntok + 7) >> 3;
#pragma unroll 1
    for (int tile = warp; tile < ntile; tile += NCW) {
      const int tok = tile * 8 + (lane >> 2);
      const __half *krow = sm.k_fresh;
      if (tok < n_old) {
        const uint32_t pn = n + 2 * (tok / KV_TOK_PER_PIECE);
        krow = reinterpret_cast<const __half *>(sm.ring[pn % NSLOTS] + (tok % KV_TOK_PER_PIECE) * KV_ROW_BYTES);
      }
      // Lane (token g, c) loads dims 32b + 8c .. +7 of its K row with one
      // 16-byte load per block b.  Rows are 256 B apart, so odd tokens load
      // the blocks in the order 1,0,3,2: each load then reads 4 even rows on
      // one half of the banks and 4 odd rows on the other (no conflict).
      const bool odd = (lane >> 2) & 1;
      uint4 kw[4];
#pragma unroll
      for (int b = 0; b < 4; ++b)
        kw[b] = *reinterpret_cast<const uint4 *>(krow + 32 * (b ^ (odd ? 1 : 0)) + 8 * (lane & 3));
      // Two accumulator chains (the legacy MMA's latency dominates here).
      float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint4 w = odd ? kw[b ^ 1] : kw[b];
        mma16816(d, qa[2 * b][0], 0u, qa[2 * b][1], 0u, w.x, w.y);
        mma16816(e, qa[2 * b + 1][0], 0u, qa[2 * b + 1][1], 0u, w.z, w.w);
      }
      d[0] += e[0];
      d[1] += e[1];
      if (lane < 8) {
        const int t0 = tile * 8 + 2 * (lane & 3);
        const float s0 = d[0] * a.attn_scale, s1 = d[1] * a.attn_scale;
        if (t0 < ntok) {
          sm.sc[t0][lane >> 2] = s0;
          wmax = fmaxf(wmax, s0);
        }
        if (t0 + 1 < ntok) {
          sm.sc[t0 + 1][lane >> 2] = s1;
          wmax = fmaxf(wmax, s1);
        }
      }
    }
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 1));
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 2));
    if (lane == 0 || lane == 4) sm.wred[warp][lane >> 2] = wmax;
    named_bar_sync(BAR_ID, NCT);
    if (sc == 0) {
      trace_mark(tr, TR_B_SC);
      trace_clock(tr, TR_B_CYC0);
    }
    // Softmax (expf as upstream, megakernel.cu:490-494): every thread derives
    // the same running max of both heads; thread (hh, tt) turns its tokens'
    // scores into weights.
    float m_new[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float cmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < NCW; ++i) cmax = fmaxf(cmax, sm.wred[i][h]);
      m_new[h] = fmaxf(m_run[h], cmax);
    }
    float psum = 0.f;
    if (ntok > 0) {
      for (int tt = tid & 127; tt < ntok; tt += 128) {
        const float pr = expf(sm.sc[tt][hh] - m_new[hh]);
        sm.sc[tt][hh] = pr;
        psum += pr;
      }
    }
    psum = warp_sum(psum);
    if (lane == 0) sm.wsum[warp] = psum;
    named_bar_sync(BAR_ID, NCT);
    if (sc == 0) trace_clock(tr, TR_B_CYC1);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float tsum = 0.f;
#pragma unroll
      for (int i = 0; i < NCW / 2; ++i) tsum += sm.wsum[h * (NCW / 2) + i];
      const float alpha = ntok == 0 ? 1.f : (m_run[h] == -INFINITY ? 0.f : expf(m_run[h] - m_new[h]));
      if (ntok > 0) {
        l_run[h] = l_run[h] * alpha + tsum;
        m_run[h] = m_new[h];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[h][i] *= alpha;
    }
    // P.V: thread (dq, ts) adds dims 4*dq..4*dq+3 of both heads over the
    // tokens t = ts mod 8 (a V row is read once for both heads; pieces hold
    // 48 tokens, a multiple of 8, so the residue is the same per piece).
    {
      auto pv_add = [&](const uint2 u, const float2 p) {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        acc[0][0] = fmaf(p.x, lo.x, acc[0][0]);
        acc[0][1] = fmaf(p.x, lo.y, acc[0][1]);
        acc[0][2] = fmaf(p.x, hi.x, acc[0][2]);
        acc[0][3] = fmaf(p.x, hi.y, acc[0][3]);
        acc[1][0] = fmaf(p.y, lo.x, acc[1][0]);
        acc[1][1] = fmaf(p.y, lo.y, acc[1][1]);
        acc[1][2] = fmaf(p.y, hi.x, acc[1][2]);
        acc[1][3] = fmaf(p.y, hi.y, acc[1][3]);
      };
#pragma unroll 1
      for (int t0 = 0; t0 < n_old; t0 += KV_TOK_PER_PIECE) {
        const uint32_t pn = n + 2 * (t0 / KV_TOK_PER_PIECE) + 1;
        const uint2 *vcol = reinterpret_cast<const uint2 *>(sm.ring[pn % NSLOTS]) + dq;
        const float2 *pr = reinterpret_cast<const float2 *>(sm.sc[t0]);
        const int cnt = min(KV_TOK_PER_PIECE, n_old - t0);
        if (cnt == KV_TOK_PER_PIECE) {
          // Full piece: this thread's 6 tokens, all loads first.
          constexpr int TPT = KV_TOK_PER_PIECE / 8;
          uint2 vv[TPT];
          float2 pp[TPT];
#pragma unroll
          for (int k = 0; k < TPT; ++k) {
            vv[k] = vcol[(ts + 8 * k) * (HD / 4)];
            pp[k] = pr[ts + 8 * k];
          }
#pragma unroll
          for (int k = 0; k < TPT; ++k) pv_add(vv[k], pp[k]);
        } else {
#pragma unroll 2
          for (int tt = ts; tt < cnt; tt += 8) pv_add(vcol[tt * (HD / 4)], pr[tt]);
        }
      }
      if (fresh && ts == (n_old & 7))
        pv_add(reinterpret_cast<const uint2 *>(sm.qkv_raw + 3 * HD)[dq],
               *reinterpret_cast<const float2 *>(sm.sc[n_old]));
    }
    if (sc == 0) trace_clock(tr, TR_B_CYC2);
    named_bar_sync(BAR_ID, NCT);
    if (lane < 2 * npair) mbar_arrive(&sm.empty[(n + lane) % NSLOTS]);
    n += 2 * npair;
  }
  st.n = n;
  trace_mark(tr, TR_B_PV);
  trace_clock(tr, TR_B_CYC3);
  // Add the eight token slices in order; thread (h, d) then holds output dim
  // d of head h.
#pragma unroll
  for (int h = 0; h < 2; ++h)
    *reinterpret_cast<float4 *>(&sm.pvp[ts][h][4 * dq]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  if (tid < 2) {
    sm.att_m[tid] = m_run[tid];
    sm.att_l[tid] = l_run[tid];
  }
  named_bar_sync(BAR_ID, NCT);
  const int dd = tid & 127;
  float acc_hd = sm.pvp[0][hh][dd];
#pragma unroll
  for (int i = 1; i < NCW; ++i) acc_hd += sm.pvp[i][hh][dd];
  {
    const int h = hh, d = dd;
    float val = acc_hd;
    float m = sm.att_m[h], lsum = sm.att_l[h];
    if (ag.S > 1 && ag.j != 0) {
      uint64_t *pp = a.ws.part + ((static_cast<size_t>(g) * MAX_SPLITS + ag.j) * 2 + h) * (HD + 2);
      ll_store(pp + d, __float_as_uint(val), ep);
      if (d < 2) ll_store(pp + HD + d, __float_as_uint(d == 0 ? m : lsum), ep);
    }
    trace_mark(tr, TR_B_PART);
    bool write_out = ag.S == 1 || ag.j == 0;
    if (!(ag.S > 1 && ag.j == 0)) trace_mark(tr, TR_B_CMB);
    if (ag.S > 1 && ag.j == 0) {
      // Combiner (split 0), one gather round: thread (h, d) loads acc_j[d] of
      // every other split j (S <= MAX_SPLITS_B200); thread 2jj + hq
      // (1 <= jj < S) also loads split jj's (m, l) of head hq.
      constexpr int NA = MAX_SPLITS_B200 - 1;
      uint32_t u[NA + 2];
      const int jm = tid >> 1, hm = tid & 1;
      const bool ml = tid >= 2 && tid < 2 * ag.S;
      st.fail |= !ll_gather<NA + 2>(
          w,
          [&](int i) {
            if (i >= NA) {
              const int jj = ml ? jm : 1, hq = ml ? hm : h;
              return a.ws.part + ((static_cast<size_t>(g) * MAX_SPLITS + jj) * 2 + hq) * (HD + 2) + HD + (i - NA);
            }
            const int jj = 1 + min(i, ag.S - 2);
            return a.ws.part + ((static_cast<size_t>(g) * MAX_SPLITS + jj) * 2 + h) * (HD + 2) + d;
          },
          ep, u, W_B);
      if (ml) {
        sm.cmb_m[hm][jm] = __uint_as_float(u[NA]);
        sm.cmb_l[hm][jm] = __uint_as_float(u[NA + 1]);
      }
      if (tid < 2) {
        sm.cmb_m[tid][0] = sm.att_m[tid];
        sm.cmb_l[tid][0] = sm.att_l[tid];
      }
      named_bar_sync(BAR_ID, NCT);
      trace_mark(tr, TR_B_CMB);
      // Rescale factors, once per (head, split): exp(m_j - M), M the max.
      if (tid < 2 * ag.S) {
        float M = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < MAX_SPLITS_B200; ++jj)
          if (jj < ag.S) M = fmaxf(M, sm.cmb_m[hm][jj]);
        const float mj = sm.cmb_m[hm][jm];
        sm.cmb_f[hm][jm] = mj == -INFINITY ? 0.f : expf(mj - M);
      }
      named_bar_sync(BAR_ID, NCT);
      // acc = sum_j acc_j f_j and l = sum_j l_j f_j, splits in order.
      float A = val * sm.cmb_f[h][0], Ls = sm.cmb_l[h][0] * sm.cmb_f[h][0];
#pragma unroll
      for (int i = 0; i < NA; ++i) {
        if (i < ag.S - 1) {
          const float f = sm.cmb_f[h][i + 1];
          A = fmaf(__uint_as_float(u[i]), f, A);
          Ls = fmaf(sm.cmb_l[h][i + 1], f, Ls);
        }
      }
      val = A;
      lsum = Ls;
    }
    if (write_out) {
      const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
      const __half o = __float2half(val * inv);
      const int col = (2 * g + h) * HD + d;
      const uint32_t other = __shfl_down_sync(0xffffffffu, h2u(o), 1);
      if ((d & 1) == 0) ll_store(a.ws.attn + col / 2, h2u(o) | (other << 16), ep);
      a.attn_out[col] = o;
    }
  }
  // New token's K (rotated) and V (raw) into the cache at position p, 8
  // bytes per lane.  Later steps of this launch read the entry with bulk
  // copies, hence the release count (the reader acquires it and issues a
  // proxy fence before its copy).  Done last: the release waits for the
  // stores, and nothing in this step reads the entry from global memory.
  if (warp == 2 && ag.last) {
    const size_t off = ((static_cast<size_t>(l) * NKV + g) * a.max_seq + p) * HD + 4 * lane;
    *reinterpret_cast<uint2 *>(a.k_cache + off) = *reinterpret_cast<const uint2 *>(sm.k_fresh + 4 * lane);
    *reinterpret_cast<uint2 *>(a.v_cache + off) = *reinterpret_cast<const uint2 *>(sm.qkv_raw + 3 * HD + 4 * lane);
    if (a.num_steps > 1) {
      __syncwarp();
      if (lane == 0) red_release_add_u32(a.ws.kv_ready, 1);
    }
  }
  trace_mark(tr, TR_B2);
  return false;
}

// ---------------------------------------------------------------- stage C
// o_proj GEMV + fp32 residual (megakernel.cu:585-610, :868-872).
__device__ __forceinline__ bool stage_c(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        uint32_t ep, unsigned long long *tr) {
  const int tid = threadIdx.x;
  trace_mark(tr, TR_C0);
  const Rows o = rows_of(H, gridDim.x, blockIdx.x);
  const int np = npieces(o.n, 2 * QS);
  const int total =
      prep_rows<QS>(sm, st.n, np, [&](int i) { return seg_piece(nullptr, 2 * QS, o.lo, o.n, i, 0); });
  st.fail |= !wait_pieces(sm, w, st.n, np, W_C);
  {
    uint32_t u[4];
    st.fail |= !ll_gather<4>(w, [&](int i) { return a.ws.attn + tid + NCT * i; }, ep, u, W_C);
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint32_t *>(sm.xb)[tid + NCT * i] = u[i];
  }
  if (named_bar_or(BAR_ID, NCT, st.fail || sm.abort)) return true;
  trace_mark(tr, TR_C1);
  gemv_cc<QS>(
      sm, st.n, np, total, sm.xb,
      [&](int, int row, float dot) {
        const float resid = __half2float(sm.hid_own[row - o.lo]);
        const float act = dot + resid;
        ll_store(a.ws.act + row, __float_as_uint(act), ep);
        sm.act_own[row - o.lo] = act;
        a.act[row] = act;
        a.res[row] = resid;
      });
  trace_mark(tr, TR_C2);
  return false;
}

// ---------------------------------------------------------------- stage D
// Post-attention RMSNorm from fp32 act (megakernel.cu:614-638) + gate/up GEMV
// + half SiLU * up (:640-675).
__device__ __forceinline__ bool stage_d(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        int l, uint32_t ep, unsigned long long *tr) {
  const int tid = threadIdx.x;
  trace_mark(tr, TR_D0);
  const Rows gu = rows_of(IM, gridDim.x, blockIdx.x);
  const int np = 2 * npieces(gu.n, 2 * H);
  const int total = prep_rows<H>(
      sm, st.n, np, [&](int i) { return seg_piece(nullptr, 2 * H, gu.lo, gu.n, i >> 1, i & 1); });
  const __half *nw = norm_ptr(sm, a, l, 3);  // converted after the gather, as in stage A
  __half wr[4];
  float h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wr[i] = __ldg(nw + tid + NCT * i);
  st.fail |= !wait_pieces(sm, w, st.n, np, W_D);
  {
    uint32_t u[4];
    st.fail |= !ll_gather<4>(w, [&](int i) { return a.ws.act + tid + NCT * i; }, ep, u, W_D);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __uint_as_float(u[i]);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(h[i], h[i], ss);
  bool abort;
  const float tot = block_sum(sm, ss, st.fail || sm.abort, &abort);
  if (abort) return true;
  trace_mark(tr, TR_D1);
  const float rstd = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    sm.xa[tid + NCT * i] = __float2half(__half2float(__float2half(h[i])) * rstd * __half2float(wr[i]));
  named_bar_sync(BAR_ID, NCT);
  gemv_wr<H, 48>(sm, st.n, np, total, sm.xa, [&](int kind, int row, float dot) {
    (kind == 0 ? sm.g_out : sm.u_out)[row - gu.lo] = dot;
  });
  named_bar_sync(BAR_ID, NCT);
  if (tid < gu.n) {
    const float act = __half2float(silu_half(sm.g_out[tid])) * sm.u_out[tid];
    const int row = gu.lo + tid;
    ll_store(a.ws.inter + row, h2u(__float2half(act)), ep);
    a.inter[row] = act;
  }
  trace_mark(tr, TR_D2);
  return false;
}

// ---------------------------------------------------------------- stage E
// Down GEMV on half(mlp_inter) + residual, rounded to fp16 (megakernel.cu:679-707).
__device__ __forceinline__ bool stage_e(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        uint32_t ep, unsigned long long *tr) {
  const int tid = threadIdx.x;
  trace_mark(tr, TR_E0);
  const Rows o = rows_of(H, gridDim.x, blockIdx.x);
  const int np = npieces(o.n, 2 * IM);
  const int total =
      prep_rows<IM>(sm, st.n, np, [&](int i) { return seg_piece(nullptr, 2 * IM, o.lo, o.n, i, 0); });
  st.fail |= !wait_pieces(sm, w, st.n, np, W_E);
  {
    uint32_t u[IM / NCT];
    st.fail |= !ll_gather<IM / NCT>(w, [&](int i) { return a.ws.inter + tid + NCT * i; }, ep, u, W_E);
#pragma unroll
    for (int i = 0; i < IM / NCT; ++i) sm.xb[tid + NCT * i] = u2h(u[i]);
  }
  if (named_bar_or(BAR_ID, NCT, st.fail || sm.abort)) return true;
  trace_mark(tr, TR_E1);
  trace_clock(tr, TR_E_CYC0);
  gemv_cc<IM>(
      sm, st.n, np, total, sm.xb,
      [&](int, int row, float dot) {
        const __half hv = __float2half(dot + sm.act_own[row - o.lo]);
        ll_store(a.ws.hidden + row, h2u(hv), ep);
        sm.hid_own[row - o.lo] = hv;
        a.hidden[row] = hv;
      },
      tr);
  trace_clock(tr, TR_E_CYC2);
  trace_mark(tr, TR_E2);
  return false;
}

// ---------------------------------------------------------------- stage F
// Final RMSNorm to fp32 (megakernel.cu:890-919), tied lm_head GEMV and this
// CTA's argmax (:1001-1109; lowest index among equal maxima).
__device__ __forceinline__ bool stage_f(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        int s, uint32_t ep_last, unsigned long long *tr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  trace_mark(tr, 0);
  if (tr != nullptr && tid == 0) tr[5] = static_cast<unsigned long long>(clock64());
  {
    __half wr[4];  // converted where used, after the gather
    float h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) wr[i] = __ldg(a.final_norm + tid + NCT * i);
    uint32_t u[4];
    st.fail |= !ll_gather<4>(w, [&](int i) { return a.ws.hidden + tid + NCT * i; }, ep_last, u, W_F);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = __half2float(u2h(u[i]));
      ss = fmaf(h[i], h[i], ss);
    }
    bool abort;
    const float tot = block_sum(sm, ss, st.fail || sm.abort, &abort);
    if (abort) return true;
    trace_mark(tr, 1);
    const float inv = rsqrtf(tot / static_cast<float>(H) + RMS_EPS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float nv = h[i] * inv * __half2float(wr[i]);
      sm.xf[tid + NCT * i] = nv;
      if (c == 0) a.norm_out[tid + NCT * i] = nv;
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
  uint32_t n = st.n;
  for (int b0 = 0; b0 < lm_np; b0 += BATCH_MAX) {
    const int nb = min(BATCH_MAX, lm_np - b0);
    int j0 = 0;
    for (int i = 0; i < nb; ++i) {
      const Piece P = seg_piece(nullptr, 2 * H, lm.lo, lm.n, b0 + i, 0);
      const uint32_t pn = n + i;
      const int slot = pn % NSLOTS;
      int r = (warp - j0) % NCW;
      if (r < 0) r += NCW;
      if (r < P.nrows) st.fail |= !wait_mbar(w, &sm.full[slot], (pn / NSLOTS) & 1, ST_TIMEOUT_FULL, W_F);
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
        if (a.logits_out != nullptr && lane == 0 && s == a.num_steps - 1) a.logits_out[idx] = v;
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
  st.n = n;
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
  trace_mark(tr, 2);
  return false;
}

// ---------------------------------------------------------------- stage G
// Global argmax over the per-CTA results (megakernel.cu:1114-1144), lowest
// index among equal maxima.  CTA 0 gathers the per-CTA pairs and publishes
// the token in one handoff word, which the other CTAs poll with one thread
// each (every CTA gathering all pairs put ~150 pollers on the same few L2
// lines).  Sets *token (uniform).
__device__ __forceinline__ bool stage_g(Smem &sm, const DecodeArgs &a, const WaitCtx &w, St &st,
                                        int s, int *token, unsigned long long *tr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = gridDim.x;
  const uint32_t eps_ = a.epoch_base + static_cast<uint32_t>(s);
  int bi = 0;
  if (blockIdx.x == 0) {
    float v = -INFINITY;
    int id = 0x7fffffff;
    if (tid < C) {
      uint32_t u[2];
      st.fail |= !ll_gather<2>(w, [&](int i) { return a.ws.amax + i * MAX_CTAS + tid; }, eps_, u, W_G);
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
    if (named_bar_or(BAR_ID, NCT, st.fail || sm.abort)) return true;
    float bv = sm.gmax_val[0];
    bi = sm.gmax_idx[0];
    for (int i = 1; i < NCW; ++i) {
      const float vv = sm.gmax_val[i];
      const int ii = sm.gmax_idx[i];
      if (vv > bv || (vv == bv && ii < bi)) {
        bv = vv;
        bi = ii;
      }
    }
    if (tid == 0) {
      ll_store(a.ws.token, static_cast<uint32_t>(bi), eps_);
      a.out_tokens[s] = bi;
    }
  } else {
    if (tid == 0) {
      uint32_t u[1];
      st.fail |= !ll_gather<1>(w, [&](int) { return a.ws.token; }, eps_, u, W_G);
      sm.gmax_idx[0] = static_cast<int>(u[0]);
    }
    if (named_bar_or(BAR_ID, NCT, st.fail || sm.abort)) return true;
    bi = sm.gmax_idx[0];
  }
  trace_mark(tr, 3);
  *token = (bi >= 0 && bi < VOCAB) ? bi : 0;
  trace_mark(tr, 4);
  if (tr != nullptr && tid == 0) tr[6] = static_cast<unsigned long long>(clock64());
  return false;
}

// CTA-wide end of a stage (tracing only: one extra barrier per stage).
__device__ __forceinline__ void trace_end(Smem &sm, unsigned long long *tr, int ev) {
  if (tr != nullptr) {
    named_bar_sync(BAR_ID, NCT);
    trace_mark(tr, ev);
    if (threadIdx.x == 0) tr[TR_FW] = sm.trace_fullwait;
  }
}

__device__ __forceinline__ void consumer(const DecodeArgs &a, Smem &sm) {
  const int C = gridDim.x, c = blockIdx.x, L = a.num_layers;
  const WaitCtx w = make_wait(a, sm);
  St st;
  st.n = 0;
  st.fail = false;
  int token = a.first_token;
  if (a.first_token_dev != nullptr) {
    token = *reinterpret_cast<const volatile int *>(a.first_token_dev);
    if (token < 0 || token >= VOCAB) {
      set_error(w, ST_BAD_TOKEN, W_A);
      token = 0;
    }
  }
  for (int i = threadIdx.x; i < min(L, NTAB_LAYERS) * 4; i += NCT)
    sm.ntab[i >> 2][i & 3] = layer_ptr(a.layers, i >> 2, norm_slot(i & 3));
  plan_rows_a(sm, C, c);
  named_bar_sync(BAR_ID, NCT);
  int s = 0;
  for (s = 0; s < a.num_steps; ++s) {
    const int p = a.start_pos + s;
    const AttnGeom ag = attn_geom(p, C, c);
    for (int l = 0; l < L; ++l) {
      const uint32_t ep = a.epoch_base + static_cast<uint32_t>(s * L + l);
      unsigned long long *tr = trace_row(a, s, l);
      if (stage_a(sm, a, w, st, l, token, ep, tr)) goto out;
      trace_end(sm, tr, TR_A3);
      if (ag.has) {
        if (stage_b(sm, a, w, st, ag, l, p, ep, tr)) goto out;
        trace_end(sm, tr, TR_B3);
      }
      if (stage_c(sm, a, w, st, ep, tr)) goto out;
      trace_end(sm, tr, TR_C3);
      if (stage_d(sm, a, w, st, l, ep, tr)) goto out;
      trace_end(sm, tr, TR_D3);
      if (stage_e(sm, a, w, st, ep, tr)) goto out;
      trace_end(sm, tr, TR_E3);
    }
    {
      unsigned long long *trf = trace_row(a, s, L);
      if (stage_f(sm, a, w, st, s, a.epoch_base + static_cast<uint32_t>(s * L + L - 1), trf)) goto out;
      if (stage_g(sm, a, w, st, s, &token, trf)) goto out;
    }
  }
  return;
out:
  if (c == 0 && threadIdx.x == 0)
    for (int s2 = s; s2 < a.num_steps; ++s2) a.out_tokens[s2] = -1;
}

__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte aligned base: bulk copies need 16-byte aligned slots, and the
  // 16-byte vector reads of the GEMVs and of the K rows rely on it.
  // Offset the shared array itself rather than an integer copy of its
  // address: the compiler then keeps every Smem access in the shared address
  // space (LDS/STS instead of generic loads and stores).
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u));
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < NSLOTS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], NCW);
    }
    sm.abort = 0;
    sm.trace_fullwait = 0;
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
  w.fullwait = nullptr;
  w.abort = &abort_flag;
  w.err = err;
  w.tag = tag;
  w.timeout_ns = timeout_ns;
  uint32_t u[1];
  ll_gather<1>(w, [&](int) { return word; }, 0xfffffff0u, u, W_SELFTEST);
}

// Handoff words of one decode launch (the Workspace layout below), plus 32
// words for the KV-ready counter, the status word and the published token.
constexpr size_t WS_LL_WORDS = H + QKV_ROWS + QS / 2 + H + IM +
                               static_cast<size_t>(NKV) * MAX_SPLITS * 2 * (HD + 2) + 2 * MAX_CTAS;
constexpr size_t WS_TAIL_WORDS = 32;

}  // namespace qb200

// Fixed workspace of launch_ldg_generate_nosync_static_ws: 618,752 bytes per
// device, enough for up to MAX_CTAS (256) CTAs and MAX_SPLITS (32) attention
// splits per KV head.  Loaded with the module, so that entry point never
// allocates.  One copy per device, shared by every call on that device.
static __device__ __align__(256) uint64_t g_static_ws[qb200::WS_LL_WORDS + qb200::WS_TAIL_WORDS];

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
unsigned long long *g_trace = nullptr;
long long g_trace_bytes = 0;
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

int current_device(int *dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail_msg(2, "cudaGetDevice failed");
    return 0;
  }
  *dev_out = dev;
  return 1;
}

// Checks that `dev` can run the decode kernel and sets its shared-memory
// attribute.  Returns the device's SM count, or 0 with the error recorded.
int probe_device(int dev) {
  int sms = 0, coop = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop) {
    fail_msg(3, "device %d does not support cooperative launch", dev);
    return 0;
  }
  if (sms < MIN_CTAS || sms > MAX_CTAS) {
    fail_msg(3, "device %d has %d SMs; this kernel needs %d..%d", dev, sms, MIN_CTAS, MAX_CTAS);
    return 0;
  }
  cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem_bytes()));
  if (e != cudaSuccess) {
    fail_msg(4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return 0;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, NTHREADS, smem_bytes());
  if (per_sm < 1) {
    fail_msg(4, "decode kernel does not fit on an SM (%zu B shared memory)", smem_bytes());
    return 0;
  }
  return sms;
}

// Lays the Workspace out over `mem` (WS_LL_WORDS + WS_TAIL_WORDS zeroed
// words) and marks `d` ready.
void bind_workspace(DevState &d, void *mem, int sms) {
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
  d.ws.token = p + 8;
  d.mem = mem;
  d.ll_bytes = WS_LL_WORDS * sizeof(uint64_t);
  d.num_sms = sms;
  if (const char *env = getenv("QB200_CTAS")) {
    const int want = atoi(env);
    if (want >= MIN_CTAS && want <= sms) d.num_sms = want;
  }
  d.epoch = 1;
  d.ready = true;
}

// Workspace of the two upstream launchers: allocated on the first call on
// each device.
DevState *get_dev(int *dev_out) {
  if (!current_device(dev_out)) return nullptr;
  DevState &d = g_dev[*dev_out];
  if (d.ready) return &d;
  const int sms = probe_device(*dev_out);
  if (!sms) return nullptr;
  const size_t total = (WS_LL_WORDS + WS_TAIL_WORDS) * sizeof(uint64_t);
  void *mem = nullptr;
  cudaError_t e = cudaMalloc(&mem, total);
  if (e != cudaSuccess) {
    fail_msg(5, "cudaMalloc(%zu) for the decode workspace: %s", total, cudaGetErrorString(e));
    return nullptr;
  }
  // The clear runs on the legacy default stream, which is not ordered with
  // the non-blocking streams callers launch on: wait for it here, so the
  // first launch cannot see it land mid-run.
  e = cudaMemset(mem, 0, total);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(mem);
    fail_msg(5, "clearing the decode workspace on device %d: %s", *dev_out, cudaGetErrorString(e));
    return nullptr;
  }
  bind_workspace(d, mem, sms);
  return &d;
}

// Workspace of launch_ldg_generate_nosync_static_ws: the module's static
// array, looked up once per device (with that device current).  The lookup
// may load the module on that device, and the clearing is followed by a
// cudaDeviceSynchronize (the clear runs on the legacy default stream, which
// is not ordered with the caller's non-blocking streams), which is why this
// set-up belongs before any stream capture.  Cleared here because every
// handoff word must start with an epoch no launch uses (0), and the status
// word and KV-ready counter at 0.
DevState g_dev_static[64];

DevState *get_dev_static(int *dev_out) {
  if (!current_device(dev_out)) return nullptr;
  DevState &d = g_dev_static[*dev_out];
  if (d.ready) return &d;
  const int sms = probe_device(*dev_out);
  if (!sms) return nullptr;
  void *mem = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&mem, g_static_ws);
  if (e != cudaSuccess || mem == nullptr) {
    fail_msg(6, "cudaGetSymbolAddress(static decode workspace) on device %d: %s", *dev_out,
             cudaGetErrorString(e));
    return nullptr;
  }
  e = cudaMemset(mem, 0, (WS_LL_WORDS + WS_TAIL_WORDS) * sizeof(uint64_t));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fail_msg(6, "clearing the static decode workspace on device %d: %s", *dev_out,
             cudaGetErrorString(e));
    return nullptr;
  }
  bind_workspace(d, mem, sms);
  return &d;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Host-side argument checks shared by every launcher; 0 when accepted.
int check_args(const DecodeArgs &a) {
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
  if (a.first_token_dev == nullptr && (a.first_token < 0 || a.first_token >= VOCAB))
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
  return 0;
}

// Takes this launch's epochs from `d` and launches on `d`'s workspace.
int launch_on(DevState &d, DecodeArgs &a, cudaStream_t st) {
  if (d.num_sms > MAX_CTAS)
    return fail_msg(3, "%d CTAs requested; the decode workspace holds per-CTA results for at most %d",
                    d.num_sms, MAX_CTAS);
  const uint64_t need = static_cast<uint64_t>(a.num_steps) * (a.num_layers + 1) + 2;
  if (static_cast<uint64_t>(d.epoch) + need >= 0xfffffff0ull) {
    cudaMemsetAsync(d.mem, 0, d.ll_bytes, st);
    cudaMemsetAsync(d.ws.token, 0, sizeof(uint64_t), st);
    d.epoch = 1;
  }
  a.epoch_base = d.epoch;
  d.epoch += static_cast<uint32_t>(need);
  d.last_tag = a.epoch_base;
  a.timeout_ns = g_timeout_ns;
  a.ws = d.ws;
  a.trace = nullptr;
  a.trace_steps = 0;
  if (g_trace != nullptr) {
    const long long per_step = static_cast<long long>(d.num_sms) * (a.num_layers + 1) * TR_N * 8;
    const long long steps = per_step > 0 ? g_trace_bytes / per_step : 0;
    if (steps > 0) {
      a.trace = g_trace;
      a.trace_steps = static_cast<int>(steps < a.num_steps ? steps : a.num_steps);
    }
  }
  if (a.num_steps > 1) cudaMemsetAsync(d.ws.kv_ready, 0, sizeof(uint32_t), st);
  void *args[] = {&a};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<void *>(decode_kernel),
                                              dim3(d.num_sms), dim3(NTHREADS), args, smem_bytes(), st);
  if (e != cudaSuccess) return fail_msg(20, "decode kernel launch: %s", cudaGetErrorString(e));
  return 0;
}

int launch_decode(DecodeArgs &a, cudaStream_t st) {
  if (check_args(a)) return t_err;
  std::lock_guard<std::mutex> lk(g_mu);
  int dev = 0;
  DevState *d = get_dev(&dev);
  if (!d) return t_err;
  return launch_on(*d, a, st);
}

int launch_decode_static_ws(DecodeArgs &a, cudaStream_t st) {
  if (check_args(a)) return t_err;
  std::lock_guard<std::mutex> lk(g_mu);
  int dev = 0;
  DevState *d = get_dev_static(&dev);
  if (!d) return t_err;
  return launch_on(*d, a, st);
}

// Kernel arguments of a generate call (parameters as launch_ldg_generate_nosync).
DecodeArgs generate_args(int first_token_id, int num_steps, const void *embed_weight,
                         const LDGLayerWeight *layer_weights, const void *final_norm_weight,
                         const void *lm_head_weight, const void *cos_table, const void *sin_table,
                         void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
                         void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
                         void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
                         void *block_max_idxs, int *output_log, int num_layers, int start_position,
                         int max_seq_len, float attn_scale) {
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
  return a;
}

}  // namespace

extern "C" {

int qwen_b200_abi_version(void) { return QWEN_B200_ABI_VERSION; }

// Shared with the operator library (ops.cu): one thread-local error slot for
// every entry point of this library.
void qb200_clear_error(void) {
  t_err = 0;
  t_msg[0] = 0;
}

int qb200_set_error(int code, const char *msg) { return fail_msg(code, "%s", msg); }

int qwen_b200_last_error(char *msg, int msg_len) {
  if (msg && msg_len > 0) {
    strncpy(msg, t_msg, msg_len - 1);
    msg[msg_len - 1] = 0;
  }
  return t_err;
}

void qwen_b200_set_wait_timeout_ns(long long ns) { g_timeout_ns = ns > 0 ? ns : 2000000000LL; }

void qwen_b200_set_trace(void *device_buffer, long long bytes) {
  g_trace = static_cast<unsigned long long *>(device_buffer);
  g_trace_bytes = device_buffer ? bytes : 0;
}

int qwen_b200_device_status(int device, uint64_t *detail) {
  if (device < 0 || device >= 64) return -1;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int rc = 0;
  uint64_t word = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    // The allocating launchers' workspace first, then the static one of
    // launch_ldg_generate_nosync_static_ws: the first failure found is
    // reported (each word only counts for its workspace's last launch).
    bool synced = false;
    for (DevState *d : {&g_dev[device], &g_dev_static[device]}) {
      if (!d->ready || rc != 0) continue;
      if (!synced) {
        cudaDeviceSynchronize();
        synced = true;
      }
      uint64_t w = 0;
      if (cudaMemcpy(&w, d->ws.err, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess) {
        rc = -2;
      } else if (static_cast<uint32_t>(w >> 32) == d->last_tag && (w & 0xffffffffull)) {
        rc = static_cast<int>((w >> 24) & 0xff);
        word = w;
      }
    }
  }
  if (detail) *detail = word;
  cudaSetDevice(prev);
  return rc;
}

int qwen_b200_workspace_info(int device, int *alloc_ready, int *static_ready) {
  if (device < 0 || device >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  if (alloc_ready) *alloc_ready = g_dev[device].ready ? 1 : 0;
  if (static_ready) *static_ready = g_dev_static[device].ready ? 1 : 0;
  return 0;
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
  DecodeArgs a = generate_args(first_token_id, num_steps, embed_weight, layer_weights,
                               final_norm_weight, lm_head_weight, cos_table, sin_table, k_cache,
                               v_cache, hidden_buffer, g_activations, g_residual, g_q, g_k, g_v,
                               g_attn_out, g_mlp_intermediate, g_normalized, block_max_vals,
                               block_max_idxs, output_log, num_layers, start_position,
                               max_seq_len, attn_scale);
  launch_decode(a, static_cast<cudaStream_t>(stream));
}

int qwen_b200_decode_step_dev(const int *input_token, int *output_token, float *logits_out,
                              const void *embed_weight, const LDGLayerWeight *layer_weights,
                              const void *final_norm_weight, const void *lm_head_weight,
                              const void *cos_table, const void *sin_table, void *k_cache, void *v_cache,
                              void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
                              void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate,
                              void *g_normalized, void *block_max_vals, void *block_max_idxs,
                              int num_layers, int position, int max_seq_len, float attn_scale,
                              void *stream) {
  if (input_token == nullptr) {
    qb200_clear_error();
    return fail_msg(13, "null input token pointer");
  }
  DecodeArgs a = generate_args(0, 1, embed_weight, layer_weights, final_norm_weight, lm_head_weight,
                               cos_table, sin_table, k_cache, v_cache, hidden_buffer, g_activations,
                               g_residual, g_q, g_k, g_v, g_attn_out, g_mlp_intermediate, g_normalized,
                               block_max_vals, block_max_idxs, output_token, num_layers, position,
                               max_seq_len, attn_scale);
  a.first_token_dev = input_token;
  a.logits_out = logits_out;
  return launch_decode(a, static_cast<cudaStream_t>(stream));
}

int launch_ldg_generate_nosync_static_ws(
    int first_token_id, int num_steps, const void *embed_weight,
    const LDGLayerWeight *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table, void *k_cache,
    void *v_cache, void *hidden_buffer, void *g_activations, void *g_residual, void *g_q,
    void *g_k, void *g_v, void *g_attn_out, void *g_mlp_intermediate, void *g_normalized,
    void *block_max_vals, void *block_max_idxs, int *output_log, int num_layers,
    int start_position, int max_seq_len, float attn_scale, void *stream) {
  DecodeArgs a = generate_args(first_token_id, num_steps, embed_weight, layer_weights,
                               final_norm_weight, lm_head_weight, cos_table, sin_table, k_cache,
                               v_cache, hidden_buffer, g_activations, g_residual, g_q, g_k, g_v,
                               g_attn_out, g_mlp_intermediate, g_normalized, block_max_vals,
                               block_max_idxs, output_log, num_layers, start_position,
                               max_seq_len, attn_scale);
  return launch_decode_static_ws(a, static_cast<cudaStream_t>(stream));
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
