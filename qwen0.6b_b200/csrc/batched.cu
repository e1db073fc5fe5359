// batched.cu - batched greedy decode of many independent sequences on one GPU
// (B200 / sm_100a): every row of a step is one sequence at its own position,
// with its own fp16 KV cache.  C ABI in include/qwen_b200_batched.h.
//
// One step = per layer
//   input RMSNorm (warp per row)                     -> xn      fp16 [R, 1024]
//   tcgen05 GEMM  xn . Wqkv^T, fp16 out              -> qkv     fp16 [R, 4096]
//   q/k RMSNorm + RoPE, K/V appended to the caches   -> qrot    fp16 [R, 2048]
//   split-KV attention (bulk-copied K/V chunks)      -> partials fp32
//   split combine                                    -> attn    fp16 [R, 2048]
//   tcgen05 GEMM  attn . Wo^T + hidden (fp32)        -> act     fp32 [R, 1024]
//   post-attention RMSNorm                           -> sact    fp16 [R, 1024]
//   tcgen05 GEMM  sact . Wgu^T, fp16 SiLU(gate)*up   -> inter   fp16 [R, 3072]
//   tcgen05 GEMM  inter . Wdown^T + act, fp16        -> hidden  fp16 [R, 1024]
// then the final RMSNorm, the tied lm_head GEMM with a fused per-tile argmax
// and the row argmax.  The rounding points are those of the upstream batch-1
// kernel (Tools/megakernel/megakernel.cu:763-1144); the projections and the
// lm_head accumulate in fp32 on the tensor cores in a different order, and the
// lm_head input is the final-normed hidden rounded to fp16 (upstream keeps it
// in fp32), which moves a logit by ~1e-4.
//
// Memory layout (HBM):
//   K, V pools  fp16 [num_seqs][layers][8][max_seq][128]: one sequence's
//               cache of one head is contiguous, so an attention chunk is one
//               bulk copy;
//   Wqkv        fp16 [layers][4096][1024] (q | k | v rows);
//   Wgu         fp16 [layers][6144][1024], rows (2i, 2i+1) = (gate_i, up_i),
//               so the SwiGLU pairs meet in one GEMM epilogue;
//   Wo, Wdown   the HF [out, in] matrices as given.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <new>
#include <stdlib.h>
#include <string.h>

#include "gemm_tc_host.h"
#include "host_err.h"
#include "ptx.cuh"
#include "qwen_b200_batched.h"

namespace qb200b {

using qb200::globaltimer_ns;
using qb200::mbar_arrive_expect_tx;
using qb200::mbar_init;
using qb200::mbar_try_wait;
using qb200::smem_u32;
using qb200::warp_sum;

constexpr int H = 1024, IM = 3072, NQ = 16, NKV = 8, HD = 128;
constexpr int QS = NQ * HD, KVS = NKV * HD, QKV = QS + 2 * KVS;
constexpr int VOCAB = 151936;
constexpr float EPS = 1e-6f;
constexpr int PAGE = 128;               // tokens per KV page (paged pools)
constexpr int CH = 64;                  // tokens per attention split (34 KB of K/V: six CTAs per SM)
static_assert(PAGE % CH == 0, "a split never crosses a page");
constexpr int ATT_THREADS = 128;
constexpr int PART = HD + 2;            // acc[128], m, l per (row, kv head, split, head)
constexpr long long WAIT_NS = 2000000000LL;
constexpr int KSPLIT = 4;               // split-K slices of the N=1024 GEMMs (o_proj, down)

__device__ __noinline__ void record_err(unsigned long long *err, uint32_t code) {
  const unsigned long long v = (static_cast<unsigned long long>(code) << 32) |
                               (static_cast<unsigned long long>(blockIdx.z & 0xffffu) << 16) |
                               (blockIdx.x & 0xffffu);
  atomicCAS(err, 0ull, v);
}

// KV pool geometry.  Contiguous pools: page = sequence, one page of max_seq
// tokens per (sequence, layer, kv head).  Paged pools: pages of PAGE tokens,
// page_table[seq * max_pages + position / PAGE] names the page of a position
// (-1: none).  Pool row of (sequence, layer, kv head g, position):
// ((page * layers + layer) * 8 + g) * page_tokens + position % page_tokens.
struct KvGeom {
  const int *page_table;  // null: contiguous pools
  int max_pages, num_pages, page_tokens, num_layers;
};

// Pool row of token `pos` of kv head g, or -1 when its page is not mapped.
__device__ __forceinline__ long long kv_row(const KvGeom &kg, int seq, int layer, int g, int pos) {
  int page = seq, off = pos;
  if (kg.page_table != nullptr) {
    page = kg.page_table[static_cast<size_t>(seq) * kg.max_pages + pos / kg.page_tokens];
    if (page < 0 || page >= kg.num_pages) return -1;
    off = pos % kg.page_tokens;
  }
  return ((static_cast<long long>(page) * kg.num_layers + layer) * NKV + g) * kg.page_tokens + off;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Lane `lane` of the warp that owns `row`: h = half(sum of the K slices of the
// previous down projection (added in slice order) + res32) for the columns
// 8 (lane + 32 j) .. +7, j < 4 -- the split-K reduction and residual of that
// GEMM with the bits of splitk_reduce_kernel's EPI_F16_RES32.  The slices
// are the outer loop so that each step issues all eight loads of the lane.
__device__ __forceinline__ void reduce_down_row(const float *__restrict__ part, int splits,
                                                const float *__restrict__ res32, int rows, int row, int lane,
                                                uint4 (&v)[4]) {
  const size_t slice4 = static_cast<size_t>(rows) * H / 4;
  const float4 *p4 = reinterpret_cast<const float4 *>(part + static_cast<size_t>(row) * H);
  const float4 *r4 = reinterpret_cast<const float4 *>(res32 + static_cast<size_t>(row) * H);
  float4 a[8], r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = r4[2 * (lane + 32 * (i >> 1)) + (i & 1)];
  if (splits <= 4) {
    // Every slice and the residual requested before the first add (one round
    // trip); the adds still run in slice order.
    float4 c[4][8];
#pragma unroll
    for (int z = 0; z < 4; ++z)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        c[z][i] = z < splits ? p4[z * slice4 + 2 * (lane + 32 * (i >> 1)) + (i & 1)] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = c[0][i];
#pragma unroll
    for (int z = 1; z < 4; ++z)
      if (z < splits)
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = add4(a[i], c[z][i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = p4[2 * (lane + 32 * (i >> 1)) + (i & 1)];
#pragma unroll 4
    for (int z = 1; z < splits; ++z) {
      float4 c[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = p4[z * slice4 + 2 * (lane + 32 * (i >> 1)) + (i & 1)];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = add4(a[i], c[i]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 x = add4(a[2 * j], r[2 * j]), y = add4(a[2 * j + 1], r[2 * j + 1]);
    __half2 *h2 = reinterpret_cast<__half2 *>(&v[j]);
    h2[0] = __floats2half2_rn(x.x, x.y);
    h2[1] = __floats2half2_rn(x.z, x.w);
    h2[2] = __floats2half2_rn(y.x, y.y);
    h2[3] = __floats2half2_rn(y.z, y.w);
  }
}

// ------------------------------------------------------------ input RMSNorm
// xn = half(h * (inv * w)), inv = rsqrtf(sum(h^2) / 1024 + eps) (megakernel.cu:806-847).
// Layer 0 gathers h = embed[token]; later layers, when the previous down
// projection left K slices (`part`), first finish it: h = half(sum + res32).
// h is stored as the row's hidden state.
__global__ void __launch_bounds__(256) input_norm_kernel(__half *__restrict__ hidden,
                                                         const __half *__restrict__ embed,
                                                         const int *__restrict__ tokens,
                                                         const float *__restrict__ part, int splits,
                                                         const float *__restrict__ res32,
                                                         const __half *__restrict__ w,
                                                         __half *__restrict__ xn, int rows,
                                                         unsigned long long *err) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  __half *hr = hidden + static_cast<size_t>(row) * H;
  uint4 v[4], wv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) wv[j] = reinterpret_cast<const uint4 *>(w)[lane + 32 * j];  // before the row's loads
  if (embed != nullptr) {
    int tok = tokens[row];
    if (tok < 0 || tok >= VOCAB) {  // recorded; the row decodes token 0 instead of reading out of bounds
      if (lane == 0) record_err(err, 2);
      tok = 0;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(embed + static_cast<size_t>(tok) * H);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = src[lane + 32 * j];
      reinterpret_cast<uint4 *>(hr)[lane + 32 * j] = v[j];
    }
  } else if (part != nullptr) {
    reduce_down_row(part, splits, res32, rows, row, lane, v);
#pragma unroll
    for (int j = 0; j < 4; ++j) reinterpret_cast<uint4 *>(hr)[lane + 32 * j] = v[j];
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = reinterpret_cast<const uint4 *>(hr)[lane + 32 * j];
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&v[j]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h2[i]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(H) + EPS);
  __half *o = xn + static_cast<size_t>(row) * H;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&v[j]);
    const __half2 *w2 = reinterpret_cast<const __half2 *>(&wv[j]);
    uint4 out;
    __half2 *o2 = reinterpret_cast<__half2 *>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h2[i]);
      const float2 g = __half22float2(w2[i]);
      o2[i] = __floats2half2_rn(__fmul_rn(f.x, __fmul_rn(inv, g.x)), __fmul_rn(f.y, __fmul_rn(inv, g.y)));
    }
    reinterpret_cast<uint4 *>(o)[lane + 32 * j] = out;
  }
}

// ------------------------------------------------ q/k RMSNorm, RoPE, KV append
// Per row (one CTA, one warp per head): 16 q heads and 8 k heads normalised over
// 128 dims (eps 1e-6, (x * inv) * w) and rotated (rotate-half, fp16 cos/sin
// tables), rounded to fp16 (megakernel.cu:339-434); rotated K and raw V go to
// the caches at the row's position.
__global__ void __launch_bounds__(32 * (NQ + NKV)) qk_rope_kv_kernel(
    const __half *__restrict__ qkv, const __half *__restrict__ q_norm,
    const __half *__restrict__ k_norm, const __half *__restrict__ cos_t,
    const __half *__restrict__ sin_t, const int *__restrict__ seq_ids,
    const int *__restrict__ positions, __half *__restrict__ k_pool, __half *__restrict__ v_pool,
    __half *__restrict__ q_rot, int layer, KvGeom kg, int max_seq, int num_seqs,
    unsigned long long *err) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = positions[row];
  const int seq_id = seq_ids[row];
  // Out-of-range sequence or position, or an unmapped page: no cache access.
  const long long row0 = (seq_id < 0 || seq_id >= num_seqs || pos < 0 || pos >= max_seq)
                             ? -1 : kv_row(kg, seq_id, layer, 0, pos);
  if (row0 < 0) {
    if (threadIdx.x == 0) record_err(err, 3);
    return;
  }
  const size_t head_stride = static_cast<size_t>(kg.page_tokens) * HD;  // kv head g -> g+1 in the pool
  const __half *src_row = qkv + static_cast<size_t>(row) * QKV;
  const __half *cosp = cos_t + static_cast<size_t>(pos) * HD;
  const __half *sinp = sin_t + static_cast<size_t>(pos) * HD;
  for (int hh = warp; hh < NQ + NKV; hh += blockDim.x >> 5) {  // one warp per head at launch size
    const bool is_q = hh < NQ;
    const __half *src = src_row + (is_q ? hh * HD : QS + (hh - NQ) * HD);
    const __half *nw = is_q ? q_norm : k_norm;
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
    for (int it = 0; it < 4; ++it) vals[it] = __fmul_rn(__fmul_rn(xv[it], inv), __half2float(nw[lane + 32 * it]));
    __half *dst = is_q ? q_rot + static_cast<size_t>(row) * QS + hh * HD
                       : k_pool + static_cast<size_t>(row0) * HD + (hh - NQ) * head_stride;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int i = lane + 32 * it;
      const int ri = it < 2 ? i : i - HD / 2;
      const float c = __half2float(cosp[ri]), s = __half2float(sinp[ri]);
      const float r = it < 2 ? __fsub_rn(__fmul_rn(vals[it], c), __fmul_rn(vals[it + 2], s))
                             : __fadd_rn(__fmul_rn(vals[it - 2], s), __fmul_rn(vals[it], c));
      dst[i] = __float2half_rn(r);
    }
  }
  // V (raw) into the cache: thread t < 256 copies elements 4t .. 4t+3.
  if (threadIdx.x >= KVS / 4) return;
  const int e = 4 * threadIdx.x, g = e / HD, d = e % HD;
  const uint2 val = *reinterpret_cast<const uint2 *>(src_row + QS + KVS + e);
  *reinterpret_cast<uint2 *>(v_pool + static_cast<size_t>(row0) * HD + g * head_stride + d) = val;
}

// ---------------------------------------------------------- split attention
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// K arrives as two 128-byte-swizzled halves (dims 0..63, 64..127) of CH rows
// each (TMA tensor copies); V as one contiguous bulk copy.
struct AttnSmem {
  __half k[2][CH * (HD / 2)];
  __half v[CH * HD];
  __half q[2][HD];
  float sc[2][CH];
  float red[4][2];
  uint64_t bar_k, bar_v;
  uint32_t abort;
};

// grid (max_splits, 8 kv heads, rows), 128 threads.  Work item (row, g, j):
// tokens [j*CH, min((j+1)*CH, pos+1)) of kv head g for q heads 2g, 2g+1;
// writes acc[128], m, l per q head (unnormalised, fp32).
// Offset of K[token][dim] in a 128-byte-swizzled half tile (rows of 128 B, the
// 16-byte chunk index XORed with the row within its 8-row atom).
__device__ __forceinline__ int k_swz(int tok, int dim) {
  const int h = dim >> 6, d = dim & 63;
  return h * CH * (HD / 2) + tok * (HD / 2) + ((((d >> 3) ^ (tok & 7)) << 3) | (d & 7));
}

__global__ void __launch_bounds__(ATT_THREADS) attn_split_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __half *__restrict__ q_rot,
    const __half *__restrict__ k_pool,
    const __half *__restrict__ v_pool, const int *__restrict__ seq_ids,
    const int *__restrict__ positions, float *__restrict__ part, int layer, KvGeom kg,
    int max_seq, int max_splits, int num_seqs, float attn_scale, unsigned long long *err) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  const int j = blockIdx.x, g = blockIdx.y, row = blockIdx.z;
  const int pos = positions[row], seq_id = seq_ids[row];
  if (seq_id < 0 || seq_id >= num_seqs || pos < 0 || pos >= max_seq) return;  // recorded by qk_rope_kv
  const int n_tok = pos + 1;
  const int t0 = j * CH;
  if (t0 >= n_tok || j >= max_splits) return;
  const int ntok = min(CH, n_tok - t0);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base: the swizzled K halves need it.
  AttnSmem &sm = *reinterpret_cast<AttnSmem *>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Row of the split's first K in the pool (a split never crosses a page:
  // paged pools use pages of CH tokens and splits start at multiples of CH).
  const long long krow_s = kv_row(kg, seq_id, layer, g, t0);
  float *pp_out = part + ((static_cast<size_t>(row) * NKV + g) * max_splits + j) * 2 * PART;
  if (krow_s < 0) {  // unmapped page: recorded, the split contributes nothing
    if (tid == 0) record_err(err, 3);
    if (tid < 2) {
      pp_out[tid * PART + HD] = -INFINITY;
      pp_out[tid * PART + HD + 1] = 0.f;
    }
    return;
  }
  const size_t krow0 = static_cast<size_t>(krow_s);
  const size_t base = krow0 * HD;
  if (tid == 0) {
    // The copies go out right after the barriers are initialised (same
    // thread); the block barrier below publishes both to the other threads.
    mbar_init(&sm.bar_k, 1);
    mbar_init(&sm.bar_v, 1);
    sm.abort = 0;
    qb200::fence_mbar_init();
    const uint32_t bytes = static_cast<uint32_t>(ntok) * HD * 2;
    const uint64_t pol = qb200::policy_evict_first();
    // Full boxes: rows past this split's tokens are read too (masked below);
    // rows past the end of the pool are zero-filled by the copy.
    mbar_arrive_expect_tx(&sm.bar_k, 2 * CH * (HD / 2) * 2);
    qb200tc::tma_load_2d(sm.k[0], &tm_k, 0, static_cast<int>(krow0), &sm.bar_k);
    qb200tc::tma_load_2d(sm.k[1], &tm_k, HD / 2, static_cast<int>(krow0), &sm.bar_k);
    mbar_arrive_expect_tx(&sm.bar_v, bytes);
    qb200::bulk_g2s(sm.v, v_pool + base, bytes, &sm.bar_v, pol);
  }
  {
    const __half *qs = q_rot + static_cast<size_t>(row) * QS + 2 * g * HD;
    reinterpret_cast<uint32_t *>(&sm.q[0][0])[tid] = reinterpret_cast<const uint32_t *>(qs)[tid];
  }
  __syncthreads();
  // Wait for K (bounded); every thread waits so all see the data.  V keeps
  // landing while the scores and the softmax run.
  auto wait_bar = [&](uint64_t *bar) {
    const uint64_t t_start = globaltimer_ns();
    while (!mbar_try_wait(bar, 0)) {
      if (static_cast<long long>(globaltimer_ns() - t_start) > WAIT_NS) {
        if (atomicExch(&sm.abort, 1u) == 0u) record_err(err, 1);
        break;
      }
    }
  };
  wait_bar(&sm.bar_k);
  __syncthreads();
  bool failed = sm.abort != 0;
  // Scores S[h][t] = q_h . k_t on the tensor cores; A rows 0/1 = the two heads.
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    qa[kk][0] = lane < 8 ? *reinterpret_cast<const uint32_t *>(&sm.q[lane >> 2][16 * kk + 2 * (lane & 3)]) : 0u;
    qa[kk][1] = lane < 8 ? *reinterpret_cast<const uint32_t *>(&sm.q[lane >> 2][16 * kk + 8 + 2 * (lane & 3)]) : 0u;
  }
  float wmax = -INFINITY;
  const int ntile = (ntok + 7) >> 3;
  if (!failed) {
    // Two tiles per warp and step (a split holds at most 8 tiles over 4
    // warps), their MMA chains interleaved; each tile's chain is unchanged.
    for (int tile = warp; tile < ntile; tile += 8) {
      const __half *kbase = &sm.k[0][0];
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      // Token of this lane's B column; the 8 tokens of a tile sit in different
      // swizzle rows, so the loads below are bank-conflict free.  A second
      // tile past the split reads rows of the first (results unused).
      const int tok0 = tile * 8 + (lane >> 2);
      const int tok1 = tile + 4 < ntile ? tok0 + 32 : tok0;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int c0 = 16 * kk + 2 * (lane & 3);
        const uint32_t b00 = *reinterpret_cast<const uint32_t *>(kbase + k_swz(tok0, c0));
        const uint32_t b01 = *reinterpret_cast<const uint32_t *>(kbase + k_swz(tok0, c0 + 8));
        const uint32_t b10 = *reinterpret_cast<const uint32_t *>(kbase + k_swz(tok1, c0));
        const uint32_t b11 = *reinterpret_cast<const uint32_t *>(kbase + k_swz(tok1, c0 + 8));
        mma16816(d[0], qa[kk][0], qa[kk][1], b00, b01);
        mma16816(d[1], qa[kk][0], qa[kk][1], b10, b11);
      }
      if (lane < 8) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int tl = tile + 4 * u;
          if (tl >= ntile) continue;
          const int tt = tl * 8 + 2 * (lane & 3);
          const float s0 = d[u][0] * attn_scale, s1 = d[u][1] * attn_scale;
          if (tt < ntok) {
            sm.sc[lane >> 2][tt] = s0;
            wmax = fmaxf(wmax, s0);
          }
          if (tt + 1 < ntok) {
            sm.sc[lane >> 2][tt + 1] = s1;
            wmax = fmaxf(wmax, s1);
          }
        }
      }
    }
  }
  wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 1));
  wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 2));
  if (lane == 0 || lane == 4) sm.red[warp][lane >> 2] = wmax;
  __syncthreads();
  const int hh = tid >> 6;             // head of this thread for softmax and P.V
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) m = fmaxf(m, sm.red[i][hh]);
  // p = expf(s - m) (megakernel.cu:490-494); 64 threads per head.
  float psum = 0.f;
  if (!failed)
    for (int t = tid & 63; t < ntok; t += 64) {
      const float p = expf(sm.sc[hh][t] - m);
      sm.sc[hh][t] = p;
      psum += p;
    }
  psum = warp_sum(psum);
  __syncthreads();  // all reads of sm.red (maxima) are done before it is reused
  if (lane == 0) sm.red[warp][0] = psum;
  __syncthreads();
  const float l = sm.red[2 * hh][0] + sm.red[2 * hh + 1][0];
  wait_bar(&sm.bar_v);
  __syncthreads();
  failed = sm.abort != 0;
  // P.V: thread (hh, dp) owns dims 2dp, 2dp+1 of head hh.
  const int dp = tid & 63;
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  if (!failed) {
    const __half2 *vcol = reinterpret_cast<const __half2 *>(sm.v) + dp;
    const float *pr = sm.sc[hh];
    int t = 0;
    for (; t + 1 < ntok; t += 2) {
      const float2 v0 = __half22float2(vcol[t * (HD / 2)]);
      const float2 v1 = __half22float2(vcol[(t + 1) * (HD / 2)]);
      a0 = fmaf(pr[t], v0.x, a0);
      a1 = fmaf(pr[t], v0.y, a1);
      b0 = fmaf(pr[t + 1], v1.x, b0);
      b1 = fmaf(pr[t + 1], v1.y, b1);
    }
    if (t < ntok) {
      const float2 v0 = __half22float2(vcol[t * (HD / 2)]);
      a0 = fmaf(pr[t], v0.x, a0);
      a1 = fmaf(pr[t], v0.y, a1);
    }
  }
  float *pp = part + ((static_cast<size_t>(row) * NKV + g) * max_splits + j) * 2 * PART + hh * PART;
  pp[2 * dp] = a0 + b0;
  pp[2 * dp + 1] = a1 + b1;
  if (dp == 0) {
    pp[HD] = failed ? -INFINITY : m;
    pp[HD + 1] = failed ? 0.f : l;
  }
}

// grid (16 q heads, rows), 128 threads: out = half(sum_j acc_j e^{m_j-M} * (1 / sum_j l_j e^{m_j-M})).
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float *__restrict__ part,
                                                          const int *__restrict__ positions,
                                                          __half *__restrict__ attn, int max_splits) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  __shared__ float s_m[HD], s_l[HD];
  const int qh = blockIdx.x, row = blockIdx.y, d = threadIdx.x;
  const int g = qh >> 1, h = qh & 1;
  const int ns = min(max_splits, max(0, (positions[row] + 1 + CH - 1) / CH));
  const float *pp = part + (static_cast<size_t>(row) * NKV + g) * max_splits * 2 * PART + h * PART;
  float A = 0.f, L = 0.f;
  if (ns <= HD) {
    // Thread j loads split j's (m, l): one round trip for all of them, where
    // a loop over the splits would wait for each load in turn.
    if (d < ns) {
      s_m[d] = pp[d * 2 * PART + HD];
      s_l[d] = pp[d * 2 * PART + HD + 1];
    }
    __syncthreads();
    float M = -INFINITY;
    for (int j = 0; j < ns; ++j) M = fmaxf(M, s_m[j]);
    if (M != -INFINITY) {
      // Eight splits' acc[d] loaded before their adds; the sums run in split order.
      for (int j0 = 0; j0 < ns; j0 += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = j0 + u < ns ? pp[(j0 + u) * 2 * PART + d] : 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          if (j < ns) {
            const float mj = s_m[j];
            const float f = mj == -INFINITY ? 0.f : expf(mj - M);
            L += s_l[j] * f;
            A = fmaf(v[u], f, A);
          }
        }
      }
    }
  } else {
    float M = -INFINITY;
    for (int j = 0; j < ns; ++j) M = fmaxf(M, pp[j * 2 * PART + HD]);
    if (M != -INFINITY) {
      for (int j = 0; j < ns; ++j) {
        const float mj = pp[j * 2 * PART + HD];
        const float f = mj == -INFINITY ? 0.f : expf(mj - M);
        L += pp[j * 2 * PART + HD + 1] * f;
        A = fmaf(pp[j * 2 * PART + d], f, A);
      }
    }
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  attn[static_cast<size_t>(row) * QS + qh * HD + d] = __float2half_rn(A * inv);
}

// --------------------------------------------------- post-attention RMSNorm
// sact = half(float(half(act)) * rstd * w), rstd from the fp32 act (megakernel.cu:614-638).
// When the o_proj GEMM left K slices (`part`), this kernel finishes it first:
// act = (sum of the slices in slice order) + float(res16), stored to `act`
// (the bits of splitk_reduce_kernel's EPI_F32_RES16).
__global__ void __launch_bounds__(256) post_norm_kernel(float *__restrict__ act,
                                                        const float *__restrict__ part, int splits,
                                                        const __half *__restrict__ res16,
                                                        const __half *__restrict__ w,
                                                        __half *__restrict__ sact, int rows) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float4 *a4 = reinterpret_cast<float4 *>(act + static_cast<size_t>(row) * H);
  float4 v[8];
  uint2 wv[8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) wv[j] = reinterpret_cast<const uint2 *>(w)[lane + 32 * j];  // before the row's loads
  if (part != nullptr) {
    const size_t slice4 = static_cast<size_t>(rows) * H / 4;
    const float4 *p4 = reinterpret_cast<const float4 *>(part + static_cast<size_t>(row) * H) + lane;
    uint2 ru[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) ru[j] = reinterpret_cast<const uint2 *>(res16 + static_cast<size_t>(row) * H)[lane + 32 * j];
    if (splits <= 4) {
      // Every slice requested before the first add; the adds run in slice order.
      float4 c[4][8];
#pragma unroll
      for (int z = 0; z < 4; ++z)
#pragma unroll
        for (int j = 0; j < 8; ++j) c[z][j] = z < splits ? p4[z * slice4 + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = c[0][j];
#pragma unroll
      for (int z = 1; z < 4; ++z)
        if (z < splits)
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = add4(v[j], c[z][j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = p4[32 * j];
#pragma unroll 4
      for (int z = 1; z < splits; ++z) {
        float4 c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = p4[z * slice4 + 32 * j];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = add4(v[j], c[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half2 *r2 = reinterpret_cast<const __half2 *>(&ru[j]);
      v[j] = add4(v[j], make_float4(__low2float(r2[0]), __high2float(r2[0]), __low2float(r2[1]), __high2float(r2[1])));
      a4[lane + 32 * j] = v[j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = a4[lane + 32 * j];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ss = fmaf(v[j].x, v[j].x, ss);
    ss = fmaf(v[j].y, v[j].y, ss);
    ss = fmaf(v[j].z, v[j].z, ss);
    ss = fmaf(v[j].w, v[j].w, ss);
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / static_cast<float>(H) + EPS);
  __half *o = sact + static_cast<size_t>(row) * H;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = 4 * (lane + 32 * j);
    const float x[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    const __half *wj = reinterpret_cast<const __half *>(&wv[j]);  // w[e .. e + 3]
    __half r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      r[i] = __float2half_rn(
          __fmul_rn(__fmul_rn(__half2float(__float2half_rn(x[i])), rstd), __half2float(wj[i])));
    *reinterpret_cast<uint2 *>(o + e) = *reinterpret_cast<const uint2 *>(r);
  }
}

// ------------------------------------------------------------ final RMSNorm
// norm = (h * inv) * w in fp32 (megakernel.cu:890-919); norm16 = half(norm)
// feeds the lm_head GEMM, norm32 (optional) is the caller's logits tap.
__global__ void __launch_bounds__(256) final_norm_kernel(__half *__restrict__ hidden,
                                                         const float *__restrict__ part, int splits,
                                                         const float *__restrict__ res32,
                                                         const __half *__restrict__ w,
                                                         __half *__restrict__ norm16,
                                                         float *__restrict__ norm32, int rows) {
  qb200::griddep_wait();  // everything below reads or overwrites earlier kernels' data
  qb200::griddep_launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  __half *hr = hidden + static_cast<size_t>(row) * H;
  uint4 v[4];
  float ss = 0.f;
  if (part != nullptr) {  // the last down projection's K slices (as input_norm_kernel)
    reduce_down_row(part, splits, res32, rows, row, lane, v);
#pragma unroll
    for (int j = 0; j < 4; ++j) reinterpret_cast<uint4 *>(hr)[lane + 32 * j] = v[j];
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = reinterpret_cast<const uint4 *>(hr)[lane + 32 * j];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&v[j]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h2[i]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(H) + EPS);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = 8 * (lane + 32 * j);
    const uint4 wv = reinterpret_cast<const uint4 *>(w)[lane + 32 * j];
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&v[j]);
    const __half2 *w2 = reinterpret_cast<const __half2 *>(&wv);
    float nv[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h2[i]);
      const float2 g = __half22float2(w2[i]);
      nv[2 * i] = __fmul_rn(__fmul_rn(f.x, inv), g.x);
      nv[2 * i + 1] = __fmul_rn(__fmul_rn(f.y, inv), g.y);
    }
    uint4 o16;
    __half2 *o2 = reinterpret_cast<__half2 *>(&o16);
#pragma unroll
    for (int i = 0; i < 4; ++i) o2[i] = __floats2half2_rn(nv[2 * i], nv[2 * i + 1]);
    reinterpret_cast<uint4 *>(norm16 + static_cast<size_t>(row) * H)[lane + 32 * j] = o16;
    if (norm32 != nullptr) {
      float4 *n4 = reinterpret_cast<float4 *>(norm32 + static_cast<size_t>(row) * H + e);
      n4[0] = make_float4(nv[0], nv[1], nv[2], nv[3]);
      n4[1] = make_float4(nv[4], nv[5], nv[6], nv[7]);
    }
  }
}

}  // namespace qb200b

// ====================================================================== host
using namespace qb200b;
using qb200tc::GemmArgs;

namespace {

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return qb200_set_error(code, buf);
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t up256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

struct Workspace {
  __half *hidden, *xn, *qkv, *qrot, *attn, *sact, *inter, *norm16;
  float *act, *part, *arg_val, *splitk;
  int *arg_idx;
  unsigned long long *err;
};

// Carves the workspace for max_rows rows (layout shared by size and carve).
size_t carve(uint8_t *base, int max_rows, int max_splits, int lm_tiles, Workspace *w) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? base + off : nullptr;
    off += up256(bytes);
    return p;
  };
  const size_t R = static_cast<size_t>(max_rows);
  Workspace t{};
  t.hidden = reinterpret_cast<__half *>(take(R * H * 2));
  t.xn = reinterpret_cast<__half *>(take(R * H * 2));
  t.qkv = reinterpret_cast<__half *>(take(R * QKV * 2));
  t.qrot = reinterpret_cast<__half *>(take(R * QS * 2));
  t.attn = reinterpret_cast<__half *>(take(R * QS * 2));
  t.sact = reinterpret_cast<__half *>(take(R * H * 2));
  t.inter = reinterpret_cast<__half *>(take(R * IM * 2));
  t.norm16 = reinterpret_cast<__half *>(take(R * H * 2));
  t.act = reinterpret_cast<float *>(take(R * H * 4));
  t.part = reinterpret_cast<float *>(take(R * NKV * max_splits * 2 * PART * 4));
  t.arg_val = reinterpret_cast<float *>(take(R * lm_tiles * 4));
  t.arg_idx = reinterpret_cast<int *>(take(R * lm_tiles * 4));
  t.splitk = reinterpret_cast<float *>(take(KSPLIT * R * H * 4));
  t.err = reinterpret_cast<unsigned long long *>(take(64));
  if (w) *w = t;
  return off;
}

struct Plan {
  int num_layers, num_seqs, max_seq, max_rows, max_splits, lm_tiles;
  QwenBatchedLayer layers[64];
  const __half *embed, *final_norm, *cos_t, *sin_t;
  __half *k_pool, *v_pool;
  Workspace ws;
  KvGeom kg;
  GemmPlan g_qkv[64], g_o[64], g_gu[64], g_down[64], g_lm;
  // Per projection (0 q|k|v, 1 o_proj, 2 gate/up, 3 down): K slices and how
  // they are added (1: inside a thread-block cluster; 0: partial tiles in the
  // workspace plus a reduction kernel).
  int ksplit[4], kcluster[4];
  CUtensorMap tm_k;   // K pool as [pages * layers * 8 * page_tokens rows, 128], 64 x CH boxes, 128B swizzle
};

// The lm_head GEMM takes 256-column tiles: the 151,936-row embedding is
// the one operand that matters, and wider tiles re-read the activation rows
// half as often.
constexpr int LM_BN = 256;
int lm_tiles_for(int) { return (VOCAB + LM_BN - 1) / LM_BN; }

}  // namespace

extern "C" {

long long qwen_b200_batched_workspace(int max_rows, int max_seq) {
  if (max_rows < 1 || max_seq < 1) return 0;
  const int max_splits = (max_seq + CH - 1) / CH;
  return static_cast<long long>(carve(nullptr, max_rows, max_splits, lm_tiles_for(max_rows), nullptr));
}

}  // extern "C"

namespace {

int create_plan(void **handle, const QwenBatchedLayer *layers, int num_layers, const void *embed,
                const void *final_norm, const void *cos_table, const void *sin_table, void *k_pool,
                void *v_pool, int num_seqs, int max_seq, int max_rows, void *workspace,
                long long workspace_bytes, const int *page_table, int num_pages, int max_pages) {
  qb200_clear_error();
  if (handle == nullptr || layers == nullptr) return fail(13, "null pointer argument");
  *handle = nullptr;
  if (num_layers < 1 || num_layers > 64) return fail(10, "num_layers=%d out of range [1, 64]", num_layers);
  if (num_seqs < 1 || max_seq < 1 || max_seq > 65536 || max_rows < 1 || max_rows > 65535 * 8)
    return fail(10, "num_seqs=%d max_seq=%d max_rows=%d out of range", num_seqs, max_seq, max_rows);
  if (page_table != nullptr && (num_pages < 1 || max_pages < 1 || static_cast<long long>(max_pages) * PAGE < max_seq))
    return fail(10, "paged pools: num_pages=%d, max_pages=%d pages of %d tokens must cover max_seq=%d",
                num_pages, max_pages, PAGE, max_seq);
  for (const void *p : {embed, final_norm, cos_table, sin_table, static_cast<const void *>(k_pool),
                        static_cast<const void *>(v_pool), static_cast<const void *>(workspace)})
    if (p == nullptr || !al16(p)) return fail(14, "pointers must be non-null and 16-byte aligned");
  for (int l = 0; l < num_layers; ++l) {
    const QwenBatchedLayer &L = layers[l];
    for (const void *p : {L.input_norm, L.w_qkv, L.q_norm, L.k_norm, L.w_o, L.post_norm, L.w_gu,
                          L.w_down})
      if (p == nullptr || !al16(p)) return fail(14, "layer %d: weight pointers must be non-null and 16-byte aligned", l);
  }
  const long long need = qwen_b200_batched_workspace(max_rows, max_seq);
  if (workspace_bytes < need)
    return fail(15, "workspace of %lld bytes, need %lld", workspace_bytes, need);
  Plan *p = new (std::nothrow) Plan();
  if (p == nullptr) return fail(5, "out of host memory");
  p->num_layers = num_layers;
  p->num_seqs = num_seqs;
  p->max_seq = max_seq;
  p->max_rows = max_rows;
  p->max_splits = (max_seq + CH - 1) / CH;
  p->lm_tiles = lm_tiles_for(max_rows);
  for (int l = 0; l < num_layers; ++l) p->layers[l] = layers[l];
  p->embed = static_cast<const __half *>(embed);
  p->final_norm = static_cast<const __half *>(final_norm);
  p->cos_t = static_cast<const __half *>(cos_table);
  p->sin_t = static_cast<const __half *>(sin_table);
  p->k_pool = static_cast<__half *>(k_pool);
  p->v_pool = static_cast<__half *>(v_pool);
  p->kg.page_table = page_table;
  p->kg.num_layers = num_layers;
  p->kg.max_pages = page_table != nullptr ? max_pages : 1;
  p->kg.num_pages = page_table != nullptr ? num_pages : num_seqs;
  p->kg.page_tokens = page_table != nullptr ? PAGE : max_seq;
  carve(static_cast<uint8_t *>(workspace), max_rows, p->max_splits, p->lm_tiles, &p->ws);
  // Tiling of the four projections: tile width (0: by output size), K slices,
  // cluster reduction.  QB200_GEMM_CFG="name:bn:ksplit:cluster,..." (names
  // qkv, o, gu, down) overrides it, for tuning runs.
  static const char *names[4] = {"qkv", "o", "gu", "down"};
  int bn_cfg[4] = {0, 0, 0, 0};
  const int ncols[4] = {QKV, H, 2 * IM, H};
  const int kdims[4] = {H, QS, H, IM};
  for (int i = 0; i < 4; ++i) {
    p->ksplit[i] = ncols[i] == H ? KSPLIT : 1;
    p->kcluster[i] = 0;
  }
  if (const char *env = getenv("QB200_GEMM_CFG")) {
    char buf[256];
    strncpy(buf, env, sizeof(buf) - 1);
    buf[sizeof(buf) - 1] = 0;
    for (char *tok = strtok(buf, ","); tok != nullptr; tok = strtok(nullptr, ",")) {
      char name[16] = {0};
      int bn = 0, ks = 1, cl = 0;
      if (sscanf(tok, "%15[^:]:%d:%d:%d", name, &bn, &ks, &cl) < 2) continue;
      for (int i = 0; i < 4; ++i) {
        if (strcmp(name, names[i]) != 0) continue;
        bn_cfg[i] = bn;
        p->ksplit[i] = ks < 1 ? 1 : ks;
        p->kcluster[i] = cl;
      }
    }
  }
  int rc = 0;
  for (int i = 0; i < 4 && rc == 0; ++i) {
    // K slices: whole k-blocks each; partial tiles must fit the workspace,
    // else the slices are added inside a cluster (at most 8).
    if (p->ksplit[i] > kdims[i] / qb200tc::BK) p->ksplit[i] = kdims[i] / qb200tc::BK;
    if (p->ksplit[i] > 1 && !p->kcluster[i] &&
        static_cast<long long>(p->ksplit[i]) * ncols[i] > static_cast<long long>(KSPLIT) * H)
      p->kcluster[i] = 1;
    if (p->kcluster[i] && p->ksplit[i] > 8) p->ksplit[i] = 8;
  }
  for (int l = 0; l < num_layers && rc == 0; ++l) {
    const QwenBatchedLayer &L = layers[l];
    rc = qb200_gemm_make_maps(&p->g_qkv[l], p->ws.xn, L.w_qkv, max_rows, QKV, H, H, H);
    if (!rc) rc = qb200_gemm_make_maps(&p->g_o[l], p->ws.attn, L.w_o, max_rows, H, QS, QS, QS);
    if (!rc) rc = qb200_gemm_make_maps(&p->g_gu[l], p->ws.sact, L.w_gu, max_rows, 2 * IM, H, H, H);
    if (!rc) rc = qb200_gemm_make_maps(&p->g_down[l], p->ws.inter, L.w_down, max_rows, H, IM, IM, IM);
    GemmPlan *gp[4] = {&p->g_qkv[l], &p->g_o[l], &p->g_gu[l], &p->g_down[l]};
    for (int i = 0; i < 4 && rc == 0; ++i)
      if (bn_cfg[i] != 0) rc = qb200_gemm_set_bn(gp[i], bn_cfg[i]);
  }
  if (!rc) rc = qb200_gemm_make_maps(&p->g_lm, p->ws.norm16, embed, max_rows, VOCAB, H, H, H);
  if (!rc) rc = qb200_gemm_set_bn(&p->g_lm, LM_BN);
  const long long k_rows = static_cast<long long>(p->kg.num_pages) * num_layers * NKV * p->kg.page_tokens;
  if (!rc && k_rows > 0x7fffffffll) rc = fail(10, "KV pool of %lld rows exceeds the tensor-map range", k_rows);
  if (!rc) rc = qb200_encode_f16_2d(&p->tm_k, k_pool, HD, k_rows, HD, HD / 2, CH, 1);
  if (rc) {
    delete p;
    return rc;
  }
  const int smem = static_cast<int>(sizeof(AttnSmem)) + 1024;
  cudaError_t e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaMemset(p->ws.err, 0, 64);
  if (e != cudaSuccess) {
    delete p;
    return fail(4, "batched set-up: %s", cudaGetErrorString(e));
  }
  *handle = p;
  return 0;
}

}  // namespace

extern "C" {

int qwen_b200_batched_create(void **handle, const QwenBatchedLayer *layers, int num_layers,
                             const void *embed, const void *final_norm, const void *cos_table,
                             const void *sin_table, void *k_pool, void *v_pool, int num_seqs,
                             int max_seq, int max_rows, void *workspace, long long workspace_bytes) {
  return create_plan(handle, layers, num_layers, embed, final_norm, cos_table, sin_table, k_pool, v_pool,
                     num_seqs, max_seq, max_rows, workspace, workspace_bytes, nullptr, 0, 0);
}

int qwen_b200_batched_create_paged(void **handle, const QwenBatchedLayer *layers, int num_layers,
                                   const void *embed, const void *final_norm, const void *cos_table,
                                   const void *sin_table, void *k_pool, void *v_pool, int num_pages,
                                   const int *page_table, int max_pages_per_seq, int num_seqs,
                                   int max_seq, int max_rows, void *workspace,
                                   long long workspace_bytes) {
  if (page_table == nullptr) {
    qb200_clear_error();
    return fail(13, "null page table");
  }
  return create_plan(handle, layers, num_layers, embed, final_norm, cos_table, sin_table, k_pool, v_pool,
                     num_seqs, max_seq, max_rows, workspace, workspace_bytes, page_table, num_pages,
                     max_pages_per_seq);
}

}  // extern "C"

namespace {

// One projection GEMM of a layer with its plan's K split.
int run_proj(Plan *p, int i, const GemmPlan &gp, int epi, const GemmArgs &g, float *partial,
             cudaStream_t st) {
  if (p->ksplit[i] > 1)
    return qb200_gemm_run_splitk(gp, epi, g, p->ksplit[i], p->kcluster[i] ? nullptr : partial, st);
  return qb200_gemm_run(gp, epi, g, st);
}

// Projection i split over K into fp32 slices [ksplit][rows][N] at `partial`
// and left unreduced: the next kernel adds the slices (in slice order) and
// the residual, as splitk_reduce_kernel would have.  True when it did so;
// false (nothing launched) when projection i is not split that way.
bool run_proj_slices(Plan *p, int i, const GemmPlan &gp, const GemmArgs &g, float *partial, cudaStream_t st,
                     int *rc) {
  *rc = 0;
  if (p->ksplit[i] < 2 || p->kcluster[i]) return false;
  GemmArgs gs = g;
  gs.out = partial;
  gs.ldo = gp.N;
  gs.res = nullptr;
  gs.k_splits = p->ksplit[i];
  *rc = qb200_gemm_run(gp, qb200tc::EPI_PARTIAL, gs, st);
  return true;
}

// Every layer of a step plus the final RMSNorm (w.norm16 feeds the lm_head).
int step_layers(Plan *p, int rows, const int *seq_ids, const int *positions, const int *tokens_in,
                float *norm_out, int max_position, float attn_scale, cudaStream_t st) {
  const Workspace &w = p->ws;
  // The norm kernels take one warp per row; one-warp CTAs spread the rows
  // over all SMs (eight rows per CTA put the 256 rows of a step on 32 SMs).
  const int nsplit = max_position / CH + 1;
  const int smem = static_cast<int>(sizeof(AttnSmem)) + 1024;
  // Every kernel of the step is launched as a programmatic dependent of the
  // previous one (it may be scheduled while its predecessor finishes and waits
  // for it with griddepcontrol.wait before touching its data).  The first
  // follows whatever the caller enqueued last, which it waits for the same way.
#define LAUNCH(kernel, grid, block, smem_bytes, ...)                                            \
  do {                                                                                         \
    const cudaError_t le = qb200_launch(kernel, grid, block, smem_bytes, st, true, __VA_ARGS__); \
    if (le != cudaSuccess) return fail(20, "%s launch: %s", #kernel, cudaGetErrorString(le));   \
  } while (0)
  // The o_proj and down projections split over K leave their slices to the
  // following norm kernel (post-attention norm, next layer's input norm or
  // the final norm), which finishes the reduction and the residual.
  const float *down_part = nullptr;  // slices of the previous layer's down projection
  for (int l = 0; l < p->num_layers; ++l) {
    const QwenBatchedLayer &L = p->layers[l];
    LAUNCH(input_norm_kernel, dim3(rows), dim3(32), 0, w.hidden, l == 0 ? p->embed : nullptr,
           tokens_in, down_part, p->ksplit[3], static_cast<const float *>(w.act),
           static_cast<const __half *>(L.input_norm), w.xn, rows, w.err);
    GemmArgs g{};
    g.M = rows;
    g.err = w.err;
    g.pdl = 1;
    g.out = w.qkv;
    g.ldo = QKV;
    if (int rc = run_proj(p, 0, p->g_qkv[l], qb200tc::EPI_F16, g, w.splitk, st)) return rc;
    LAUNCH(qk_rope_kv_kernel, dim3(rows), dim3(32 * (NQ + NKV)), 0, static_cast<const __half *>(w.qkv),
           static_cast<const __half *>(L.q_norm), static_cast<const __half *>(L.k_norm), p->cos_t,
           p->sin_t, seq_ids, positions, p->k_pool, p->v_pool, w.qrot, l, p->kg, p->max_seq,
           p->num_seqs, w.err);
    LAUNCH(attn_split_kernel, dim3(nsplit, NKV, rows), dim3(ATT_THREADS), smem, p->tm_k,
           static_cast<const __half *>(w.qrot), static_cast<const __half *>(p->k_pool),
           static_cast<const __half *>(p->v_pool), seq_ids, positions, w.part, l, p->kg,
           p->max_seq, p->max_splits, p->num_seqs, attn_scale, w.err);
    LAUNCH(attn_combine_kernel, dim3(NQ, rows), dim3(HD), 0, static_cast<const float *>(w.part),
           positions, w.attn, p->max_splits);
    g.out = w.act;
    g.ldo = H;
    g.res = w.hidden;
    int rc = 0;
    const bool o_sliced = run_proj_slices(p, 1, p->g_o[l], g, w.splitk, st, &rc);
    if (rc) return rc;
    if (!o_sliced && (rc = run_proj(p, 1, p->g_o[l], qb200tc::EPI_F32_RES16, g, w.splitk, st))) return rc;
    LAUNCH(post_norm_kernel, dim3(rows), dim3(32), 0, w.act,
           o_sliced ? static_cast<const float *>(w.splitk) : nullptr, p->ksplit[1],
           static_cast<const __half *>(w.hidden), static_cast<const __half *>(L.post_norm), w.sact, rows);
    g.out = w.inter;
    g.ldo = IM;
    g.res = nullptr;
    if (int rc = run_proj(p, 2, p->g_gu[l], qb200tc::EPI_SWIGLU, g, w.splitk, st)) return rc;
    g.out = w.hidden;
    g.ldo = H;
    g.res = w.act;
    const bool down_sliced = run_proj_slices(p, 3, p->g_down[l], g, w.splitk, st, &rc);
    if (rc) return rc;
    if (!down_sliced && (rc = run_proj(p, 3, p->g_down[l], qb200tc::EPI_F16_RES32, g, w.splitk, st))) return rc;
    down_part = down_sliced ? w.splitk : nullptr;
  }
  LAUNCH(final_norm_kernel, dim3(rows), dim3(32), 0, w.hidden, down_part, p->ksplit[3],
         static_cast<const float *>(w.act), p->final_norm, w.norm16, norm_out, rows);
#undef LAUNCH
  return 0;
}

int check_step(Plan *p, int rows, const int *seq_ids, const int *positions, const int *tokens_in,
               const void *out, int max_position) {
  if (p == nullptr) return fail(13, "null handle");
  if (rows < 1 || rows > p->max_rows) return fail(10, "rows=%d out of range [1, %d]", rows, p->max_rows);
  if (max_position < 0 || max_position >= p->max_seq)
    return fail(11, "max_position=%d outside the KV cache (max_seq=%d)", max_position, p->max_seq);
  if (seq_ids == nullptr || positions == nullptr || tokens_in == nullptr || out == nullptr)
    return fail(13, "null pointer argument");
  return 0;
}

}  // namespace

extern "C" {

int qwen_b200_batched_step(void *handle, int rows, const int *seq_ids, const int *positions,
                           const int *tokens_in, int *tokens_out, float *norm_out, int max_position,
                           float attn_scale, void *stream) {
  qb200_clear_error();
  Plan *p = static_cast<Plan *>(handle);
  if (int rc = check_step(p, rows, seq_ids, positions, tokens_in, tokens_out, max_position)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Workspace &w = p->ws;
  if (int rc = step_layers(p, rows, seq_ids, positions, tokens_in, norm_out, max_position, attn_scale, st))
    return rc;
  GemmArgs g{};
  g.M = rows;
  g.err = w.err;
  g.pdl = 1;
  g.out = nullptr;
  g.ldo = 1;
  g.part_val = w.arg_val;
  g.part_idx = w.arg_idx;
  if (int rc = qb200_gemm_run_argmax(p->g_lm, g, st)) return rc;
  if (int rc = qb200_argmax_reduce(w.arg_val, w.arg_idx, p->lm_tiles, rows, tokens_out, st, true))
    return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "batched step launch: %s", cudaGetErrorString(e));
  return 0;
}

int qwen_b200_batched_step_logits(void *handle, int rows, const int *seq_ids, const int *positions,
                                  const int *tokens_in, float *logits, long long ld, float *norm_out,
                                  int max_position, float attn_scale, void *stream) {
  qb200_clear_error();
  Plan *p = static_cast<Plan *>(handle);
  if (int rc = check_step(p, rows, seq_ids, positions, tokens_in, logits, max_position)) return rc;
  if (ld < VOCAB || (ld & 3) != 0 || (reinterpret_cast<uintptr_t>(logits) & 15u) != 0)
    return fail(14, "logits: ld=%lld must be >= %d and a multiple of 4, pointer 16-byte aligned", ld, VOCAB);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Workspace &w = p->ws;
  if (int rc = step_layers(p, rows, seq_ids, positions, tokens_in, norm_out, max_position, attn_scale, st))
    return rc;
  GemmArgs g{};
  g.M = rows;
  g.err = w.err;
  g.pdl = 1;
  g.out = logits;
  g.ldo = static_cast<int>(ld);
  if (int rc = qb200_gemm_run(p->g_lm, qb200tc::EPI_F32, g, st)) return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "batched step launch: %s", cudaGetErrorString(e));
  return 0;
}

int qwen_b200_batched_status(void *handle, uint64_t *detail) {
  Plan *p = static_cast<Plan *>(handle);
  if (p == nullptr) return -1;
  unsigned long long v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&v, p->ws.err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return -2;
  if (detail) *detail = v;
  if (v != 0) cudaMemset(p->ws.err, 0, sizeof(v));  // reported once
  return static_cast<int>(v >> 32);
}

void qwen_b200_batched_destroy(void *handle) { delete static_cast<Plan *>(handle); }

}  // extern "C"
