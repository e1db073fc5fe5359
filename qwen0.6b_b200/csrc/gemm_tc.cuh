// gemm_tc.cuh - tcgen05 (5th-generation tensor core) GEMM for sm_100a with the
// fused epilogues of the batched decode layer.
//
//   C[M, N] = A[M, K] . B[N, K]^T      A, B fp16 K-major (row-major [rows, K]),
//                                       fp32 accumulation in tensor memory;
//   or, with an MN-major B (the weight stored [K, N], N contiguous, as the
//   upstream Tools/swiglu operators keep it), C[M, N] = A[M, K] . B[K, N].
//
// One CTA computes one 128 x BN tile over the whole K range:
//   warp 0      one lane streams A/B k-blocks (128 / BN rows x 64 halves) into a
//               STAGES-deep shared-memory ring with TMA (128-byte swizzle, no
//               multicast), completing on "full" mbarriers;
//   warp 1      allocates BN tensor-memory columns, then one lane issues
//               tcgen05.mma (M=128, N=BN, K=16) four times per k-block and
//               frees each stage with tcgen05.commit on its "empty" mbarrier;
//               a last commit signals the accumulator;
//   warps 2..5  epilogue: tcgen05.ld the accumulator rows of their TMEM lane
//               quadrant (warp % 4), apply the fused epilogue, store to global.
// Every mbarrier wait is bounded (wall clock); a wait that gives up records a
// status word, the roles fall through, and tensor memory is released only
// after the last issued MMA has completed (or its own bounded wait gave up).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace qb200tc {

using qb200::globaltimer_ns;
using qb200::mbar_arrive_expect_tx;
using qb200::mbar_init;
using qb200::mbar_try_wait;
using qb200::smem_u32;

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 halves = one 128-byte swizzle row
// Ring depth: at most as many 24 / 32 KB stages as fit next to the barriers
// (one CTA per SM); the launcher picks fewer (two CTAs per SM) for grids
// larger than the GPU.
template <int BN>
constexpr int max_stages() {
  return BN == 64 ? 8 : (BN == 128 ? 6 : 4);  // 24 / 32 / 48 KB stages
}
constexpr int THREADS = 192;           // 6 warps
// Row pitch (floats) of an epilogue warp's staging tile: 32 rows of up to 96
// values; 25 16-byte units per row (odd), so the row-parallel writes of 32
// lanes and the row-contiguous reads both spread over all banks.
constexpr int EPI_PITCH = 100;
constexpr long long WAIT_NS = 2000000000LL;

enum Epilogue : int {
  EPI_F16 = 0,         // out16[r, c] = half(acc)
  EPI_F32 = 1,         // out32[r, c] = acc
  EPI_F32_RES16 = 2,   // out32[r, c] = acc + float(res16[r, c])          (o_proj + residual)
  EPI_SWIGLU = 3,      // columns (2i, 2i+1) = (gate_i, up_i):
                       //   out16[r, i] = half(float(silu_half(half(g))) * u)
  EPI_F16_RES32 = 4,   // out16[r, c] = half(acc + res32[r, c])            (down + residual)
  EPI_ARGMAX = 5,      // part_val/part_idx[r, tile] = max / lowest argmax over the tile's columns
  EPI_PARTIAL = 6,     // split-K: out32[z, r, c] = this CTA's partial sum over its k-range z
  EPI_SWIGLU2 = 7,     // BL_MN2: accumulator columns [0, BN/2) = gate, [BN/2, BN) = up of the
                       //   same BN/2 outputs: g = acc + bias[c], u = acc + bias2[c] (fp32),
                       //   out16[r, c] = half(s), s = g / (1 + exp(-g)) * u, and with lo_col the
                       //   rounding residual half(s - half(s)) at column lo_col + c (so a following
                       //   GEMM over [hi | lo] with B's K wrapped sees s to ~22 bits); out2 / out3
                       //   (if set) = half(g), half(u)
};

// Layout of the B operand in global memory (and so in shared memory).
enum BLayout : int {
  BL_K = 0,    // [N, K] K-major; the tile is one 128-byte-swizzled TMA box
  BL_MN = 1,   // [K, N] MN-major; BN / 64 boxes of 64 columns x BK rows
  BL_MN2 = 2,  // two [K, N] MN-major matrices (gate, up): 64 columns of each (BN = 128)
};

struct GemmArgs {
  int M, N, K;
  int ldo;                      // leading dimension of the output (elements)
  void *out;                    // fp16 or fp32 [M, ldo]
  const void *res;              // residual (fp16 or fp32 [M, ldo]) or nullptr
  float *part_val;              // EPI_ARGMAX: [M, n_tiles]
  int *part_idx;
  int n_tiles;
  int k_splits;                 // grid.z: the K range is cut into this many slices (EPI_PARTIAL)
  int stages;                   // ring depth of this launch (<= max_stages<BN>())
  int cluster_k;                // split-K reduced inside a (1, 1, k_splits) cluster (see below)
  int pdl;                      // host side: launch as a programmatic dependent of the previous kernel
  unsigned long long *err;      // status word (nullptr: none)
  const void *bias;             // fp16 [N] added before rounding (EPI_F16, EPI_SWIGLU2 gate) or nullptr
  const void *bias2;            // fp16 [N] up bias of EPI_SWIGLU2 or nullptr
  void *out2, *out3;            // EPI_SWIGLU2: fp16 gate / up caches [M, ldo] or nullptr
  int lo_col;                   // EPI_SWIGLU2: > 0: also out16[r, lo_col + c] = half(s - half(s))
  int b_kwrap;                  // > 0: B's K coordinate wraps after this many k-blocks
  int m_fast;                   // grid.x walks the row tiles, grid.y the column tiles (set by the launcher)
  int a_box;                    // rows per A copy (the A map's box height: 128, or M rounded up to 8 when
                                //   M < 128 -- the slot's other rows only feed accumulator rows >= M)
};

template <int BN>
struct GemmSmem {
  static constexpr int MAX_STAGES = max_stages<BN>();
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr size_t bytes(int stages) { return static_cast<size_t>(stages) * STAGE + 256 + 1024; }
  // Ring stages the epilogue needs for its staging tiles: the clustered
  // split-K partial tile (128 rows of BN + 4 floats) or four warps' staging
  // rows (32 x EPI_PITCH floats each).
  static constexpr int min_stages(bool clustered) {
    const int need = clustered ? BM * (BN + 4) * 4 : 4 * 32 * EPI_PITCH * 4;
    return (need + STAGE - 1) / STAGE;
  }
};

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);        // start address
  d |= static_cast<uint64_t>(1u) << 16;                         // LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                 // SBO: next 8-row atom
  d |= static_cast<uint64_t>(1u) << 46;                         // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                         // SWIZZLE_128B
  return d;
}

// MN-major operand, 128-byte swizzle: each K row of 64 MN elements is 128 B,
// 8-row atoms are 1024 B apart (stride dimension), and the 64-element MN
// blocks are `lbo` bytes apart (leading dimension).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);        // start address
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;      // LBO: next 64-element MN block
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                 // SBO: next 8-row K atom
  d |= static_cast<uint64_t>(1u) << 46;                         // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                         // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: A, B fp16, D fp32, A K-major, M=128; B
// K-major, or MN-major ("transpose B", bit 16) when b_mn.
template <int BN>
__device__ __forceinline__ constexpr uint32_t idesc_f16(bool b_mn = false) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (b_mn ? (1u << 16) : 0u) |
         (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

// One k-block (K = 4 x 16) on a converged warp: an elected lane issues the
// four MMAs and the commit of their completion to the mbarrier at `bar`
// (shared address); the first MMA accumulates when `acc` is non-zero.
static_assert(BK == 64, "mma4_commit_elect covers one 64-element k-block");
__device__ __forceinline__ void mma4_commit_elect(uint32_t tmem_d, uint64_t a0, uint64_t a1, uint64_t a2,
                                                  uint64_t a3, uint64_t b0, uint64_t b1, uint64_t b2,
                                                  uint64_t b3, uint32_t idesc, uint32_t acc, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p, q, t;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "setp.ne.b32 q, %10, 0;\n\t"
      "setp.eq.b32 t, 0, 0;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %9, q;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %9, t;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %9, t;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %9, t;\n\t"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t}" ::"r"(tmem_d),
      "l"(a0), "l"(a1), "l"(a2), "l"(a3), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(acc), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// Two 32-column TMEM loads of this thread's lane (at taddr0 and taddr1) and
// one wait: v[0..31] from taddr0, v[32..63] from taddr1.  Loads and wait
// are one asm statement, so no use of v can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr0, uint32_t taddr1, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr0), "r"(taddr1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

static __device__ __noinline__ void gemm_record(unsigned long long *err, uint32_t code) {
  if (err == nullptr) return;
  const unsigned long long v = (static_cast<unsigned long long>(code) << 32) |
                               (static_cast<unsigned long long>(blockIdx.y & 0xffffu) << 16) |
                               (blockIdx.x & 0xffffu);
  atomicCAS(err, 0ull, v);
}

// Bounded wait; false when it gave up (or another role already did).
static __device__ __noinline__ bool gemm_wait_slow(uint64_t *bar, uint32_t parity,
                                            volatile uint32_t *abort, unsigned long long *err,
                                            uint32_t code) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
      *abort = 1;
      gemm_record(err, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool gemm_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort,
                                          unsigned long long *err, uint32_t code) {
  return mbar_try_wait(bar, parity) || gemm_wait_slow(bar, parity, abort, err, code);
}

// Half-precision SiLU with the upstream decode kernel's rounding steps
// (megakernel.cu:141-154): every operation on fp16, exp2 of the fp16
// argument evaluated in fp32 and rounded, reciprocal likewise.
__device__ __forceinline__ __half silu_half(__half x) {
  const __half log2e = __float2half_rn(1.44269504088896340736f);
  const __half t = __hmul_rn(__hneg(x), log2e);
  const __half e = __float2half_rn(exp2f(__half2float(t)));
  const __half d = __hadd_rn(__float2half_rn(1.0f), e);
  const __half r = __float2half_rn(1.0f / __half2float(d));
  return __hmul_rn(x, r);
}

// Output dtype of a staged epilogue.
template <int EPI>
constexpr bool kEpiF16Out = EPI == EPI_F16 || EPI == EPI_F16_RES32 || EPI == EPI_SWIGLU;

// Eight consecutive outputs x[0..7] of one row at element offset o: the
// residual of the epilogue added in fp32 (16-byte loads when `vec`).
template <int EPI>
__device__ __forceinline__ void add_residual8(const GemmArgs &g, size_t o, float (&x)[8], bool vec) {
  if constexpr (EPI == EPI_F32_RES16) {
    const __half *r = static_cast<const __half *>(g.res) + o;
    if (vec) {
      const uint4 u = *reinterpret_cast<const uint4 *>(r);
      const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[2 * i] = __fadd_rn(x[2 * i], __low2float(h[i]));
        x[2 * i + 1] = __fadd_rn(x[2 * i + 1], __high2float(h[i]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __fadd_rn(x[i], __half2float(r[i]));
    }
  } else if constexpr (EPI == EPI_F16_RES32) {
    const float *r = static_cast<const float *>(g.res) + o;
    if (vec) {
      const float4 a = reinterpret_cast<const float4 *>(r)[0], b = reinterpret_cast<const float4 *>(r)[1];
      const float rr[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __fadd_rn(x[i], rr[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __fadd_rn(x[i], r[i]);
    }
  }
}

// The same eight outputs rounded to the output type and stored: one or two
// 16-byte stores when `vec`, else element by element.
template <int EPI>
__device__ __forceinline__ void store_unit8(const GemmArgs &g, size_t o, const float (&x)[8], bool vec) {
  if constexpr (kEpiF16Out<EPI>) {
    __half *out = static_cast<__half *>(g.out) + o;
    if (vec) {
      uint4 pk;
      __half2 *h = reinterpret_cast<__half2 *>(&pk);
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
      *reinterpret_cast<uint4 *>(out) = pk;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = __float2half_rn(x[i]);
    }
  } else {
    float *out = static_cast<float *>(g.out) + o;
    if constexpr (EPI == EPI_PARTIAL) out += static_cast<size_t>(blockIdx.z) * g.M * g.ldo;
    if (vec) {
      reinterpret_cast<float4 *>(out)[0] = make_float4(x[0], x[1], x[2], x[3]);
      reinterpret_cast<float4 *>(out)[1] = make_float4(x[4], x[5], x[6], x[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = x[i];
    }
  }
}

// Epilogue of one warp (rows rbase..rbase+31 of the tile, TMEM lanes at tq)
// for EPI_F16, EPI_F32, EPI_F32_RES16, EPI_F16_RES32, EPI_SWIGLU and
// EPI_PARTIAL.  Per 64 accumulator columns: one TMEM load per row (thread),
// the per-element math of the epilogue, the fp32 results into the warp's
// staging rows; then the warp stores the 32 rows row-contiguously, 8 outputs
// per lane and step (the residual is added there), so that each store
// instruction writes whole 128-byte lines instead of 32 scattered pieces.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_staged(const GemmArgs &g, uint32_t tq, float *stg, int rbase, int n0,
                                                int lane) {
  constexpr bool PAIRS = EPI == EPI_SWIGLU;  // (gate, up) column pairs -> one output
  constexpr int OUTS = PAIRS ? 32 : 64;      // outputs per 64 accumulator columns
  constexpr int UPR = OUTS / 8;              // 8-output units per row
  const int nout = PAIRS ? g.N / 2 : g.N;
  const size_t esz = kEpiF16Out<EPI> ? 2 : 4;
  bool vec = (reinterpret_cast<uintptr_t>(g.out) & 15u) == 0 && (static_cast<size_t>(g.ldo) * esz) % 16 == 0;
  if constexpr (EPI == EPI_F32_RES16 || EPI == EPI_F16_RES32)
    vec = vec && (reinterpret_cast<uintptr_t>(g.res) & 15u) == 0 && (g.ldo % 8) == 0;
  float *srow = stg + lane * EPI_PITCH;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 64) {
    const int oc0 = PAIRS ? (n0 + c0) / 2 : n0 + c0;
    if (oc0 >= nout) break;  // warp-uniform
    float v[64];
    tmem_ld64(tq + c0, tq + c0 + 32, v);
    if constexpr (PAIRS) {
      // out = half(float(silu_half(half(gate))) * up), kept exactly as fp32.
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = __half2float(__float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(v[2 * i]))), v[2 * i + 1])));
    } else if constexpr (EPI == EPI_F16) {
      if (g.bias != nullptr) {
        const __half *b = static_cast<const __half *>(g.bias) + oc0;
        const int nv = min(64, nout - oc0);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < nv) v[i] = __fadd_rn(v[i], __half2float(b[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < OUTS / 4; ++i)
      reinterpret_cast<float4 *>(srow)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    __syncwarp();
    // Lane l takes the units l, l + 32, ... (unit u = row u / UPR, outputs
    // 8 (u % UPR) ..): every staged value and residual is loaded before the
    // first store, so the loads are not serialised behind the stores.
    float x[UPR][8];
    bool ok[UPR];
#pragma unroll
    for (int t = 0; t < UPR; ++t) {
      const int u = lane + 32 * t, r = u / UPR, j = u % UPR;
      const int row = rbase + r, oc = oc0 + 8 * j;
      ok[t] = row < g.M && oc < nout;
      const float4 *s4 = reinterpret_cast<const float4 *>(stg + r * EPI_PITCH) + 2 * j;
      const float4 a = s4[0], b = s4[1];
      x[t][0] = a.x; x[t][1] = a.y; x[t][2] = a.z; x[t][3] = a.w;
      x[t][4] = b.x; x[t][5] = b.y; x[t][6] = b.z; x[t][7] = b.w;
      if (ok[t]) add_residual8<EPI>(g, static_cast<size_t>(row) * g.ldo + oc, x[t], vec);
    }
    __syncwarp();  // the staging rows are rewritten by the next chunk
#pragma unroll
    for (int t = 0; t < UPR; ++t) {
      const int u = lane + 32 * t, r = u / UPR, j = u % UPR;
      if (ok[t]) store_unit8<EPI>(g, static_cast<size_t>(rbase + r) * g.ldo + oc0 + 8 * j, x[t], vec);
    }
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Eight halves into dst: one 16-byte store when `vec`, else element by element.
__device__ __forceinline__ void put_half8(__half *dst, const float (&x)[8], bool vec) {
  if (vec) {
    uint4 pk;
    __half2 *h = reinterpret_cast<__half2 *>(&pk);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    *reinterpret_cast<uint4 *>(dst) = pk;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = __float2half_rn(x[i]);
  }
}

// EPI_SWIGLU2 epilogue of one warp: accumulator columns [0, BN/2) are the
// gate and [BN/2, BN) the up projections of output columns n0/2 + c.  Per 32
// outputs: g and u (bias added in fp32), s = g / (1 + exp(-g)) * u staged as
// fp32, then stored row-contiguously as half(s), the residual
// half(s - half(s)) at column lo_col + c, and the gate / up caches.
template <int BN>
__device__ __forceinline__ void epilogue_swiglu2(const GemmArgs &g, uint32_t tq, float *stg, int rbase, int n0,
                                                 int lane) {
  const int nout = g.N / 2;
  __half *out = static_cast<__half *>(g.out);
  __half *out2 = static_cast<__half *>(g.out2);
  __half *out3 = static_cast<__half *>(g.out3);
  const __half *bias = static_cast<const __half *>(g.bias);
  const __half *bias2 = static_cast<const __half *>(g.bias2);
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = al(out) && (g.ldo % 8) == 0 && (g.lo_col % 8) == 0 && (out2 == nullptr || al(out2)) &&
                   (out3 == nullptr || al(out3));
  float *srow = stg + lane * EPI_PITCH;
#pragma unroll 1
  for (int c0 = 0; c0 < BN / 2; c0 += 32) {
    const int oc0 = n0 / 2 + c0;
    if (oc0 >= nout) break;  // warp-uniform
    float v[64];
    tmem_ld64(tq + c0, tq + BN / 2 + c0, v);
    const int nv = min(32, nout - oc0);
    if (bias != nullptr) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) v[i] = __fadd_rn(v[i], __half2float(bias[oc0 + i]));
    }
    if (bias2 != nullptr) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) v[32 + i] = __fadd_rn(v[32 + i], __half2float(bias2[oc0 + i]));
    }
    if (out2 != nullptr || out3 != nullptr) {  // the gate / up caches are staged only when asked for
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        reinterpret_cast<float4 *>(srow + 32)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        reinterpret_cast<float4 *>(srow + 64)[i] =
            make_float4(v[32 + 4 * i], v[33 + 4 * i], v[34 + 4 * i], v[35 + 4 * i]);
      }
    }
    // s = g * u * 1 / (1 + 2^(-g log2 e)) with one ex2.approx and one
    // rcp.approx per output (relative errors ~2^-22 and 1 ulp, plus |g| 2^-24
    // from the scaled argument): branch-free, so the 32 outputs overlap.  The
    // library exp and IEEE division each carry special-case branches that
    // serialised them (2.4 - 12 us per tile).  g -> -inf gives 2^+inf = inf
    // and a reciprocal of 0, so s = 0.  Far inside the fp16 ulp (2^-11) of
    // the stored hi part; the lo part carries the rest to ~2^-21.
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float e = ex2_approx(__fmul_rn(v[i], -1.4426950408889634f));
      v[i] = __fmul_rn(__fmul_rn(v[i], v[32 + i]), rcp_approx(__fadd_rn(1.0f, e)));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      reinterpret_cast<float4 *>(srow)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    __syncwarp();
    // Lane l takes the units l, l + 32, l + 64, l + 96 (row u / 4, outputs
    // 8 (u % 4) ..), all staged values loaded before the first store.
    const bool caches = out2 != nullptr || out3 != nullptr;
    float sv[4][8], gv[4][8], uv[4][8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int u = lane + 32 * t, r = u >> 2, j = u & 3;
      const float *sr = stg + r * EPI_PITCH + 8 * j;
#pragma unroll
      for (int i = 0; i < 8; ++i) sv[t][i] = sr[i];
      if (caches) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          gv[t][i] = sr[32 + i];
          uv[t][i] = sr[64 + i];
        }
      }
    }
    __syncwarp();  // the staging rows are rewritten by the next chunk
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int u = lane + 32 * t, r = u >> 2, j = u & 3;
      const int row = rbase + r, oc = oc0 + 8 * j;
      if (row >= g.M || oc >= nout) continue;
      float lo[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) lo[i] = __fsub_rn(sv[t][i], __half2float(__float2half_rn(sv[t][i])));
      const size_t o = static_cast<size_t>(row) * g.ldo + oc;
      put_half8(out + o, sv[t], vec);
      if (g.lo_col > 0) put_half8(out + o + g.lo_col, lo, vec);
      if (out2 != nullptr) put_half8(out2 + o, gv[t], vec);
      if (out3 != nullptr) put_half8(out3 + o, uv[t], vec);
    }
  }
}

template <int BN, int EPI, int BL = BL_K>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_b2, const GemmArgs g) {
  using S = GemmSmem<BN>;
  static_assert(BL != BL_MN2 || (BN == 128 && EPI == EPI_SWIGLU2), "gate|up tiles are 64 + 64 columns");
  static_assert(EPI != EPI_SWIGLU2 || BL == BL_MN2, "EPI_SWIGLU2 needs the gate|up B layout");
  const int STAGES = g.stages;
  const uint32_t stage_tx = static_cast<uint32_t>(g.a_box * BK * 2 + S::B_BYTES);  // bytes landing per stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(base + STAGES * S::STAGE);
  uint64_t *empty = full + S::MAX_STAGES;
  uint64_t *acc_full = empty + S::MAX_STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile uint32_t *abort = tmem_slot + 1;
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Split-K reduced in the cluster (launched with cluster dims (1, 1, k_splits)).
  constexpr bool CAN_CLUSTER = EPI == EPI_F16 || EPI == EPI_F32 || EPI == EPI_F32_RES16 ||
                               EPI == EPI_F16_RES32 || EPI == EPI_SWIGLU;
  const bool clustered = CAN_CLUSTER && g.cluster_k != 0 && gridDim.z > 1;
  constexpr int TPITCH = BN + 4;  // fp32 partial tile row pitch (16-byte shift per row)
  const int nk_all = (g.K + BK - 1) / BK;
  // Split-K slice of this CTA (a single slice unless EPI_PARTIAL).
  const int kb0 = static_cast<int>((static_cast<long long>(nk_all) * blockIdx.z) / gridDim.z);
  const int nk = static_cast<int>((static_cast<long long>(nk_all) * (blockIdx.z + 1)) / gridDim.z) - kb0;
  // Row tiles on grid.x (m_fast) when B does not stay in L2: the row tiles
  // of a column tile then run together and B streams from DRAM once.
  const int tile_m = g.m_fast ? blockIdx.x : blockIdx.y, tile_n = g.m_fast ? blockIdx.y : blockIdx.x;
  const int m0 = tile_m * BM, n0 = tile_n * BN;
  // B tile of k-block kb into dst (one k-block: BK rows of K).  MN-major:
  // boxes of 64 columns x BK rows, each BK * 128 bytes; BL_MN2 takes the
  // gate and the up columns [n0 / 2, n0 / 2 + 64) of the two matrices.
  auto load_b = [&](uint8_t *dst, int kb, uint64_t *bar) {
    if (g.b_kwrap > 0) kb %= g.b_kwrap;
    if constexpr (BL == BL_K) {
      tma_load_2d(dst, &tm_b, kb * BK, n0, bar);
    } else if constexpr (BL == BL_MN) {
#pragma unroll
      for (int j = 0; j < BN / 64; ++j) tma_load_2d(dst + j * BK * 128, &tm_b, n0 + 64 * j, kb * BK, bar);
    } else {
      tma_load_2d(dst, &tm_b, n0 / 2, kb * BK, bar);
      tma_load_2d(dst + BK * 128, &tm_b2, n0 / 2, kb * BK, bar);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort = 0;
    qb200::fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The next kernel of the stream may be scheduled now; it waits for this
  // grid before it reads anything this grid writes.
  if (threadIdx.x == 0) qb200::griddep_launch_dependents();

  // The producer and MMA warps run their loops as whole warps (every lane
  // waits on the barriers) and one lane issues; the MMAs go out predicated
  // on an elected lane, which keeps the warp converged around them (a branch
  // to a single lane around each k-block's MMAs costs ~60 % more issue time).
  if (warp == 0) {
    // B (weights) does not depend on the preceding kernel: the first ring
    // stages are armed and their weight tiles requested before the grid
    // dependency wait; A (activations) follows it.
    const int pre = min(STAGES, nk);
    if (lane == 0) {
      for (int kb = 0; kb < pre; ++kb) {
        uint8_t *st = base + kb * S::STAGE;
        mbar_arrive_expect_tx(&full[kb], stage_tx);
        load_b(st + S::A_BYTES, kb0 + kb, &full[kb]);
      }
      qb200::griddep_wait();
      for (int kb = 0; kb < pre; ++kb)
        tma_load_2d(base + kb * S::STAGE, &tm_a, (kb0 + kb) * BK, m0, &full[kb]);
    }
    __syncwarp();
    int issued = pre;
    for (int kb = pre; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!gemm_wait(&empty[s], ((kb / STAGES) - 1) & 1, abort, g.err, 1)) break;
      if (lane == 0) {
        uint8_t *st = base + s * S::STAGE;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_2d(st, &tm_a, (kb0 + kb) * BK, m0, &full[s]);
        load_b(st + S::A_BYTES, kb0 + kb, &full[s]);
      }
      __syncwarp();
      issued = kb + 1;
    }
    // Every issued copy lands before the CTA may exit (matters after an abort).
    for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[kb % STAGES], (kb / STAGES) & 1))
        if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
          if (lane == 0) gemm_record(g.err, 4);
          break;
        }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f16<BN>(BL != BL_K);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!gemm_wait(&full[s], (kb / STAGES) & 1, abort, g.err, 2)) break;
      tc_fence_after();
      const uint32_t sa = smem_u32(base + s * S::STAGE);
      const uint32_t sb = sa + S::A_BYTES;
      // K-major operands advance 16 elements (32 bytes) along their rows per
      // MMA; an MN-major B advances 16 rows (two 1024-byte atoms).
      uint64_t bd[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) bd[k] = BL == BL_K ? sw128_desc(sb + 32 * k) : sw128_mn_desc(sb + 2048 * k, BK * 128);
      mma4_commit_elect(tmem, sw128_desc(sa), sw128_desc(sa + 32), sw128_desc(sa + 64), sw128_desc(sa + 96), bd[0],
                        bd[1], bd[2], bd[3], idesc, kb != 0 ? 1u : 0u, smem_u32(&empty[s]));
    }
    // Signals the accumulator once every MMA issued above has completed
    // (also after an abort, so tensor memory is never freed under an MMA).
    if (lane == 0) mma_commit(acc_full);
    __syncwarp();
  } else {
    // Epilogue warps 2..5: TMEM lane quadrant = warp % 4.  Residuals and the
    // output buffers belong to earlier kernels until the dependency wait.
    qb200::griddep_wait();
    const int q = warp & 3;
    bool ok = gemm_wait(acc_full, 0, abort, g.err, 3);
    ok = __all_sync(0xffffffffu, ok && !*abort);  // tcgen05.ld below is warp-collective
    tc_fence_after();
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16);
    if (ok && clustered) {
      // This k slice's partial tile into shared memory (the ring is idle:
      // every copy has landed and every MMA has completed).
      float *trow = reinterpret_cast<float *>(base) + (32 * q + lane) * TPITCH;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        float v[64];
        tmem_ld64(tq + c0, tq + c0 + 32, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          reinterpret_cast<float4 *>(trow + c0)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    } else if (ok && EPI == EPI_ARGMAX) {
      const int row = m0 + 32 * q + lane;
      float best = -INFINITY;
      int best_i = 0x7fffffff;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        const int col = n0 + c0;
        if (col >= g.N) break;  // warp-uniform
        float v[64];
        tmem_ld64(tq + c0, tq + c0 + 32, v);
        const int nvalid = min(64, g.N - col);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < nvalid && v[i] > best) {
            best = v[i];
            best_i = col + i;
          }
      }
      if (row < g.M) {
        g.part_val[static_cast<size_t>(row) * g.n_tiles + tile_n] = best;
        g.part_idx[static_cast<size_t>(row) * g.n_tiles + tile_n] = best_i;
      }
    } else if (ok && m0 + 32 * q < g.M) {  // (a warp whose 32 rows are all past M has nothing to do)
      // The ring is idle (every copy landed, every MMA completed): each warp
      // stages its 32 rows there, then stores them row-contiguously.
      float *stg = reinterpret_cast<float *>(base) + q * (32 * EPI_PITCH);
      if constexpr (EPI == EPI_SWIGLU2)
        epilogue_swiglu2<BN>(g, tq, stg, m0 + 32 * q, n0, lane);
      else
        epilogue_staged<BN, EPI>(g, tq, stg, m0 + 32 * q, n0, lane);
    }
  }
  // Lanes 1..31 of warps 0 and 1 skipped their roles' loops: they wait here
  // for lane 0, so that each warp reaches the CTA barrier converged (a barrier
  // counts whole warps, and tensor memory is freed only after it).
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (clustered) {
    // Split-K reduced inside the cluster: every rank adds the k slices'
    // partial tiles for its share of the tile's rows, in slice order (as the
    // separate reduction kernel adds its slices, so the bits are the same),
    // then applies the epilogue.  Every thread of every CTA takes both
    // cluster barriers, also after an abort.
    cluster_sync_all();
    const int Z = static_cast<int>(gridDim.z);
    const int rank = static_cast<int>(cluster_rank());
    const int rows_per = (BM + Z - 1) / Z;
    const int r0 = rank * rows_per, r1 = min(BM, r0 + rows_per);
    if (warp >= 2 && !*abort) {
      constexpr int C4 = BN / 4;
      const int t = threadIdx.x - 64;  // 0..127
      // Two entries per thread and step, every distributed-shared-memory load
      // of both issued before the first add (one round trip per step).
      const int count = (r1 - r0) * C4;
      for (int i0 = t; i0 < count; i0 += 256) {
        float4 pz[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int idx = i0 + 128 * u;
          if (idx >= count) continue;
          const int lrow = r0 + idx / C4, c = 4 * (idx % C4);
          const uint32_t trow = smem_u32(base) + static_cast<uint32_t>(lrow * TPITCH) * 4u;
#pragma unroll
          for (int z = 0; z < 8; ++z)
            if (z < Z) pz[u][z] = ld_dsmem_f4(map_rank(trow + c * 4, z));
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int idx = i0 + 128 * u;
          if (idx >= count) continue;
          const int lrow = r0 + idx / C4, c = 4 * (idx % C4);
          const int row = m0 + lrow, col = n0 + c;
          if (row >= g.M || col >= g.N) continue;
          float4 acc = pz[u][0];
#pragma unroll
          for (int z = 1; z < 8; ++z) {
            if (z < Z) {
              acc.x = __fadd_rn(acc.x, pz[u][z].x);
              acc.y = __fadd_rn(acc.y, pz[u][z].y);
              acc.z = __fadd_rn(acc.z, pz[u][z].z);
              acc.w = __fadd_rn(acc.w, pz[u][z].w);
            }
          }
          const size_t o = static_cast<size_t>(row) * g.ldo + col;
          if constexpr (EPI == EPI_F32_RES16) {
            const __half *r = static_cast<const __half *>(g.res) + o;
            *reinterpret_cast<float4 *>(static_cast<float *>(g.out) + o) =
                make_float4(__fadd_rn(acc.x, __half2float(r[0])), __fadd_rn(acc.y, __half2float(r[1])),
                            __fadd_rn(acc.z, __half2float(r[2])), __fadd_rn(acc.w, __half2float(r[3])));
          } else if constexpr (EPI == EPI_F16_RES32) {
            const float4 r = *reinterpret_cast<const float4 *>(static_cast<const float *>(g.res) + o);
            __half2 h[2] = {__floats2half2_rn(__fadd_rn(acc.x, r.x), __fadd_rn(acc.y, r.y)),
                            __floats2half2_rn(__fadd_rn(acc.z, r.z), __fadd_rn(acc.w, r.w))};
            *reinterpret_cast<uint2 *>(static_cast<__half *>(g.out) + o) = *reinterpret_cast<const uint2 *>(h);
          } else if constexpr (EPI == EPI_F32) {
            *reinterpret_cast<float4 *>(static_cast<float *>(g.out) + o) = acc;
          } else if constexpr (EPI == EPI_SWIGLU) {
            // Column pairs (gate, up) -> output column col / 2 (ldo counts outputs).
            __half *out = static_cast<__half *>(g.out) + static_cast<size_t>(row) * g.ldo + col / 2;
            __half2 h = __halves2half2(
                __float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(acc.x))), acc.y)),
                __float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(acc.z))), acc.w)));
            *reinterpret_cast<__half2 *>(out) = h;
          } else if constexpr (EPI == EPI_F16) {
            if (g.bias != nullptr) {
              const __half *b = static_cast<const __half *>(g.bias) + col;
              acc.x = __fadd_rn(acc.x, __half2float(b[0]));
              acc.y = __fadd_rn(acc.y, __half2float(b[1]));
              acc.z = __fadd_rn(acc.z, __half2float(b[2]));
              acc.w = __fadd_rn(acc.w, __half2float(b[3]));
            }
            __half2 h[2] = {__floats2half2_rn(acc.x, acc.y), __floats2half2_rn(acc.z, acc.w)};
            *reinterpret_cast<uint2 *>(static_cast<__half *>(g.out) + o) = *reinterpret_cast<const uint2 *>(h);
          }
        }
      }
    }
    cluster_sync_all();  // the other ranks' tiles are no longer read
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Persistent row argmax over C = A . B^T (the lm_head: B = the vocabulary
// rows, A = at most a few row tiles of hidden states).  One CTA per SM walks
// the tiles t = blockIdx.x, + gridDim.x, ... in row-tile-fastest order (tile
// t = column tile t / mt, row tile t % mt, so the row tiles of a column tile
// run at the same time and B streams from DRAM once).  The copy ring and the
// MMA issue continue from one tile into the next; the accumulator is double
// buffered in tensor memory (2 x BN columns), so a tile's argmax epilogue
// overlaps the next tile's mainloop and no tile waits for a last, mostly
// empty wave.  Against the one-tile-per-CTA grid (same row-tile order) on the
// full vocabulary: 0.075 against 0.081 ms at 64 rows, 0.115 against 0.114 at
// 256, 0.120 against 0.114 at one row -- the B stream, not the per-tile
// overhead, sets the pace.  Output: part_val / part_idx [M, n_tiles] as
// EPI_ARGMAX (largest value, lowest column of the tile).
template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_argmax_persistent(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                           const GemmArgs g) {
  using S = GemmSmem<BN>;
  const int STAGES = g.stages;
  const uint32_t stage_tx = static_cast<uint32_t>(g.a_box * BK * 2 + S::B_BYTES);  // bytes landing per stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(base + STAGES * S::STAGE);
  uint64_t *empty = full + S::MAX_STAGES;
  uint64_t *acc_full = empty + S::MAX_STAGES;  // [2]
  uint64_t *acc_empty = acc_full + 2;          // [2]
  uint64_t *mma_done = acc_empty + 2;          // every issued MMA has completed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  volatile uint32_t *abort = tmem_slot + 1;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(TMEM_COLS <= 512, "two accumulators must fit tensor memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (g.M + BM - 1) / BM, ntl = (g.N + BN - 1) / BN;
  const int tiles = mt * ntl, nk = g.K / BK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    qb200::fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) qb200::griddep_launch_dependents();

  if (warp == 0) {
    // Producer: k-block c (counted over this CTA's tiles) goes to stage
    // c % STAGES; the first pass over the ring finds every stage free.
    qb200::griddep_wait();
    long long c = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const int m0 = (t % mt) * BM, n0 = (t / mt) * BN;
      for (int kb = 0; kb < nk; ++kb, ++c) {
        const int s = static_cast<int>(c % STAGES);
        if (!gemm_wait(&empty[s], static_cast<uint32_t>((c / STAGES) & 1) ^ 1u, abort, g.err, 1)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t *st = base + s * S::STAGE;
          mbar_arrive_expect_tx(&full[s], stage_tx);
          tma_load_2d(st, &tm_a, kb * BK, m0, &full[s]);
          tma_load_2d(st + S::A_BYTES, &tm_b, kb * BK, n0, &full[s]);
        }
        __syncwarp();
      }
    }
    // Every issued copy lands before the CTA may exit.
    for (long long d = (c > STAGES ? c - STAGES : 0); d < c; ++d) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[d % STAGES], static_cast<uint32_t>((d / STAGES) & 1)))
        if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
          if (lane == 0) gemm_record(g.err, 4);
          break;
        }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f16<BN>(false);
    long long c = 0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
      const int b = it & 1;
      // The epilogue has read this accumulator's previous tile.
      if (!gemm_wait(&acc_empty[b], static_cast<uint32_t>((it >> 1) & 1) ^ 1u, abort, g.err, 5)) break;
      tc_fence_after();
      const uint32_t acc = tmem + static_cast<uint32_t>(b * BN);
      for (int kb = 0; kb < nk; ++kb, ++c) {
        const int s = static_cast<int>(c % STAGES);
        if (!gemm_wait(&full[s], static_cast<uint32_t>((c / STAGES) & 1), abort, g.err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(base + s * S::STAGE), sb = sa + S::A_BYTES;
        mma4_commit_elect(acc, sw128_desc(sa), sw128_desc(sa + 32), sw128_desc(sa + 64), sw128_desc(sa + 96),
                          sw128_desc(sb), sw128_desc(sb + 32), sw128_desc(sb + 64), sw128_desc(sb + 96), idesc,
                          kb != 0 ? 1u : 0u, smem_u32(&empty[s]));
      }
      if (lane == 0) mma_commit(&acc_full[b]);  // this tile's MMAs have completed
      __syncwarp();
    }
    // Tensor memory is freed only after every issued MMA has completed (also
    // after an abort); the wait is bounded.
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(mma_done, 0))
      if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
        if (lane == 0) gemm_record(g.err, 6);
        break;
      }
  } else {
    // Epilogue warps 2..5: TMEM lane quadrant = warp % 4.
    qb200::griddep_wait();
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const int b = it & 1, m0 = (t % mt) * BM, tile_n = t / mt, n0 = tile_n * BN;
      bool ok = gemm_wait(&acc_full[b], static_cast<uint32_t>((it >> 1) & 1), abort, g.err, 3);
      ok = __all_sync(0xffffffffu, ok && !*abort);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(b * BN);
      const int row = m0 + 32 * q + lane;
      float best = -INFINITY;
      int best_i = 0x7fffffff;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        const int col = n0 + c0;
        if (col >= g.N) break;  // warp-uniform
        float v[64];
        tmem_ld64(tq + c0, tq + c0 + 32, v);
        const int nvalid = min(64, g.N - col);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < nvalid && v[i] > best) {
            best = v[i];
            best_i = col + i;
          }
      }
      // The accumulator is free for the tile after next.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) qb200::mbar_arrive(&acc_empty[b]);
      if (row < g.M) {
        g.part_val[static_cast<size_t>(row) * g.n_tiles + tile_n] = best;
        g.part_idx[static_cast<size_t>(row) * g.n_tiles + tile_n] = best_i;
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace qb200tc
