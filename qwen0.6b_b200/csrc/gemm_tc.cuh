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
};

template <int BN>
struct GemmSmem {
  static constexpr int MAX_STAGES = max_stages<BN>();
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr size_t bytes(int stages) { return static_cast<size_t>(stages) * STAGE + 256 + 1024; }
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

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
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

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
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

template <int BN, int EPI, int BL = BL_K>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_b2, const GemmArgs g) {
  using S = GemmSmem<BN>;
  static_assert(BL != BL_MN2 || (BN == 128 && EPI == EPI_SWIGLU2), "gate|up tiles are 64 + 64 columns");
  static_assert(EPI != EPI_SWIGLU2 || BL == BL_MN2, "EPI_SWIGLU2 needs the gate|up B layout");
  const int STAGES = g.stages;
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
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
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

  if (warp == 0) {
    if (lane == 0) {
      // B (weights) does not depend on the preceding kernel: the first ring
      // stages are armed and their weight tiles requested before the grid
      // dependency wait; A (activations) follows it.
      const int pre = min(STAGES, nk);
      for (int kb = 0; kb < pre; ++kb) {
        uint8_t *st = base + kb * S::STAGE;
        mbar_arrive_expect_tx(&full[kb], S::STAGE);
        load_b(st + S::A_BYTES, kb0 + kb, &full[kb]);
      }
      qb200::griddep_wait();
      for (int kb = 0; kb < pre; ++kb)
        tma_load_2d(base + kb * S::STAGE, &tm_a, (kb0 + kb) * BK, m0, &full[kb]);
      int issued = pre;
      for (int kb = pre; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (!gemm_wait(&empty[s], ((kb / STAGES) - 1) & 1, abort, g.err, 1)) break;
        uint8_t *st = base + s * S::STAGE;
        mbar_arrive_expect_tx(&full[s], S::STAGE);
        tma_load_2d(st, &tm_a, (kb0 + kb) * BK, m0, &full[s]);
        load_b(st + S::A_BYTES, kb0 + kb, &full[s]);
        issued = kb + 1;
      }
      // Every issued copy lands before the CTA may exit (matters after an abort).
      for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[kb % STAGES], (kb / STAGES) & 1))
          if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
            gemm_record(g.err, 4);
            break;
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16<BN>(BL != BL_K);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (!gemm_wait(&full[s], (kb / STAGES) & 1, abort, g.err, 2)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(base + s * S::STAGE);
        const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          // K-major B advances 16 elements (32 bytes) along its rows; MN-major
          // B advances 16 rows (two 1024-byte atoms).
          const uint64_t bd = BL == BL_K ? sw128_desc(sb + 32 * k) : sw128_mn_desc(sb + 2048 * k, BK * 128);
          mma_f16(tmem, sw128_desc(sa + 32 * k), bd, idesc, (kb | k) != 0 ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      // Signals the accumulator once every MMA issued above has completed
      // (also after an abort, so tensor memory is never freed under an MMA).
      mma_commit(acc_full);
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quadrant = warp % 4.  Residuals and the
    // output buffers belong to earlier kernels until the dependency wait.
    qb200::griddep_wait();
    const int q = warp & 3;
    const int row = m0 + 32 * q + lane;
    bool ok = gemm_wait(acc_full, 0, abort, g.err, 3);
    ok = __all_sync(0xffffffffu, ok && !*abort);  // tcgen05.ld below is warp-collective
    tc_fence_after();
    if (ok && clustered) {
      // This k slice's partial tile into shared memory (the ring is idle:
      // every copy has landed and every MMA has completed).
      const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16);
      float *trow = reinterpret_cast<float *>(base) + (32 * q + lane) * TPITCH;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tq + c0, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<float4 *>(trow + c0)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    } else if (ok && EPI == EPI_SWIGLU2) {
      // Columns c of the gate half and c + BN/2 of the up half are output
      // column n0 / 2 + c.
      const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16);
      const int nout = g.N / 2;
#pragma unroll 1
      for (int c0 = 0; c0 < BN / 2; c0 += 16) {
        float gv[16], uv[16];
        tmem_ld16(tq + c0, gv);
        tmem_ld16(tq + BN / 2 + c0, uv);
        const int col = n0 / 2 + c0;
        if (row >= g.M || col >= nout) continue;
        const int nvalid = min(16, nout - col);
        const size_t o = static_cast<size_t>(row) * g.ldo + col;
        __half *out = static_cast<__half *>(g.out) + o;
        // Eight packed pairs per output (s hi, s lo, gate, up), stored as two
        // 16-byte stores each when the 16 columns are whole and aligned (the
        // planned shapes), else element by element.
        uint32_t ph[8], pl[8], pg[8], pu[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float sv[2], gg[2], uu[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const bool in = i + j < nvalid;
            gg[j] = (g.bias != nullptr && in) ? __fadd_rn(gv[i + j], __half2float(static_cast<const __half *>(g.bias)[col + i + j])) : gv[i + j];
            uu[j] = (g.bias2 != nullptr && in) ? __fadd_rn(uv[i + j], __half2float(static_cast<const __half *>(g.bias2)[col + i + j])) : uv[i + j];
            sv[j] = __fmul_rn(__fdiv_rn(gg[j], __fadd_rn(1.0f, expf(-gg[j]))), uu[j]);
          }
          const __half2 hi = __floats2half2_rn(sv[0], sv[1]);
          const __half2 lo = __floats2half2_rn(__fsub_rn(sv[0], __low2float(hi)), __fsub_rn(sv[1], __high2float(hi)));
          const __half2 gh = __floats2half2_rn(gg[0], gg[1]);
          const __half2 uh = __floats2half2_rn(uu[0], uu[1]);
          ph[i / 2] = *reinterpret_cast<const uint32_t *>(&hi);
          pl[i / 2] = *reinterpret_cast<const uint32_t *>(&lo);
          pg[i / 2] = *reinterpret_cast<const uint32_t *>(&gh);
          pu[i / 2] = *reinterpret_cast<const uint32_t *>(&uh);
        }
        auto put = [&](__half *dst, const uint32_t (&p)[8]) {
          if (nvalid == 16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            reinterpret_cast<uint4 *>(dst)[0] = make_uint4(p[0], p[1], p[2], p[3]);
            reinterpret_cast<uint4 *>(dst)[1] = make_uint4(p[4], p[5], p[6], p[7]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < nvalid) dst[i] = __ushort_as_half(static_cast<unsigned short>(p[i / 2] >> (16 * (i & 1))));
          }
        };
        put(out, ph);
        if (g.lo_col > 0) put(out + g.lo_col, pl);
        if (g.out2 != nullptr) put(static_cast<__half *>(g.out2) + o, pg);
        if (g.out3 != nullptr) put(static_cast<__half *>(g.out3) + o, pu);
      }
    } else if (ok) {
      const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16);
      float best = -INFINITY;
      int best_i = 0x7fffffff;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tq + c0, v);
        const int col = n0 + c0;
        if (row >= g.M || col >= g.N) continue;
        const size_t o = static_cast<size_t>(row) * g.ldo + col;
        const int nvalid = min(16, g.N - col);
        if constexpr (EPI == EPI_F16) {
          __half *out = static_cast<__half *>(g.out) + o;
          if (g.bias != nullptr) {
            const __half *b = static_cast<const __half *>(g.bias) + col;
            for (int i = 0; i < nvalid; ++i) v[i] = __fadd_rn(v[i], __half2float(b[i]));
          }
          if (nvalid == 16) {
            uint4 pk[2];
            __half2 *h = reinterpret_cast<__half2 *>(pk);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            reinterpret_cast<uint4 *>(out)[0] = pk[0];
            reinterpret_cast<uint4 *>(out)[1] = pk[1];
          } else {
            for (int i = 0; i < nvalid; ++i) out[i] = __float2half_rn(v[i]);
          }
        } else if constexpr (EPI == EPI_PARTIAL) {
          float *out = static_cast<float *>(g.out) +
                       static_cast<size_t>(blockIdx.z) * g.M * g.ldo + o;
          if (nvalid == 16) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<float4 *>(out)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            for (int i = 0; i < nvalid; ++i) out[i] = v[i];
          }
        } else if constexpr (EPI == EPI_F32 || EPI == EPI_F32_RES16) {
          float *out = static_cast<float *>(g.out) + o;
          for (int i = 0; i < nvalid; ++i) {
            float x = v[i];
            if constexpr (EPI == EPI_F32_RES16)
              x = __fadd_rn(x, __half2float(static_cast<const __half *>(g.res)[o + i]));
            out[i] = x;
          }
        } else if constexpr (EPI == EPI_F16_RES32) {
          __half *out = static_cast<__half *>(g.out) + o;
          const float *res = static_cast<const float *>(g.res) + o;
          for (int i = 0; i < nvalid; ++i) out[i] = __float2half_rn(__fadd_rn(v[i], res[i]));
        } else if constexpr (EPI == EPI_SWIGLU) {
          // ldo counts output columns (inter); column pair (2i, 2i+1) -> output i.
          __half *out = static_cast<__half *>(g.out) + static_cast<size_t>(row) * g.ldo + col / 2;
          __align__(16) __half act[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            act[i] = __float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(v[2 * i]))), v[2 * i + 1]));
          if (nvalid == 16 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
            *reinterpret_cast<uint4 *>(out) = *reinterpret_cast<const uint4 *>(act);
          } else {
            for (int i = 0; i + 1 < nvalid; i += 2) out[i / 2] = act[i / 2];
          }
        } else if constexpr (EPI == EPI_ARGMAX) {
          for (int i = 0; i < nvalid; ++i)
            if (v[i] > best) {
              best = v[i];
              best_i = col + i;
            }
        }
      }
      if constexpr (EPI == EPI_ARGMAX) {
        if (row < g.M) {
          g.part_val[static_cast<size_t>(row) * g.n_tiles + blockIdx.x] = best;
          g.part_idx[static_cast<size_t>(row) * g.n_tiles + blockIdx.x] = best_i;
        }
      }
    }
  }
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
      for (int idx = t; idx < (r1 - r0) * C4; idx += 128) {
        const int lrow = r0 + idx / C4, c = 4 * (idx % C4);
        const int row = m0 + lrow, col = n0 + c;
        if (row >= g.M || col >= g.N) continue;
        const uint32_t trow = smem_u32(base) + static_cast<uint32_t>(lrow * TPITCH) * 4u;
        float4 pz[8];
#pragma unroll
        for (int z = 0; z < 8; ++z)
          if (z < Z) pz[z] = ld_dsmem_f4(map_rank(trow + c * 4, z));
        float4 acc = pz[0];
#pragma unroll
        for (int z = 1; z < 8; ++z) {
          if (z < Z) {
            acc.x = __fadd_rn(acc.x, pz[z].x);
            acc.y = __fadd_rn(acc.y, pz[z].y);
            acc.z = __fadd_rn(acc.z, pz[z].z);
            acc.w = __fadd_rn(acc.w, pz[z].w);
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
    cluster_sync_all();  // the other ranks' tiles are no longer read
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace qb200tc
