// ops.cu - standalone RMSNorm and SwiGLU operators for B200 (sm_100a): the
// replacements of the upstream Tools/rmsnorm and Tools/swiglu extensions, with
// the C ABI of include/qwen_b200_ops.h.
//
// RMSNorm (rmsnorm.cuh:17-176): one warp per row, 16-byte loads, fp32 sum of
// squares, the upstream rounding points.  Memory-bound and tiny.
//
// SwiGLU (swiglu.cu:89-130, :267-310): upstream accumulates in c10::Half, so
// every product and every partial sum is rounded to fp16 in ascending index
// order.  That makes each output a serial chain over the reduction index that
// cannot be reassociated, split or put on tensor cores without changing the
// result.  The B200 design keeps the chain exact and restructures everything
// around it:
//  * one "chain GEMM" kernel, C[r, n] = init[n] (+)= A[r, k] (*) B[k, n] with
//    fp16-rounded (*) and (+), k ascending; used for gate/up (two B matrices
//    sharing the A loads, SiLU epilogue) and for down;
//  * the SwiGLU activations are computed once per row and reused by every
//    down-projection output (upstream recomputes them per output element,
//    O(rows * hidden^2 * inter));
//  * A and B tiles are streamed through a 4-stage shared-memory ring by TMA
//    tensor copies (one producer lane, mbarrier completion, no multicast), so
//    weight bytes stay in flight while the chains run;
//  * each thread carries one half2 chain (two adjacent output columns; in the
//    gate/up kernel the gate and up chains of a column pair sit on partner
//    lanes and meet by a shuffle), using the non-contracting __hmul2_rn /
//    __hadd2_rn so products are never fused into an FMA; per 8 steps the
//    loads and products are issued first and only the adds form the chain;
//  * each kernel is a programmatic dependent of the previous one: it requests
//    its first weight tiles before waiting for the kernel whose output it reads.
// The chain latency (reduction length x dependent fp16 add latency) bounds a
// small-batch call; the fp16 ALU issue rate bounds a large-batch one.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "gemm_tc_host.h"
#include "host_err.h"
#include "launch.h"
#include "ptx.cuh"
#include "qwen_b200_ops.h"

namespace qb200ops {

using qb200::fence_mbar_init;
using qb200::globaltimer_ns;
using qb200::mbar_arrive;
using qb200::mbar_arrive_expect_tx;
using qb200::mbar_init;
using qb200::mbar_try_wait;
using qb200::smem_u32;

constexpr int RB = 16;                  // rows per tile
constexpr int CB = 16;                  // output columns per tile
constexpr int KC = 128;                 // reduction chunk per ring stage
constexpr int NST = 4;                  // ring stages
// Consumer threads: RB rows x CB/2 column pairs, each thread one half2 chain
// (two adjacent output columns).  In the DUAL (gate/up) kernel SPLIT puts the
// gate and up chains of a column pair on two partner threads (shortest chain
// per thread: the latency-bound small-row case); without SPLIT one thread
// carries both (fewer instructions: the issue-bound many-row case).  + one
// producer warp.
template <bool DUAL, bool SPLIT>
constexpr int cons_threads() {
  return RB * (CB / 2) * (DUAL && SPLIT ? 2 : 1);
}
template <bool DUAL, bool SPLIT>
constexpr int chain_threads() {
  return cons_threads<DUAL, SPLIT>() + 32;
}
constexpr int A_BYTES = RB * KC * 2;    // TMA box {KC, RB} of A [rows, K]
constexpr int B_BYTES = KC * CB * 2;    // TMA box {CB, KC} of B [K, N]
constexpr int MAX_ROW_TILES = 65535;
constexpr long long WAIT_NS = 2000000000LL;

constexpr uint32_t ERR_FULL_WAIT = 1, ERR_EMPTY_WAIT = 2, ERR_DRAIN_WAIT = 3;

// Status word of the operator kernels: (code << 32) | (blockIdx.y << 16) | blockIdx.x
// of the first bounded wait that gave up.
__device__ unsigned long long g_ops_err = 0;

struct ChainArgs {
  const __half *init0;  // [N] start values of chain 0 (bias) or nullptr (+0)
  const __half *init1;  // [N] start values of chain 1 (DUAL) or nullptr
  __half *out;          // [rows, N]
  __half *cache0;       // DUAL: [rows, N] final chain-0 values (gate) or nullptr
  __half *cache1;       // DUAL: [rows, N] final chain-1 values (up) or nullptr
  int rows, K, N;
};

template <bool DUAL>
constexpr int stage_bytes() {
  return A_BYTES + B_BYTES * (DUAL ? 2 : 1);
}

template <bool DUAL>
constexpr size_t chain_smem_bytes() {
  return static_cast<size_t>(NST) * stage_bytes<DUAL>() + 2 * NST * sizeof(uint64_t) + 16 + 1024;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __noinline__ void record_error(uint32_t code) {
  const unsigned long long v = (static_cast<unsigned long long>(code) << 32) |
                               (static_cast<unsigned long long>(blockIdx.y & 0xffffu) << 16) |
                               (blockIdx.x & 0xffffu);
  atomicCAS(&g_ops_err, 0ull, v);
}

// Bounded mbarrier wait: gives up after WAIT_NS or when the CTA's abort flag
// is set; the first thread to give up records the error and sets the flag.
__device__ __noinline__ bool wait_bar_slow(uint64_t *bar, uint32_t parity,
                                           volatile uint32_t *abort, uint32_t code) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
      *abort = 1;
      record_error(code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile uint32_t *abort,
                                         uint32_t code) {
  return mbar_try_wait(bar, parity) || wait_bar_slow(bar, parity, abort, code);
}

// c10::Half SiLU as upstream instantiates it (swiglu.cu:60-63): the Half
// operand is widened, x / (1 + expf(-x)) evaluated in fp32, rounded on return.
__device__ __forceinline__ __half silu_c10(__half x) {
  const float xf = __half2float(x);
  return __float2half_rn(xf / (1.0f + expf(-xf)));
}

// grid (ceil(N / CB), ceil(rows / RB)), chain_threads<DUAL, SPLIT>() threads,
// chain_smem_bytes<DUAL>().
template <bool DUAL, bool SPLIT>
__global__ void __launch_bounds__(chain_threads<DUAL, SPLIT>())
    chain_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b0,
                      const __grid_constant__ CUtensorMap tm_b1, const ChainArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Offset the array itself (not an integer copy of its address), so that
  // the compiler keeps every access in the shared address space (LDS/STS,
  // not generic loads).
  uint8_t *base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int SB = stage_bytes<DUAL>();
  uint64_t *full = reinterpret_cast<uint64_t *>(base + NST * SB);
  uint64_t *empty = full + NST;
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(empty + NST);

  constexpr int CONS = cons_threads<DUAL, SPLIT>();
  const int tid = threadIdx.x;
  const int nchunks = (p.K + KC - 1) / KC;
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONS / 32);
    }
    *abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) qb200::griddep_launch_dependents();

  if (tid >= CONS) {
    // Producer: one lane streams A and B chunks into the ring.  The weights
    // (B) of the first stages are requested before waiting for the previous
    // kernel of the stream, whose output A may be.
    if (tid != CONS) return;
    const int pre = min(NST, nchunks);
    for (int c = 0; c < pre; ++c) {
      uint8_t *st = base + c * SB;
      mbar_arrive_expect_tx(&full[c], SB);
      tma_load_2d(st + A_BYTES, &tm_b0, blockIdx.x * CB, c * KC, &full[c]);
      if constexpr (DUAL) tma_load_2d(st + A_BYTES + B_BYTES, &tm_b1, blockIdx.x * CB, c * KC, &full[c]);
    }
    qb200::griddep_wait();
    for (int c = 0; c < pre; ++c) tma_load_2d(base + c * SB, &tm_a, c * KC, blockIdx.y * RB, &full[c]);
    int issued = pre;
    for (int c = pre; c < nchunks; ++c) {
      const int s = c % NST;
      if (!wait_bar(&empty[s], ((c / NST) - 1) & 1, abort, ERR_EMPTY_WAIT)) break;
      uint8_t *st = base + s * SB;
      mbar_arrive_expect_tx(&full[s], SB);
      tma_load_2d(st, &tm_a, c * KC, blockIdx.y * RB, &full[s]);
      tma_load_2d(st + A_BYTES, &tm_b0, blockIdx.x * CB, c * KC, &full[s]);
      if constexpr (DUAL) tma_load_2d(st + A_BYTES + B_BYTES, &tm_b1, blockIdx.x * CB, c * KC, &full[s]);
      issued = c + 1;
    }
    // Let every issued copy land before the CTA can exit.
    for (int c = (issued > NST ? issued - NST : 0); c < issued; ++c) {
      const int s = c % NST;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[s], (c / NST) & 1)) {
        if (static_cast<long long>(globaltimer_ns() - t0) > WAIT_NS) {
          record_error(ERR_DRAIN_WAIT);
          break;
        }
      }
    }
    return;
  }

  // Consumers: thread = (row in tile, chain m, column pair); m selects gate
  // (0) or up (1) in the DUAL kernel.  Outputs and biases belong to earlier
  // kernels until the dependency wait.
  qb200::griddep_wait();
  const int lane = tid & 31;
  const int cp = tid & 7;
  constexpr bool TWO = DUAL && !SPLIT;            // both chains on this thread
  const int m = DUAL && SPLIT ? (tid >> 3) & 1 : 0;
  const int rl = DUAL && SPLIT ? tid >> 4 : tid >> 3;
  const int r = blockIdx.y * RB + rl;
  const int n = blockIdx.x * CB + 2 * cp;
  const bool active = r < p.rows && n < p.N;  // N is even, so n + 1 < N too
  const __half2 zero = __float2half2_rn(0.0f);
  const __half *init = m == 0 ? p.init0 : p.init1;
  __half2 acc = (init != nullptr && n < p.N) ? *reinterpret_cast<const __half2 *>(init + n) : zero;
  __half2 acc_up = zero;  // TWO: the up chain
  if (TWO && p.init1 != nullptr && n < p.N) acc_up = *reinterpret_cast<const __half2 *>(p.init1 + n);
  for (int c = 0; c < nchunks; ++c) {
    const int s = c % NST;
    // A warp leaves together (the final shuffle needs every lane).
    if (!__all_sync(0xffffffffu, wait_bar(&full[s], (c / NST) & 1, abort, ERR_FULL_WAIT))) return;
    const int kn = min(KC, p.K - c * KC);  // a multiple of 8
    if (active) {
      const uint8_t *st = base + s * SB;
      const __half *arow = reinterpret_cast<const __half *>(st) + rl * KC;
      const __half2 *bm = reinterpret_cast<const __half2 *>(st + A_BYTES + m * B_BYTES) + cp;
      const __half2 *bu = reinterpret_cast<const __half2 *>(st + A_BYTES + B_BYTES) + cp;
#pragma unroll 2
      for (int k = 0; k < kn; k += 8) {
        // Loads and products of 8 steps first, then the dependent fp16 adds
        // in ascending k: only the adds form the serial chain.
        const uint4 av = *reinterpret_cast<const uint4 *>(arow + k);
        const __half *ah = reinterpret_cast<const __half *>(&av);
        __half2 pr[8], pu[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const __half2 x2 = __half2half2(ah[j]);
          pr[j] = __hmul2_rn(x2, bm[(k + j) * (CB / 2)]);
          if constexpr (TWO) pu[j] = __hmul2_rn(x2, bu[(k + j) * (CB / 2)]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc = __hadd2_rn(acc, pr[j]);
          if constexpr (TWO) acc_up = __hadd2_rn(acc_up, pu[j]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  const size_t o = static_cast<size_t>(r) * p.N + n;
  if constexpr (DUAL) {
    __half2 up = acc_up;
    if constexpr (SPLIT) {
      // The up chain of this (row, column pair) is lane ^ 8 of the same warp.
      uint32_t mine = *reinterpret_cast<uint32_t *>(&acc);
      const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 8);
      up = *reinterpret_cast<const __half2 *>(&other);
    }
    if (!active) return;
    if (m == 0) {
      const __half g0 = __low2half(acc), g1 = __high2half(acc);
      const __half u0 = __low2half(up), u1 = __high2half(up);
      *reinterpret_cast<__half2 *>(p.out + o) =
          __halves2half2(__hmul_rn(silu_c10(g0), u0), __hmul_rn(silu_c10(g1), u1));
      if (p.cache0 != nullptr) *reinterpret_cast<__half2 *>(p.cache0 + o) = acc;
      if (TWO && p.cache1 != nullptr) *reinterpret_cast<__half2 *>(p.cache1 + o) = up;
    } else if (p.cache1 != nullptr) {
      *reinterpret_cast<__half2 *>(p.cache1 + o) = acc;
    }
  } else {
    if (!active) return;
    *reinterpret_cast<__half2 *>(p.out + o) = acc;
  }
}

// RMSNorm, one warp per row (blockDim / 32 rows per CTA).  With `res`, the
// fused form: res = half(x + res) written back, then normalise res.
// Elements below (cols / 4) * 4 follow upstream's vector path, the rest its
// scalar remainder path (rmsnorm.cuh:47-76, :95-108), whose rounding differs.
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(__half *__restrict__ out, float *__restrict__ rms,
                   const __half *__restrict__ x, const __half *__restrict__ w,
                   __half *__restrict__ res, long long rows, int cols, float eps) {
  qb200::griddep_wait();
  qb200::griddep_launch_dependents();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __half *xr = x + row * cols;
  __half *rr = res != nullptr ? res + row * cols : nullptr;
  __half *orow = out + row * cols;
  float ss = 0.0f;
  if ((cols & 7) == 0) {
    const int nv = cols >> 3;
    for (int i = lane; i < nv; i += 32) {
      uint4 v = reinterpret_cast<const uint4 *>(xr)[i];
      __half2 *h = reinterpret_cast<__half2 *>(&v);
      if (rr != nullptr) {
        uint4 rv = reinterpret_cast<const uint4 *>(rr)[i];
        const __half2 *hr = reinterpret_cast<const __half2 *>(&rv);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __hadd2_rn(h[j], hr[j]);
        reinterpret_cast<uint4 *>(rr)[i] = v;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  } else {
    const int vec_end = (cols >> 2) << 2;
    for (int i = lane; i < cols; i += 32) {
      float v;
      if (rr != nullptr) {
        const float sum = __half2float(xr[i]) + __half2float(rr[i]);
        rr[i] = __float2half_rn(sum);
        v = i < vec_end ? __half2float(rr[i]) : sum;
      } else {
        v = __half2float(xr[i]);
      }
      ss = fmaf(v, v, ss);
    }
  }
  ss = qb200::warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
  if (lane == 0) rms[row] = 1.0f / inv;
  const __half *src = rr != nullptr ? rr : xr;
  if ((cols & 7) == 0) {
    const int nv = cols >> 3;
    for (int i = lane; i < nv; i += 32) {
      uint4 v = reinterpret_cast<const uint4 *>(src)[i];
      const uint4 wv = reinterpret_cast<const uint4 *>(w)[i];
      __half2 *h = reinterpret_cast<__half2 *>(&v);
      const __half2 *hw = reinterpret_cast<const __half2 *>(&wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        const float2 g = __half22float2(hw[j]);
        if (rr != nullptr)
          h[j] = __floats2half2_rn(__fmul_rn(f.x, __fmul_rn(inv, g.x)), __fmul_rn(f.y, __fmul_rn(inv, g.y)));
        else
          h[j] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, inv), g.x), __fmul_rn(__fmul_rn(f.y, inv), g.y));
      }
      reinterpret_cast<uint4 *>(orow)[i] = v;
    }
  } else {
    const int vec_end = (cols >> 2) << 2;
    for (int i = lane; i < cols; i += 32) {
      const float f = __half2float(src[i]);
      const float g = __half2float(w[i]);
      const bool vec_form = rr != nullptr && i < vec_end;
      orow[i] = __float2half_rn(vec_form ? __fmul_rn(f, __fmul_rn(inv, g)) : __fmul_rn(__fmul_rn(f, inv), g));
    }
  }
}

}  // namespace qb200ops

// ====================================================================== host
using namespace qb200ops;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_ops_mu;
EncodeTiledFn g_encode = nullptr;
bool g_attr_set[64][2][2] = {};

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return qb200_set_error(code, buf);
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

EncodeTiledFn encoder() {
  std::lock_guard<std::mutex> lk(g_ops_mu);
  if (g_encode == nullptr) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  return g_encode;
}

int make_map(CUtensorMap *m, const void *ptr, long long inner, long long outer, int box_inner,
             int box_outer) {
  return qb200_encode_f16_2d(m, ptr, inner, outer, inner, box_inner, box_outer, 0);
}

template <bool DUAL, bool SPLIT>
int ensure_attr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(2, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lk(g_ops_mu);
  if (!g_attr_set[dev][DUAL][SPLIT]) {
    const cudaError_t e = cudaFuncSetAttribute(chain_gemm_kernel<DUAL, SPLIT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(chain_smem_bytes<DUAL>()));
    if (e != cudaSuccess) return fail(4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    g_attr_set[dev][DUAL][SPLIT] = true;
  }
  return 0;
}

template <bool DUAL, bool SPLIT>
int launch_chain_t(const CUtensorMap &ma, const CUtensorMap &mb0, const CUtensorMap &mb1,
                   const ChainArgs &args, cudaStream_t st) {
  if (int rc = ensure_attr<DUAL, SPLIT>()) return rc;
  const dim3 grid((args.N + CB - 1) / CB, (args.rows + RB - 1) / RB);
  const cudaError_t e = qb200_launch(chain_gemm_kernel<DUAL, SPLIT>, grid,
                                     dim3(chain_threads<DUAL, SPLIT>()), chain_smem_bytes<DUAL>(), st,
                                     true, ma, mb0, mb1, args);
  if (e != cudaSuccess) return fail(20, "SwiGLU kernel launch: %s", cudaGetErrorString(e));
  return 0;
}

// C[rows, N] = chain(A[rows, K], B0[K, N] (, B1)).
template <bool DUAL>
int launch_chain(const __half *a, const __half *b0, const __half *b1, const ChainArgs &args,
                 cudaStream_t st) {
  CUtensorMap ma, mb0, mb1;
  if (int rc = make_map(&ma, a, args.K, args.rows, KC, RB)) return rc;
  if (int rc = make_map(&mb0, b0, args.N, args.K, CB, KC)) return rc;
  if (DUAL) {
    if (int rc = make_map(&mb1, b1, args.N, args.K, CB, KC)) return rc;
  } else {
    mb1 = mb0;
  }
  // Gate/up of a single row tile: one chain per thread (latency-bound); more
  // rows: both chains per thread (issue-bound).
  if (DUAL && args.rows <= RB) return launch_chain_t<DUAL, true>(ma, mb0, mb1, args, st);
  return launch_chain_t<DUAL, false>(ma, mb0, mb1, args, st);
}

int check_swiglu(const void *x, const void *wg, const void *wu, const void *wd, const void *bg,
                 const void *bu, const void *bd, long long rows, int hidden, int inter) {
  if (rows < 0 || rows > static_cast<long long>(MAX_ROW_TILES) * RB)
    return fail(10, "rows=%lld out of range [0, %d]", rows, MAX_ROW_TILES * RB);
  if (hidden <= 0 || inter <= 0 || (hidden & 7) || (inter & 7))
    return fail(10, "hidden=%d and inter=%d must be positive multiples of 8", hidden, inter);
  if (rows == 0) return 0;  // nothing to read or write; empty tensors may have null pointers
  if (x == nullptr || wg == nullptr || wu == nullptr) return fail(13, "null pointer argument");
  for (const void *q : {x, wg, wu, wd, bg, bu, bd})
    if (q != nullptr && !al16(q)) return fail(14, "SwiGLU operands must be 16-byte aligned");
  return 0;
}

long long round256(long long b) { return (b + 255) & ~255ll; }

// SwiGLU + down workspace: the activations (fp16 s for the chains, its hi |
// lo parts for the tensor cores), then room for the down projection's fp32 K
// slices: 12 bytes per activation, i.e. 8 slices whenever hidden <= 3 inter / 8
// (Qwen3-0.6B: hidden = inter / 3).
long long swiglu_ws_act(long long rows, int inter) { return round256(rows * inter * 4); }
long long swiglu_ws_part(long long rows, int inter) { return round256(rows * inter * 12); }

int rmsnorm_launch(void *out, float *rms, const void *input, const void *weight, void *residual,
                   long long rows, int cols, float eps, cudaStream_t st) {
  if (rows < 0 || cols <= 0) return fail(10, "rows=%lld cols=%d out of range", rows, cols);
  if (rows == 0) return 0;
  if (out == nullptr || rms == nullptr || input == nullptr || weight == nullptr)
    return fail(13, "null pointer argument");
  if ((cols & 7) == 0) {
    for (const void *q : {static_cast<const void *>(out), input, weight,
                          static_cast<const void *>(residual)})
      if (q != nullptr && !al16(q)) return fail(14, "RMSNorm operands must be 16-byte aligned");
  }
  // Up to a few thousand rows: one-warp CTAs, so that the rows spread over
  // all SMs (eight rows per CTA put 256 rows on 32 SMs); more: eight per CTA.
  const int wpc = rows >= 8 * 148 ? 8 : 1;
  const long long blocks = (rows + wpc - 1) / wpc;
  if (blocks > 0x7fffffffll) return fail(10, "rows=%lld too large", rows);
  const cudaError_t e = qb200_launch(
      rmsnorm_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * wpc), 0, st, true,
      static_cast<__half *>(out), rms, static_cast<const __half *>(input),
      static_cast<const __half *>(weight), static_cast<__half *>(residual), rows, cols, eps);
  if (e != cudaSuccess) return fail(20, "RMSNorm kernel launch: %s", cudaGetErrorString(e));
  return 0;
}

int swiglu_forward_launch(const void *x, const void *wg, const void *wu, const void *bg,
                          const void *bu, void *out, void *gc, void *uc, long long rows,
                          int hidden, int inter, cudaStream_t st) {
  ChainArgs a{};
  a.init0 = static_cast<const __half *>(bg);
  a.init1 = static_cast<const __half *>(bu);
  a.out = static_cast<__half *>(out);
  a.cache0 = static_cast<__half *>(gc);
  a.cache1 = static_cast<__half *>(uc);
  a.rows = static_cast<int>(rows);
  a.K = hidden;
  a.N = inter;
  return launch_chain<true>(static_cast<const __half *>(x), static_cast<const __half *>(wg),
                            static_cast<const __half *>(wu), a, st);
}

int down_launch(const void *s, const void *wd, const void *bd, void *out, long long rows,
                int hidden, int inter, cudaStream_t st) {
  ChainArgs a{};
  a.init0 = static_cast<const __half *>(bd);
  a.out = static_cast<__half *>(out);
  a.rows = static_cast<int>(rows);
  a.K = inter;
  a.N = hidden;
  const __half *wdh = static_cast<const __half *>(wd);
  return launch_chain<false>(static_cast<const __half *>(s), wdh, wdh, a, st);
}

// Rows from which the dispatching entry points take the tensor-core path.
constexpr long long TC_MIN_ROWS = 64;

bool tc_shape_ok(int hidden, int inter) { return hidden % 64 == 0 && inter % 64 == 0 && hidden >= 64; }

// s[rows, inter] = silu(g) * u, g = x . w_gate + b_gate, u = x . w_up + b_up in
// fp32, then out[rows, hidden] = half(s . w_down + b_down): two tcgen05 GEMMs
// with fp32 accumulation on the upstream [K, N] weight layout (MN-major B).
// The gate|up GEMM holds 64 gate and 64 up columns per 128-column tile and
// stores s as fp16 hi = half(s) and lo = half(s - hi) ([rows, 2 inter] in
// sbuf); the down GEMM runs over K = 2 inter ([hi | lo] against w_down read
// twice), so s enters it with ~22 significant bits, and splits K into fp32
// slices in `part` (part_bytes) added by a reduction kernel -- or, when they
// do not fit there, over a thread-block cluster, which measured slower (18 us
// against 10 us at 64 rows, 14 against 12.5 at 256).
int swiglu_down_tc(const void *x, const void *wg, const void *wu, const void *wd, const void *bg,
                   const void *bu, const void *bd, void *sbuf, float *part, long long part_bytes, void *out,
                   long long rows, int hidden, int inter, cudaStream_t st) {
  const int M = static_cast<int>(rows);
  GemmPlan p1{};
  if (int rc = qb200_gemm_make_maps_mn(&p1, x, wg, wu, M, inter, hidden, hidden, inter, 128)) return rc;
  qb200tc::GemmArgs g1{};
  // Both GEMMs are programmatic dependents of their predecessor: launch and
  // weight-tile prefetch overlap the previous kernel's tail.
  g1.pdl = 1;
  g1.out = sbuf;
  g1.ldo = 2 * inter;
  g1.lo_col = inter;
  g1.bias = bg;
  g1.bias2 = bu;
  if (int rc = qb200_gemm_run(p1, qb200tc::EPI_SWIGLU2, g1, st)) return rc;
  GemmPlan p2{};
  if (int rc = qb200_gemm_make_maps_mn(&p2, sbuf, wd, nullptr, M, hidden, 2 * inter, 2 * inter, hidden,
                                       64, inter))
    return rc;
  qb200tc::GemmArgs g2{};
  g2.pdl = 1;
  g2.out = out;
  g2.ldo = hidden;
  g2.bias = bd;
  g2.b_kwrap = inter / qb200tc::BK;
  // 64-column tiles (128-column ones with 8 slices measured slower).
  const int nk = 2 * inter / qb200tc::BK;
  for (int splits : {8, 4, 2})
    if (splits <= nk && static_cast<long long>(splits) * M * hidden * 4 <= part_bytes)
      return qb200_gemm_run_splitk(p2, qb200tc::EPI_F16, g2, splits, part, st);
  const int tiles = (hidden / 64) * ((M + qb200tc::BM - 1) / qb200tc::BM);
  return qb200_gemm_run_splitk(p2, qb200tc::EPI_F16, g2, min(nk, tiles >= 32 ? 4 : 8), nullptr, st);
}

}  // namespace

// 2-D fp16 tensor [outer, inner] with row pitch `pitch` elements, box
// {box_inner, box_outer}, zero fill out of bounds; swizzle128 selects the
// 128-byte shared-memory swizzle.  0 or an error code (message recorded).
int qb200_encode_f16_2d(CUtensorMap *m, const void *ptr, long long inner, long long outer,
                        long long pitch, int box_inner, int box_outer, int swizzle128) {
  // A tensor map is a pure function of these arguments: the last few are kept
  // (operators re-plan their GEMMs on every call with the same buffers).
  struct Key {
    const void *ptr;
    long long inner, outer, pitch;
    int box_inner, box_outer, swizzle128;
    bool operator==(const Key &o) const {
      return ptr == o.ptr && inner == o.inner && outer == o.outer && pitch == o.pitch &&
             box_inner == o.box_inner && box_outer == o.box_outer && swizzle128 == o.swizzle128;
    }
  };
  constexpr int NCACHE = 64;
  static Key keys[NCACHE];
  static CUtensorMap maps[NCACHE];
  static int used = 0, next = 0;
  static std::mutex mu;
  const Key k{ptr, inner, outer, pitch, box_inner, box_outer, swizzle128};
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < used; ++i) {
      if (keys[i] == k) {
        *m = maps[i];
        return 0;
      }
    }
  }
  EncodeTiledFn enc = encoder();
  if (enc == nullptr) return fail(30, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                    : CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(31, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  std::lock_guard<std::mutex> lk(mu);
  keys[next] = k;
  maps[next] = *m;
  next = (next + 1) % NCACHE;
  if (used < NCACHE) ++used;
  return 0;
}

extern "C" {

int qwen_b200_rmsnorm_forward(void *out, float *rms, const void *input, const void *weight,
                              void *residual, long long rows, int cols, float eps, void *stream) {
  qb200_clear_error();
  return rmsnorm_launch(out, rms, input, weight, residual, rows, cols, eps,
                        static_cast<cudaStream_t>(stream));
}

int qwen_b200_swiglu_forward(const void *x, const void *w_gate, const void *w_up,
                             const void *b_gate, const void *b_up, void *out, void *gate_cache,
                             void *up_cache, long long rows, int hidden, int inter, void *stream) {
  qb200_clear_error();
  if (int rc = check_swiglu(x, w_gate, w_up, nullptr, b_gate, b_up, nullptr, rows, hidden, inter))
    return rc;
  if (rows == 0) return 0;
  if (out == nullptr) return fail(13, "null pointer argument");
  for (const void *q : {static_cast<const void *>(out), static_cast<const void *>(gate_cache),
                        static_cast<const void *>(up_cache)})
    if (q != nullptr && !al16(q)) return fail(14, "SwiGLU operands must be 16-byte aligned");
  return swiglu_forward_launch(x, w_gate, w_up, b_gate, b_up, out, gate_cache, up_cache, rows,
                               hidden, inter, static_cast<cudaStream_t>(stream));
}

long long qwen_b200_swiglu_forward_down_workspace(long long rows, int inter) {
  if (rows < 0 || inter < 0) return 0;
  return swiglu_ws_act(rows, inter) + swiglu_ws_part(rows, inter);
}

int qwen_b200_swiglu_forward_down(const void *x, const void *w_gate, const void *w_up,
                                  const void *w_down, const void *b_gate, const void *b_up,
                                  const void *b_down, void *out, void *workspace,
                                  long long rows, int hidden, int inter, void *stream) {
  qb200_clear_error();
  if (int rc = check_swiglu(x, w_gate, w_up, w_down, b_gate, b_up, b_down, rows, hidden, inter))
    return rc;
  if (rows == 0) return 0;
  if (w_down == nullptr || out == nullptr || workspace == nullptr)
    return fail(13, "null pointer argument");
  if (!al16(out) || !al16(workspace)) return fail(14, "SwiGLU operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = swiglu_forward_launch(x, w_gate, w_up, b_gate, b_up, workspace, nullptr, nullptr,
                                     rows, hidden, inter, st))
    return rc;
  return down_launch(workspace, w_down, b_down, out, rows, hidden, inter, st);
}

int qwen_b200_swiglu_forward_down_ex(const void *x, const void *w_gate, const void *w_up,
                                     const void *w_down, const void *b_gate, const void *b_up,
                                     const void *b_down, void *out, void *workspace,
                                     long long rows, int hidden, int inter, int mode, void *stream) {
  qb200_clear_error();
  if (mode < -1 || mode > 1) return fail(10, "mode=%d: -1 (by size), 0 (tensor cores) or 1 (exact)", mode);
  const bool tc = mode == 0 || (mode == -1 && rows >= TC_MIN_ROWS && tc_shape_ok(hidden, inter));
  if (!tc) return qwen_b200_swiglu_forward_down(x, w_gate, w_up, w_down, b_gate, b_up, b_down, out,
                                                workspace, rows, hidden, inter, stream);
  if (int rc = check_swiglu(x, w_gate, w_up, w_down, b_gate, b_up, b_down, rows, hidden, inter))
    return rc;
  if (rows == 0) return 0;
  if (!tc_shape_ok(hidden, inter))
    return fail(10, "the tensor-core path needs hidden and inter multiples of 64 (got %d, %d)", hidden, inter);
  if (rows > 0x7fffffffll) return fail(10, "rows=%lld out of range", rows);
  if (w_down == nullptr || out == nullptr || workspace == nullptr)
    return fail(13, "null pointer argument");
  if (!al16(out) || !al16(workspace)) return fail(14, "SwiGLU operands must be 16-byte aligned");
  float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + swiglu_ws_act(rows, inter));
  return swiglu_down_tc(x, w_gate, w_up, w_down, b_gate, b_up, b_down, workspace, part,
                        swiglu_ws_part(rows, inter), out, rows, hidden, inter, static_cast<cudaStream_t>(stream));
}

int qwen_b200_rmsnorm_swiglu_down_ex(const void *x, const void *norm_weight, void *residual,
                                     float eps, const void *w_gate, const void *w_up,
                                     const void *w_down, const void *b_gate, const void *b_up,
                                     const void *b_down, void *normed, float *rms, void *out,
                                     void *workspace, long long rows, int hidden, int inter, int mode,
                                     void *stream) {
  qb200_clear_error();
  if (mode < -1 || mode > 1) return fail(10, "mode=%d: -1 (by size), 0 (tensor cores) or 1 (exact)", mode);
  const bool tc = mode == 0 || (mode == -1 && rows >= TC_MIN_ROWS && tc_shape_ok(hidden, inter));
  if (!tc) return qwen_b200_rmsnorm_swiglu_down(x, norm_weight, residual, eps, w_gate, w_up, w_down,
                                                b_gate, b_up, b_down, normed, rms, out, workspace,
                                                rows, hidden, inter, stream);
  if (int rc = check_swiglu(x, w_gate, w_up, w_down, b_gate, b_up, b_down, rows, hidden, inter))
    return rc;
  if (rows == 0) return 0;
  if (!tc_shape_ok(hidden, inter))
    return fail(10, "the tensor-core path needs hidden and inter multiples of 64 (got %d, %d)", hidden, inter);
  if (rows > 0x7fffffffll) return fail(10, "rows=%lld out of range", rows);
  if (norm_weight == nullptr || w_down == nullptr || rms == nullptr || out == nullptr ||
      workspace == nullptr)
    return fail(13, "null pointer argument");
  for (const void *q : {norm_weight, static_cast<const void *>(residual),
                        static_cast<const void *>(normed), static_cast<const void *>(out),
                        static_cast<const void *>(workspace)})
    if (q != nullptr && !al16(q)) return fail(14, "operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *nbuf = normed != nullptr ? normed : ws;
  void *sbuf = ws + round256(rows * hidden * 2);
  if (int rc = rmsnorm_launch(nbuf, rms, x, norm_weight, residual, rows, hidden, eps, st)) return rc;
  float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(sbuf) + swiglu_ws_act(rows, inter));
  return swiglu_down_tc(nbuf, w_gate, w_up, w_down, b_gate, b_up, b_down, sbuf, part, swiglu_ws_part(rows, inter),
                        out, rows, hidden, inter, st);
}

long long qwen_b200_rmsnorm_swiglu_down_workspace(long long rows, int hidden, int inter) {
  if (rows < 0 || hidden < 0 || inter < 0) return 0;
  return round256(rows * hidden * 2) + swiglu_ws_act(rows, inter) + swiglu_ws_part(rows, inter);
}

int qwen_b200_rmsnorm_swiglu_down(const void *x, const void *norm_weight, void *residual,
                                  float eps, const void *w_gate, const void *w_up,
                                  const void *w_down, const void *b_gate, const void *b_up,
                                  const void *b_down, void *normed, float *rms, void *out,
                                  void *workspace, long long rows, int hidden, int inter,
                                  void *stream) {
  qb200_clear_error();
  if (int rc = check_swiglu(x, w_gate, w_up, w_down, b_gate, b_up, b_down, rows, hidden, inter))
    return rc;
  if (rows == 0) return 0;
  if (norm_weight == nullptr || w_down == nullptr || rms == nullptr || out == nullptr ||
      workspace == nullptr)
    return fail(13, "null pointer argument");
  for (const void *q : {norm_weight, static_cast<const void *>(residual),
                        static_cast<const void *>(normed), static_cast<const void *>(out),
                        static_cast<const void *>(workspace)})
    if (q != nullptr && !al16(q)) return fail(14, "operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *nbuf = normed != nullptr ? normed : ws;
  void *sbuf = ws + round256(rows * hidden * 2);
  if (int rc = rmsnorm_launch(nbuf, rms, x, norm_weight, residual, rows, hidden, eps, st)) return rc;
  if (int rc = swiglu_forward_launch(nbuf, w_gate, w_up, b_gate, b_up, sbuf, nullptr, nullptr, rows,
                                     hidden, inter, st))
    return rc;
  return down_launch(sbuf, w_down, b_down, out, rows, hidden, inter, st);
}

int qwen_b200_ops_status(uint64_t *detail) {
  unsigned long long v = 0;
  int rc = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&v, g_ops_err, sizeof(v)) != cudaSuccess) {
    rc = -2;
  } else if (v != 0) {
    rc = static_cast<int>(v >> 32);
    const unsigned long long zero = 0;
    cudaMemcpyToSymbol(g_ops_err, &zero, sizeof(zero));
  }
  if (detail) *detail = v;
  return rc;
}

}  // extern "C"
