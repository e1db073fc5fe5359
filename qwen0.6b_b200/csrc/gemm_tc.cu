// gemm_tc.cu - host side of the tcgen05 GEMM (gemm_tc.cuh): tensor maps, tile
// width choice, the final argmax reduction of EPI_ARGMAX, and the test entry
// point of include/qwen_b200_batched.h.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "gemm_tc.cuh"
#include "gemm_tc_host.h"
#include "host_err.h"
#include "qwen_b200_batched.h"

namespace qb200tc {

// Row argmax over the per-tile partials: largest value, lowest column index
// among equal values.  One warp per row.
__global__ void argmax_reduce_kernel(const float *__restrict__ part_val,
                                     const int *__restrict__ part_idx, int n_tiles, int rows,
                                     int *__restrict__ out) {
  qb200::griddep_wait();
  qb200::griddep_launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = lane; t < n_tiles; t += 32) {
    const float v = part_val[static_cast<size_t>(row) * n_tiles + t];
    const int i = part_idx[static_cast<size_t>(row) * n_tiles + t];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  if (lane == 0) out[row] = bi == 0x7fffffff ? -1 : bi;
}

// Split-K reduction: sum the k_splits fp32 partial slices in slice order and
// apply the final epilogue (EPI_F16: + bias in fp32 when given, as the GEMM
// epilogue).  Thread = 4 consecutive columns of one row.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float *__restrict__ part,
                                                            int splits, int M, int N, int epi,
                                                            const void *__restrict__ res,
                                                            const __half *__restrict__ bias,
                                                            void *__restrict__ out, int ldo) {
  qb200::griddep_wait();
  qb200::griddep_launch_dependents();
  const long long q = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nq = N / 4;
  if (q >= static_cast<long long>(M) * nq) return;
  const int row = static_cast<int>(q / nq), col = static_cast<int>(q % nq) * 4;
  const size_t slice = static_cast<size_t>(M) * N;
  float4 acc = reinterpret_cast<const float4 *>(part + static_cast<size_t>(row) * N + col)[0];
  for (int z = 1; z < splits; ++z) {
    const float4 v = reinterpret_cast<const float4 *>(part + z * slice + static_cast<size_t>(row) * N + col)[0];
    acc.x = __fadd_rn(acc.x, v.x);
    acc.y = __fadd_rn(acc.y, v.y);
    acc.z = __fadd_rn(acc.z, v.z);
    acc.w = __fadd_rn(acc.w, v.w);
  }
  const float a[4] = {acc.x, acc.y, acc.z, acc.w};
  const size_t o = static_cast<size_t>(row) * ldo + col;
  if (epi == EPI_SWIGLU) {
    // Column pairs (gate, up) -> output column col / 2 (ldo counts outputs).
    __half *out16 = static_cast<__half *>(out) + static_cast<size_t>(row) * ldo + col / 2;
    out16[0] = __float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(a[0]))), a[1]));
    out16[1] = __float2half_rn(__fmul_rn(__half2float(silu_half(__float2half_rn(a[2]))), a[3]));
  } else if (epi == EPI_F32_RES16) {
    const __half *r = static_cast<const __half *>(res) + o;
    float4 w;
    w.x = __fadd_rn(a[0], __half2float(r[0]));
    w.y = __fadd_rn(a[1], __half2float(r[1]));
    w.z = __fadd_rn(a[2], __half2float(r[2]));
    w.w = __fadd_rn(a[3], __half2float(r[3]));
    *reinterpret_cast<float4 *>(static_cast<float *>(out) + o) = w;
  } else if (epi == EPI_F16_RES32) {
    const float4 r = *reinterpret_cast<const float4 *>(static_cast<const float *>(res) + o);
    __half2 h[2] = {__floats2half2_rn(__fadd_rn(a[0], r.x), __fadd_rn(a[1], r.y)),
                    __floats2half2_rn(__fadd_rn(a[2], r.z), __fadd_rn(a[3], r.w))};
    *reinterpret_cast<uint2 *>(static_cast<__half *>(out) + o) = *reinterpret_cast<const uint2 *>(h);
  } else if (epi == EPI_F32) {
    *reinterpret_cast<float4 *>(static_cast<float *>(out) + o) = acc;
  } else {  // EPI_F16
    float b[4] = {a[0], a[1], a[2], a[3]};
    if (bias != nullptr)
      for (int i = 0; i < 4; ++i) b[i] = __fadd_rn(b[i], __half2float(bias[col + i]));
    __half2 h[2] = {__floats2half2_rn(b[0], b[1]), __floats2half2_rn(b[2], b[3])};
    *reinterpret_cast<uint2 *>(static_cast<__half *>(out) + o) = *reinterpret_cast<const uint2 *>(h);
  }
}

// Like argmax_reduce_kernel, but keeps the winning value too and offsets the
// index (a vocabulary shard's first row): out_val / out_idx [rows].
__global__ void argmax_pair_kernel(const float *__restrict__ part_val,
                                   const int *__restrict__ part_idx, int n_tiles, int rows,
                                   long long offset, float *__restrict__ out_val,
                                   int *__restrict__ out_idx) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = lane; t < n_tiles; t += 32) {
    const float v = part_val[static_cast<size_t>(row) * n_tiles + t];
    const int i = part_idx[static_cast<size_t>(row) * n_tiles + t];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  if (lane == 0) {
    out_val[row] = best;
    out_idx[row] = bi == 0x7fffffff ? -1 : static_cast<int>(bi + offset);
  }
}

// Cross-shard pick: vals / idxs [world, rows] (one pair per shard and row) ->
// out[r] = index of the largest value, lowest index among equal values.
__global__ void argmax_pick_kernel(const float *__restrict__ vals, const int *__restrict__ idxs,
                                   int world, int rows, int *__restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float best = -INFINITY;
  int bi = -1;
  for (int w = 0; w < world; ++w) {
    const float v = vals[static_cast<size_t>(w) * rows + r];
    const int i = idxs[static_cast<size_t>(w) * rows + r];
    if (i < 0) continue;
    if (bi < 0 || v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  out[r] = bi;
}

}  // namespace qb200tc

using namespace qb200tc;

namespace {

std::mutex g_mu;
bool g_attr[64][3][8][3] = {};  // [device][BN 64/128/256][epilogue][B layout]

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return qb200_set_error(code, buf);
}

template <int BN, int EPI, int BL = BL_K>
int launch_t(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mb2, const GemmArgs &g,
             cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(2, "cudaGetDevice failed");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    bool &done = g_attr[dev][BN == 64 ? 0 : (BN == 128 ? 1 : 2)][EPI][BL];
    if (!done) {
      const cudaError_t e = cudaFuncSetAttribute(
          gemm_tc_kernel<BN, EPI, BL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
          static_cast<int>(GemmSmem<BN>::bytes(GemmSmem<BN>::MAX_STAGES)));
      if (e != cudaSuccess) return fail(4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done = true;
    }
  }
  // B larger than a quarter of L2 (the lm_head's 311 MB): the row tiles of a
  // column tile are launched next to each other (grid.x), so that the second
  // row tile reads B from L2 instead of DRAM.
  const unsigned mt = static_cast<unsigned>((g.M + BM - 1) / BM), nt = static_cast<unsigned>((g.N + BN - 1) / BN);
  if (g.a_box < 8 || g.a_box > BM || (g.a_box & 7)) return fail(10, "A box of %d rows", g.a_box);
  GemmArgs ga = g;
  ga.m_fast = mt > 1 && nt <= 65535u && static_cast<long long>(g.N) * g.K * 2 > (32ll << 20);
  const dim3 grid(ga.m_fast ? mt : nt, ga.m_fast ? nt : mt, g.k_splits > 1 ? g.k_splits : 1);
  // One wave of CTAs: the deepest ring; more: a ring half as deep, so that
  // two CTAs share an SM.
  const long long ctas = static_cast<long long>(grid.x) * grid.y * grid.z;
  ga.stages = ctas <= 148 ? GemmSmem<BN>::MAX_STAGES : GemmSmem<BN>::MAX_STAGES / 2;
  // The epilogue stages its tiles in the ring.
  ga.stages = max(ga.stages, GemmSmem<BN>::min_stages(ga.cluster_k != 0 && grid.z > 1));
  const cudaError_t e = qb200_launch_cl(gemm_tc_kernel<BN, EPI, BL>, grid, dim3(THREADS),
                                        GemmSmem<BN>::bytes(ga.stages), st, ga.pdl != 0,
                                        ga.cluster_k ? static_cast<int>(grid.z) : 1, ma, mb, mb2, ga);
  if (e != cudaSuccess) return fail(20, "GEMM launch: %s", cudaGetErrorString(e));
  return 0;
}

template <int BN>
int launch_bn(int epi, const CUtensorMap &ma, const CUtensorMap &mb, const GemmArgs &g,
              cudaStream_t st) {
  switch (epi) {
    case EPI_F16: return launch_t<BN, EPI_F16>(ma, mb, mb, g, st);
    case EPI_F32: return launch_t<BN, EPI_F32>(ma, mb, mb, g, st);
    case EPI_F32_RES16: return launch_t<BN, EPI_F32_RES16>(ma, mb, mb, g, st);
    case EPI_SWIGLU: return launch_t<BN, EPI_SWIGLU>(ma, mb, mb, g, st);
    case EPI_F16_RES32: return launch_t<BN, EPI_F16_RES32>(ma, mb, mb, g, st);
    case EPI_ARGMAX: return launch_t<BN, EPI_ARGMAX>(ma, mb, mb, g, st);
    case EPI_PARTIAL: return launch_t<BN, EPI_PARTIAL>(ma, mb, mb, g, st);
    default: return fail(10, "unknown epilogue %d", epi);
  }
}

// MN-major B: the plain projection (EPI_F16, optional bias; split-K inside a
// cluster) and the gate|up pair (EPI_SWIGLU2, BN = 128).
template <int BN>
int launch_bn_mn(int epi, const GemmPlan &p, const GemmArgs &g, cudaStream_t st) {
  if (p.bl == BL_MN2) {
    if (epi != EPI_SWIGLU2 || BN != 128) return fail(10, "the gate|up layout takes EPI_SWIGLU2 at BN 128");
    return launch_t<128, EPI_SWIGLU2, BL_MN2>(p.ma, p.mb, p.mb2, g, st);
  }
  switch (epi) {
    case EPI_F16: return launch_t<BN, EPI_F16, BL_MN>(p.ma, p.mb, p.mb, g, st);
    case EPI_F32: return launch_t<BN, EPI_F32, BL_MN>(p.ma, p.mb, p.mb, g, st);
    case EPI_PARTIAL: return launch_t<BN, EPI_PARTIAL, BL_MN>(p.ma, p.mb, p.mb, g, st);
    default: return fail(10, "epilogue %d is not built for an MN-major B", epi);
  }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rows per A copy: a whole 128-row tile, or, for fewer planned rows, the rows
// rounded up to a swizzle atom (8): the tile's other rows are never copied.
int a_box_rows(int M) { return M >= BM ? BM : ((M + 7) / 8) * 8; }

bool g_attr_argmax[64][3] = {};  // [device][BN 64/128/256]
int g_sm_count[64] = {};

template <int BN>
int launch_argmax(const GemmPlan &p, const GemmArgs &g, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(2, "cudaGetDevice failed");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    bool &done = g_attr_argmax[dev][BN == 64 ? 0 : (BN == 128 ? 1 : 2)];
    if (!done) {
      cudaError_t e = cudaFuncSetAttribute(gemm_argmax_persistent<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(GemmSmem<BN>::bytes(GemmSmem<BN>::MAX_STAGES)));
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return fail(4, "argmax GEMM set-up: %s", cudaGetErrorString(e));
      done = true;
    }
  }
  GemmArgs ga = g;
  ga.stages = GemmSmem<BN>::MAX_STAGES;
  const long long tiles = static_cast<long long>((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const unsigned grid = static_cast<unsigned>(tiles < g_sm_count[dev] ? tiles : g_sm_count[dev]);
  const cudaError_t e = qb200_launch(gemm_argmax_persistent<BN>, dim3(grid), dim3(THREADS),
                                     GemmSmem<BN>::bytes(ga.stages), st, ga.pdl != 0, p.ma, p.mb, ga);
  if (e != cudaSuccess) return fail(20, "argmax GEMM launch: %s", cudaGetErrorString(e));
  return 0;
}

}  // namespace

int qb200_gemm_run_argmax(const GemmPlan &p, GemmArgs g, cudaStream_t st) {
  if (p.bl != BL_K) return fail(10, "the persistent argmax GEMM takes a K-major B");
  if (g.part_val == nullptr || g.part_idx == nullptr) return fail(13, "argmax partials missing");
  g.M = (g.M > 0 && g.M < p.M) ? g.M : p.M;
  g.N = p.N;
  g.K = p.K;
  g.a_box = p.a_box;
  g.n_tiles = (p.N + p.bn - 1) / p.bn;
  if (g.a_box < 8 || g.a_box > BM || (g.a_box & 7)) return fail(10, "A box of %d rows", g.a_box);
  if (p.bn == 256) return launch_argmax<256>(p, g, st);
  return p.bn == 128 ? launch_argmax<128>(p, g, st) : launch_argmax<64>(p, g, st);
}

int qb200_gemm_bn(int M, int N) {
  const long long tiles128 = static_cast<long long>((N + 127) / 128) * ((M + BM - 1) / BM);
  return tiles128 >= 120 ? 128 : 64;
}

int qb200_gemm_make_maps(GemmPlan *p, const void *a, const void *b, int M, int N, int K, int lda,
                         int ldb) {
  if (M < 1 || N < 16 || K < BK || (N & 15) || (K % BK))
    return fail(10, "GEMM shape M=%d N=%d K=%d: need M >= 1, N a multiple of 16, K a multiple of %d",
                M, N, K, BK);
  if (!al16(a) || !al16(b) || (lda & 7) || (ldb & 7))
    return fail(14, "GEMM operands must be 16-byte aligned with row pitches a multiple of 8");
  p->M = M;
  p->N = N;
  p->K = K;
  p->bn = qb200_gemm_bn(M, N);
  p->b_ptr = b;
  p->ldb = ldb;
  p->a_box = a_box_rows(M);
  if (int rc = qb200_encode_f16_2d(&p->ma, a, K, M, lda, BK, p->a_box, 1)) return rc;
  if (int rc = qb200_encode_f16_2d(&p->mb, b, K, N, ldb, BK, p->bn, 1)) return rc;
  return 0;
}

int qb200_gemm_run(const GemmPlan &p, int epi, GemmArgs g, cudaStream_t st) {
  g.M = (g.M > 0 && g.M < p.M) ? g.M : p.M;  // fewer rows than planned: the rest stay untouched
  g.a_box = p.a_box;
  g.N = p.N;
  g.K = p.K;
  g.n_tiles = (p.N + p.bn - 1) / p.bn;
  if (p.bl != BL_K)
    return p.bn == 128 ? launch_bn_mn<128>(epi, p, g, st) : launch_bn_mn<64>(epi, p, g, st);
  if (p.bn == 256) return launch_bn<256>(epi, p.ma, p.mb, g, st);
  return p.bn == 128 ? launch_bn<128>(epi, p.ma, p.mb, g, st) : launch_bn<64>(epi, p.ma, p.mb, g, st);
}

int qb200_gemm_set_bn(GemmPlan *p, int bn) {
  if (p->bl != BL_K || (bn != 64 && bn != 128 && bn != 256))
    return fail(10, "tile width %d: 64, 128 or 256 columns (K-major B only)", bn);
  p->bn = bn;
  // The B tensor map's box height is the tile width.
  return qb200_encode_f16_2d(&p->mb, p->b_ptr, p->K, p->N, p->ldb, BK, bn, 1);
}

int qb200_gemm_make_maps_mn(GemmPlan *p, const void *a, const void *b, const void *b2, int M, int N,
                            int K, int lda, int ldb, int bn, int b_rows) {
  if (b_rows <= 0) b_rows = K;
  const int n_cols = b2 != nullptr ? 2 * N : N;  // gate|up: the accumulator holds both
  if (M < 1 || N < 64 || K < BK || (N & 63) || (K % BK) || b_rows < BK || (b_rows % BK))
    return fail(10, "GEMM shape M=%d N=%d K=%d: need N a multiple of 64 and K a multiple of %d", M, N,
                K, BK);
  if (!al16(a) || !al16(b) || (b2 != nullptr && !al16(b2)) || (lda & 7) || (ldb & 7))
    return fail(14, "GEMM operands must be 16-byte aligned with row pitches a multiple of 8");
  if (b2 != nullptr && bn != 128) return fail(10, "the gate|up layout needs 128-column tiles");
  p->M = M;
  p->N = n_cols;
  p->K = K;
  p->bn = bn;
  p->bl = b2 != nullptr ? BL_MN2 : BL_MN;
  p->a_box = a_box_rows(M);
  if (int rc = qb200_encode_f16_2d(&p->ma, a, K, M, lda, BK, p->a_box, 1)) return rc;
  // B stored [K, N] (N contiguous): boxes of 64 columns x BK rows, 128-byte swizzle.
  if (int rc = qb200_encode_f16_2d(&p->mb, b, N, b_rows, ldb, 64, BK, 1)) return rc;
  if (b2 != nullptr) {
    if (int rc = qb200_encode_f16_2d(&p->mb2, b2, N, b_rows, ldb, 64, BK, 1)) return rc;
  } else {
    p->mb2 = p->mb;
  }
  return 0;
}

int qb200_gemm_run_splitk(const GemmPlan &p, int epi, GemmArgs g, int splits, float *partial,
                          cudaStream_t st) {
  const int nk = p.K / BK;
  if (splits < 2 || splits > nk) return fail(10, "k_splits=%d out of range [2, %d]", splits, nk);
  if (epi != EPI_F16 && epi != EPI_F32 && epi != EPI_F32_RES16 && epi != EPI_F16_RES32 && epi != EPI_SWIGLU)
    return fail(10, "epilogue %d cannot follow a split-K reduction", epi);
  if (splits <= 8 && partial == nullptr) {
    // The k slices of a tile form one cluster and are added in shared memory.
    GemmArgs gc = g;
    gc.k_splits = splits;
    gc.cluster_k = 1;
    return qb200_gemm_run(p, epi, gc, st);
  }
  GemmArgs gp = g;
  gp.out = partial;
  gp.ldo = p.N;
  gp.res = nullptr;
  gp.k_splits = splits;
  if (int rc = qb200_gemm_run(p, EPI_PARTIAL, gp, st)) return rc;
  const int M = (g.M > 0 && g.M < p.M) ? g.M : p.M;
  const long long threads = static_cast<long long>(M) * (p.N / 4);
  const cudaError_t e = qb200_launch(splitk_reduce_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)),
                                     dim3(256), 0, st, g.pdl != 0, static_cast<const float *>(partial),
                                     splits, M, p.N, epi, g.res, static_cast<const __half *>(g.bias), g.out,
                                     g.ldo);
  if (e != cudaSuccess) return fail(20, "split-K reduce launch: %s", cudaGetErrorString(e));
  return 0;
}

int qb200_argmax_reduce(const float *part_val, const int *part_idx, int n_tiles, int rows, int *out,
                        cudaStream_t st, bool pdl) {
  const int wpb = 8;
  const cudaError_t e = qb200_launch(argmax_reduce_kernel, dim3((rows + wpb - 1) / wpb), dim3(32 * wpb), 0,
                                     st, pdl, part_val, part_idx, n_tiles, rows, out);
  if (e != cudaSuccess) return fail(20, "argmax launch: %s", cudaGetErrorString(e));
  return 0;
}

extern "C" {

// The lm_head argmax takes 256-column tiles: four N = 256 MMAs per k-block
// keep the tensor pipe at its peak rate, where N = 128 ones lose ~40 % to the
// per-k-block commit (103 -> 69 us per 311 MB lm_head at 256 rows, cold).
constexpr int LMHEAD_BN = 256;

long long qwen_b200_lmhead_argmax_workspace(int rows, int vocab_rows) {
  if (rows < 1 || vocab_rows < 16) return 0;
  return static_cast<long long>(rows) * ((vocab_rows + LMHEAD_BN - 1) / LMHEAD_BN) * 8;
}

int qwen_b200_lmhead_argmax(const void *hidden, const void *weight, int rows, int vocab_rows,
                            long long index_offset, float *out_val, int *out_idx, void *workspace,
                            void *stream) {
  qb200_clear_error();
  if (hidden == nullptr || weight == nullptr || out_val == nullptr || out_idx == nullptr ||
      workspace == nullptr)
    return fail(13, "null pointer argument");
  if (index_offset < 0 || index_offset + vocab_rows > 0x7fffffffll)
    return fail(10, "index_offset=%lld out of range", index_offset);
  GemmPlan p{};
  if (int rc = qb200_gemm_make_maps(&p, hidden, weight, rows, vocab_rows, 1024, 1024, 1024)) return rc;
  if (int rc = qb200_gemm_set_bn(&p, LMHEAD_BN)) return rc;
  const int n_tiles = (vocab_rows + p.bn - 1) / p.bn;
  GemmArgs g{};
  g.ldo = 1;
  g.part_val = static_cast<float *>(workspace);
  g.part_idx = reinterpret_cast<int *>(g.part_val + static_cast<size_t>(rows) * n_tiles);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = qb200_gemm_run_argmax(p, g, st)) return rc;
  const int wpb = 8;
  argmax_pair_kernel<<<(rows + wpb - 1) / wpb, 32 * wpb, 0, st>>>(g.part_val, g.part_idx, n_tiles,
                                                                 rows, index_offset, out_val, out_idx);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "argmax launch: %s", cudaGetErrorString(e));
  return 0;
}

int qwen_b200_argmax_pick(const float *vals, const int *idxs, int world, int rows, int *out,
                          void *stream) {
  qb200_clear_error();
  if (vals == nullptr || idxs == nullptr || out == nullptr) return fail(13, "null pointer argument");
  if (world < 1 || rows < 1) return fail(10, "world=%d rows=%d out of range", world, rows);
  argmax_pick_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(vals, idxs, world,
                                                                                    rows, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "pick launch: %s", cudaGetErrorString(e));
  return 0;
}

long long qwen_b200_gemm_argmax_workspace(int M, int N) {
  if (M < 1 || N < 16) return 0;
  const int bn = qb200_gemm_bn(M, N);
  const long long tiles = (N + bn - 1) / bn;
  return static_cast<long long>(M) * tiles * 8;
}

int qwen_b200_gemm_f16(int epilogue, const void *a, const void *b, void *out, const void *res,
                       void *workspace, int M, int N, int K, int ldo, int k_splits, void *stream) {
  return qwen_b200_gemm_f16_tiled(epilogue, a, b, out, res, workspace, M, N, K, ldo, k_splits, 0,
                                  stream);
}

int qwen_b200_gemm_f16_tiled(int epilogue, const void *a, const void *b, void *out, const void *res,
                             void *workspace, int M, int N, int K, int ldo, int k_splits, int bn,
                             void *stream) {
  qb200_clear_error();
  if (a == nullptr || b == nullptr || out == nullptr) return fail(13, "null pointer argument");
  if (epilogue < 0 || epilogue > EPI_ARGMAX) return fail(10, "unknown epilogue %d", epilogue);
  if ((epilogue == EPI_F32_RES16 || epilogue == EPI_F16_RES32) && res == nullptr)
    return fail(13, "this epilogue needs a residual");
  if (epilogue == EPI_ARGMAX && workspace == nullptr) return fail(13, "argmax needs a workspace");
  if (k_splits > 8 && workspace == nullptr) return fail(13, "more than 8 k slices need a workspace");
  GemmPlan p{};
  if (int rc = qb200_gemm_make_maps(&p, a, b, M, N, K, K, K)) return rc;
  if (bn != 0) {
    if (epilogue == EPI_ARGMAX) return fail(10, "the argmax epilogue takes the default tile width");
    if (int rc = qb200_gemm_set_bn(&p, bn)) return rc;
  }
  GemmArgs g{};
  g.ldo = epilogue == EPI_SWIGLU ? N / 2 : (epilogue == EPI_ARGMAX ? 1 : ldo);
  if (epilogue != EPI_ARGMAX && epilogue != EPI_SWIGLU && ldo < N)
    return fail(10, "ldo=%d < N=%d", ldo, N);
  g.out = out;
  g.res = res;
  const int n_tiles = (N + p.bn - 1) / p.bn;
  if (epilogue == EPI_ARGMAX) {
    g.part_val = static_cast<float *>(workspace);
    g.part_idx = reinterpret_cast<int *>(static_cast<float *>(workspace) +
                                         static_cast<size_t>(M) * n_tiles);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k_splits > 1) return qb200_gemm_run_splitk(p, epilogue, g, k_splits, static_cast<float *>(workspace), st);
  if (int rc = qb200_gemm_run(p, epilogue, g, st)) return rc;
  if (epilogue == EPI_ARGMAX)
    return qb200_argmax_reduce(g.part_val, g.part_idx, n_tiles, M, static_cast<int *>(out), st);
  return 0;
}

}  // extern "C"
