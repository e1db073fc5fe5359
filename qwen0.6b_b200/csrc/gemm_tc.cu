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

}  // namespace qb200tc

using namespace qb200tc;

namespace {

std::mutex g_mu;
bool g_attr[64][2][6] = {};

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return qb200_set_error(code, buf);
}

template <int BN, int EPI>
int launch_t(const CUtensorMap &ma, const CUtensorMap &mb, const GemmArgs &g, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(2, "cudaGetDevice failed");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    bool &done = g_attr[dev][BN == 128][EPI];
    if (!done) {
      const cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(GemmSmem<BN>::BYTES));
      if (e != cudaSuccess) return fail(4, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done = true;
    }
  }
  const dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM);
  gemm_tc_kernel<BN, EPI><<<grid, THREADS, GemmSmem<BN>::BYTES, st>>>(ma, mb, g);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "GEMM launch: %s", cudaGetErrorString(e));
  return 0;
}

template <int BN>
int launch_bn(int epi, const CUtensorMap &ma, const CUtensorMap &mb, const GemmArgs &g,
              cudaStream_t st) {
  switch (epi) {
    case EPI_F16: return launch_t<BN, EPI_F16>(ma, mb, g, st);
    case EPI_F32: return launch_t<BN, EPI_F32>(ma, mb, g, st);
    case EPI_F32_RES16: return launch_t<BN, EPI_F32_RES16>(ma, mb, g, st);
    case EPI_SWIGLU: return launch_t<BN, EPI_SWIGLU>(ma, mb, g, st);
    case EPI_F16_RES32: return launch_t<BN, EPI_F16_RES32>(ma, mb, g, st);
    case EPI_ARGMAX: return launch_t<BN, EPI_ARGMAX>(ma, mb, g, st);
    default: return fail(10, "unknown epilogue %d", epi);
  }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

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
  if (int rc = qb200_encode_f16_2d(&p->ma, a, K, M, lda, BK, BM, 1)) return rc;
  if (int rc = qb200_encode_f16_2d(&p->mb, b, K, N, ldb, BK, p->bn, 1)) return rc;
  return 0;
}

int qb200_gemm_run(const GemmPlan &p, int epi, GemmArgs g, cudaStream_t st) {
  g.M = (g.M > 0 && g.M < p.M) ? g.M : p.M;  // fewer rows than planned: the rest stay untouched
  g.N = p.N;
  g.K = p.K;
  g.n_tiles = (p.N + p.bn - 1) / p.bn;
  return p.bn == 128 ? launch_bn<128>(epi, p.ma, p.mb, g, st) : launch_bn<64>(epi, p.ma, p.mb, g, st);
}

int qb200_argmax_reduce(const float *part_val, const int *part_idx, int n_tiles, int rows, int *out,
                        cudaStream_t st) {
  const int wpb = 8;
  argmax_reduce_kernel<<<(rows + wpb - 1) / wpb, 32 * wpb, 0, st>>>(part_val, part_idx, n_tiles,
                                                                   rows, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "argmax launch: %s", cudaGetErrorString(e));
  return 0;
}

extern "C" {

long long qwen_b200_gemm_argmax_workspace(int M, int N) {
  if (M < 1 || N < 16) return 0;
  const int bn = qb200_gemm_bn(M, N);
  const long long tiles = (N + bn - 1) / bn;
  return static_cast<long long>(M) * tiles * 8;
}

int qwen_b200_gemm_f16(int epilogue, const void *a, const void *b, void *out, const void *res,
                       void *workspace, int M, int N, int K, int ldo, void *stream) {
  qb200_clear_error();
  if (a == nullptr || b == nullptr || out == nullptr) return fail(13, "null pointer argument");
  if (epilogue < 0 || epilogue > EPI_ARGMAX) return fail(10, "unknown epilogue %d", epilogue);
  if ((epilogue == EPI_F32_RES16 || epilogue == EPI_F16_RES32) && res == nullptr)
    return fail(13, "this epilogue needs a residual");
  if (epilogue == EPI_ARGMAX && workspace == nullptr) return fail(13, "argmax needs a workspace");
  GemmPlan p{};
  if (int rc = qb200_gemm_make_maps(&p, a, b, M, N, K, K, K)) return rc;
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
  if (int rc = qb200_gemm_run(p, epilogue, g, st)) return rc;
  if (epilogue == EPI_ARGMAX)
    return qb200_argmax_reduce(g.part_val, g.part_idx, n_tiles, M, static_cast<int *>(out), st);
  return 0;
}

}  // extern "C"
