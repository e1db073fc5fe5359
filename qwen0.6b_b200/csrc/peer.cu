// peer.cu - cross-GPU exchange of the vocabulary-sharded lm_head's per-row
// (max logit, index) pairs through peer memory, and the CUDA IPC plumbing it
// needs (include/qwen_b200_batched.h).
//
// No upstream counterpart: upstream evaluates the whole lm_head on one GPU
// (Tools/megakernel/megakernel.cu:1001-1144).  Here each rank stores its pairs
// straight into every rank's receive buffer over NVLink (plain 8-byte stores
// at system scope, no multicast, no library kernel on peer memory) and picks
// the token from its own buffer once every rank's pairs of the call are in.
//
// Receive buffer of every rank: [2][world][rows][2] 8-byte words, half
// (epoch & 1) used by a call: word 0 = fp32 value bits, word 1 = index, each
// with the call's epoch in its high 32 bits.  Alternating halves make reuse
// safe: a rank writes call k+2 into the half that holds call k only after it
// saw every rank's call k+1 pairs, which each rank stores only after it
// finished reading call k.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "host_err.h"
#include "ptx.cuh"
#include "qwen_b200_batched.h"

namespace {

constexpr int MAX_WORLD = 8;

struct PeerPtrs {
  uint64_t *buf[MAX_WORLD];
};

__device__ __forceinline__ void st_sys_u64(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One thread per row.  Stores this rank's pair into slot [rank] of every
// rank's buffer, then waits (bounded) for every rank's pair of this epoch in
// its own buffer and picks the largest value, lowest index among equal ones.
// A wait that gives up writes -1 and records (code 1 | rank | row) in *err.
__global__ void argmax_exchange_kernel(const float *__restrict__ val, const int *__restrict__ idx,
                                       PeerPtrs peers, int world, int rank, int rows, uint32_t epoch,
                                       long long timeout_ns, int *__restrict__ out,
                                       unsigned long long *err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const size_t half = static_cast<size_t>(epoch & 1u) * world * rows * 2;
  const uint64_t tag = static_cast<uint64_t>(epoch) << 32;
  const uint64_t wv = tag | __float_as_uint(val[r]);
  const uint64_t wi = tag | static_cast<uint32_t>(idx[r]);
  for (int q = 0; q < world; ++q) {
    uint64_t *dst = peers.buf[q] + half + (static_cast<size_t>(rank) * rows + r) * 2;
    st_sys_u64(dst, wv);
    st_sys_u64(dst + 1, wi);
  }
  const uint64_t *mine = peers.buf[rank] + half;
  float best = -INFINITY;
  int bi = -1;
  const uint64_t t0 = qb200::globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    const uint64_t *src = mine + (static_cast<size_t>(q) * rows + r) * 2;
    uint64_t a = ld_sys_u64(src), b = ld_sys_u64(src + 1);
    while (static_cast<uint32_t>(a >> 32) != epoch || static_cast<uint32_t>(b >> 32) != epoch) {
      if (static_cast<long long>(qb200::globaltimer_ns() - t0) > timeout_ns) {
        if (err != nullptr)
          atomicCAS(err, 0ull, (1ull << 32) | (static_cast<unsigned long long>(q) << 24) | static_cast<unsigned>(r));
        out[r] = -1;
        return;
      }
      a = ld_sys_u64(src);
      b = ld_sys_u64(src + 1);
    }
    const float v = __uint_as_float(static_cast<uint32_t>(a));
    const int i = static_cast<int>(static_cast<uint32_t>(b));
    if (i < 0) continue;
    if (bi < 0 || v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  out[r] = bi;
}

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return qb200_set_error(code, buf);
}

}  // namespace

extern "C" {

long long qwen_b200_peer_buffer_bytes(int world, int rows) {
  if (world < 1 || world > MAX_WORLD || rows < 1) return 0;
  return 2ll * world * rows * 2 * 8;
}

int qwen_b200_peer_buffer_create(long long bytes, void **ptr, void *ipc_handle) {
  qb200_clear_error();
  if (ptr == nullptr || ipc_handle == nullptr || bytes <= 0) return fail(13, "null pointer or empty buffer");
  *ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // the clear lands before any peer writes
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    return fail(5, "peer buffer of %lld bytes: %s", bytes, cudaGetErrorString(e));
  }
  *ptr = p;
  return 0;
}

int qwen_b200_peer_buffer_open(const void *ipc_handle, void **ptr) {
  qb200_clear_error();
  if (ptr == nullptr || ipc_handle == nullptr) return fail(13, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(6, "opening a peer buffer: %s", cudaGetErrorString(e));
  return 0;
}

int qwen_b200_peer_buffer_close(void *ptr, int opened) {
  qb200_clear_error();
  if (ptr == nullptr) return 0;
  const cudaError_t e = opened ? cudaIpcCloseMemHandle(ptr) : cudaFree(ptr);
  if (e != cudaSuccess) return fail(6, "releasing a peer buffer: %s", cudaGetErrorString(e));
  return 0;
}

int qwen_b200_argmax_exchange(const float *val, const int *idx, void *const *peer_bufs, int world,
                              int rank, int rows, unsigned epoch, long long timeout_ns, int *out,
                              unsigned long long *status, void *stream) {
  qb200_clear_error();
  if (val == nullptr || idx == nullptr || peer_bufs == nullptr || out == nullptr)
    return fail(13, "null pointer argument");
  if (world < 1 || world > MAX_WORLD || rank < 0 || rank >= world || rows < 1)
    return fail(10, "world=%d rank=%d rows=%d out of range (world <= %d)", world, rank, rows, MAX_WORLD);
  if (epoch == 0) return fail(10, "epoch 0 is the cleared buffers' tag");
  PeerPtrs pp{};
  for (int q = 0; q < world; ++q) {
    if (peer_bufs[q] == nullptr) return fail(13, "null peer buffer %d", q);
    pp.buf[q] = static_cast<uint64_t *>(peer_bufs[q]);
  }
  const int threads = 128;
  argmax_exchange_kernel<<<(rows + threads - 1) / threads, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      val, idx, pp, world, rank, rows, epoch, timeout_ns > 0 ? timeout_ns : 2000000000ll, out, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(20, "exchange launch: %s", cudaGetErrorString(e));
  return 0;
}

}  // extern "C"
