// Token sampling over fp32 logits rows: temperature, top-k, top-p, Gumbel-max
// draws from a Philox-4x32-10 stream.  C ABI in include/qwen_b200_sample.h
// (semantics there).  One 1024-thread CTA per row.
//
// Thresholds are exact radix selections on the order-preserving 32-bit key of
// z = logit / temperature, three digit levels (bits 31..21, 20..10, 9..0):
//   top-k: count histogram, find the bin holding the k-th largest key;
//   top-p: softmax-mass histogram of the top-k survivors, find the bin where
//          the mass accumulated from the top first reaches top_p * Z.
// Level 0 reads the row; the elements of the boundary bin are collected into
// shared memory (when they fit) and levels 1-2 run there, otherwise they read
// the row again with the bin's prefix as a filter.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#include "host_err.h"
#include "qwen_b200_sample.h"

namespace {

constexpr int NT = 1024;
constexpr int NW = NT / 32;
constexpr int NBIN = 2048;
constexpr int CAP = 8192;  // boundary-bin elements kept in shared memory

struct SampleArgs {
  const float *logits;
  long long ld;
  int vocab;
  float temperature;
  int top_k;
  float top_p;
  uint32_t seed_lo, seed_hi, off_lo, off_hi;
  const int *row_seq, *row_pos;  // optional per-row stream keys
  int *out;
  float *kept_min;
};

struct SampleSmem {
  uint32_t cnt[NBIN];
  float mass[NBIN];
  uint32_t cand_key[CAP];
  float cand_w[CAP];
  int cand_i[CAP];  // element indices of a window list
  uint32_t n_cand;
  int found;
  float before_f;
  uint32_t before_u;
  float red_f[NW];
  int red_i[NW];
};

// Order-preserving map float -> uint32 (larger float, larger key) and back.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return b ^ ((b >> 31) ? 0xffffffffu : 0x80000000u);
}
__device__ __forceinline__ float kval(uint32_t k) {
  return __uint_as_float((k >> 31) ? (k ^ 0x80000000u) : ~k);
}

// Digit of `key` at level 0/1/2 and the key bits above it.
__device__ __forceinline__ uint32_t digit(uint32_t key, int level) {
  return level == 0 ? key >> 21 : (level == 1 ? (key >> 10) & 2047u : key & 1023u);
}
__device__ __forceinline__ uint32_t above(uint32_t key, int level) {
  return level == 0 ? 0u : (level == 1 ? key >> 21 : key >> 10);
}
__device__ __forceinline__ int nbins(int level) { return level == 2 ? 1024 : 2048; }
__device__ __forceinline__ uint32_t compose(uint32_t prefix, int level, uint32_t d) {
  return level == 0 ? d : (level == 1 ? (prefix << 11) | d : (prefix << 10) | d);
}

// Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): 10 rounds of the
// multiply-xor bijection with a Weyl-sequence key schedule.
__device__ __forceinline__ uint4 philox(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// u in (0, 1) from 24 random bits; Gumbel noise -log(-log u).
__device__ __forceinline__ float gumbel(uint32_t x) {
  const float u = (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

__device__ __forceinline__ float block_max(SampleSmem &s, float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) s.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = s.red_f[0];
  for (int i = 1; i < NW; ++i) m = fmaxf(m, s.red_f[i]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ float block_sum(SampleSmem &s, float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) s.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < NW; ++i) t += s.red_f[i];
  __syncthreads();
  return t;
}

// (value, index) argmax, lowest index among equal values.
__device__ __forceinline__ void better(float &v, int &i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}
__device__ __forceinline__ int block_argmax(SampleSmem &s, float v, int i) {
  for (int o = 16; o > 0; o >>= 1) better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
  if ((threadIdx.x & 31) == 0) {
    s.red_f[threadIdx.x >> 5] = v;
    s.red_i[threadIdx.x >> 5] = i;
  }
  __syncthreads();
  float bv = s.red_f[0];
  int bi = s.red_i[0];
  for (int w = 1; w < NW; ++w) better(bv, bi, s.red_f[w], s.red_i[w]);
  __syncthreads();
  return bi;
}

// Visits every element of the row as (index, z, key), four consecutive
// elements per thread and round (one Philox draw covers the four).
template <class F>
__device__ __forceinline__ void for_row(const SampleArgs &a, const float *lg, F f) {
  const int V = a.vocab;
  for (int g = threadIdx.x; 4 * g < V; g += NT) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * g + j;
      if (i < V) {
        const float z = a.temperature > 0.f ? __fdiv_rn(lg[i], a.temperature) : lg[i];
        f(i, z, fkey(z));
      }
    }
  }
}

// Finds, scanning bins from the top (largest keys) down, the first non-empty
// bin whose cumulative value (counts, or masses when MASS) reaches `target`;
// returns it and leaves the cumulative value of the bins above it in
// s.before_u / s.before_f.
template <bool MASS>
__device__ int find_bin(SampleSmem &s, int nb, float target_f, uint32_t target_u) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Thread t owns descending positions 2t, 2t+1 (bin nb-1-r).
  float vf[2] = {0.f, 0.f};
  uint32_t vu[2] = {0u, 0u}, c[2] = {0u, 0u};
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int r = 2 * tid + q;
    if (r < nb) {
      const int b = nb - 1 - r;
      c[q] = s.cnt[b];
      vf[q] = s.mass[b];
      vu[q] = s.cnt[b];
    }
  }
  if (tid == 0) s.found = 0x7fffffff;
  // Inclusive scan of the pair sums over the block.
  float pf = vf[0] + vf[1];
  uint32_t pu = vu[0] + vu[1];
  float xf = pf;
  uint32_t xu = pu;
  for (int o = 1; o < 32; o <<= 1) {
    const float yf = __shfl_up_sync(0xffffffffu, xf, o);
    const uint32_t yu = __shfl_up_sync(0xffffffffu, xu, o);
    if (lane >= o) {
      xf += yf;
      xu += yu;
    }
  }
  __shared__ float wf[NW];
  __shared__ uint32_t wu[NW];
  if (lane == 31) {
    wf[warp] = xf;
    wu[warp] = xu;
  }
  __syncthreads();
  if (warp == 0) {
    float a = lane < NW ? wf[lane] : 0.f;
    uint32_t b = lane < NW ? wu[lane] : 0u;
    for (int o = 1; o < 32; o <<= 1) {
      const float ya = __shfl_up_sync(0xffffffffu, a, o);
      const uint32_t yb = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) {
        a += ya;
        b += yb;
      }
    }
    if (lane < NW) {
      wf[lane] = a;
      wu[lane] = b;
    }
  }
  __syncthreads();
  float bf = xf - pf + (warp > 0 ? wf[warp - 1] : 0.f);
  uint32_t bu = xu - pu + (warp > 0 ? wu[warp - 1] : 0u);
  int hit = 0x7fffffff;
  float hit_bf = 0.f;
  uint32_t hit_bu = 0u;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int r = 2 * tid + q;
    const bool reach = MASS ? (bf + vf[q] >= target_f) : (bu + vu[q] >= target_u);
    if (r < nb && c[q] > 0 && reach && hit == 0x7fffffff) {
      hit = r;
      hit_bf = bf;
      hit_bu = bu;
    }
    bf += vf[q];
    bu += vu[q];
  }
  if (hit != 0x7fffffff) atomicMin(&s.found, hit);
  __syncthreads();
  const int r = s.found;
  if (hit == r) {
    s.before_f = hit_bf;
    s.before_u = hit_bu;
  }
  __syncthreads();
  return r == 0x7fffffff ? -1 : nb - 1 - r;
}

// Exact key of the boundary element: the k-th largest key (top-k, counts)
// or the last key of the top-p set (MASS), among the elements with key >=
// floor_key.  w(z) is the element's softmax weight (MASS only).
template <bool MASS, class W>
__device__ uint32_t select_key(SampleSmem &s, const SampleArgs &a, const float *lg, uint32_t floor_key,
                               float target_f, uint32_t target_u, W w) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0;
  bool in_list = false;
  for (int level = 0; level < 3; ++level) {
    const int nb = nbins(level);
    for (int b = tid; b < nb; b += NT) {
      s.cnt[b] = 0u;
      s.mass[b] = 0.f;
    }
    __syncthreads();
    auto add = [&](uint32_t key, float wt) {
      const uint32_t d = digit(key, level);
      atomicAdd(&s.cnt[d], 1u);
      if (MASS) atomicAdd(&s.mass[d], wt);
    };
    if (in_list) {
      const int n = static_cast<int>(s.n_cand);
      for (int i = tid; i < n; i += NT) add(s.cand_key[i], s.cand_w[i]);
    } else {
      for_row(a, lg, [&](int, float z, uint32_t key) {
        if (key >= floor_key && above(key, level) == prefix) add(key, MASS ? w(z) : 0.f);
      });
    }
    __syncthreads();
    const int bin = find_bin<MASS>(s, nb, target_f, target_u);
    if (bin < 0) return floor_key;  // rounding left the target unreached: keep everything
    target_f -= s.before_f;
    target_u -= s.before_u;
    const uint32_t n_bin = s.cnt[bin];
    prefix = compose(prefix, level, static_cast<uint32_t>(bin));
    if (level == 2) return prefix;
    // Collect the boundary bin's elements for the next levels when they fit.
    if (!in_list && n_bin <= static_cast<uint32_t>(CAP)) {
      __syncthreads();
      if (tid == 0) s.n_cand = 0u;
      __syncthreads();
      const int lvl = level;
      for_row(a, lg, [&](int, float z, uint32_t key) {
        if (key >= floor_key && (lvl == 0 ? key >> 21 : key >> 10) == prefix) {
          const uint32_t slot = atomicAdd(&s.n_cand, 1u);
          if (slot < static_cast<uint32_t>(CAP)) {
            s.cand_key[slot] = key;
            s.cand_w[slot] = MASS ? w(z) : 0.f;
          }
        }
      });
      __syncthreads();
      in_list = true;
    }
    if (in_list) {
      // Compact the list to the chosen bin (a no-op right after collecting).
      const int n = static_cast<int>(s.n_cand);
      __syncthreads();
      if (tid == 0) s.found = 0;
      __syncthreads();
      // Two-step compaction through registers (n <= CAP = 8 per thread).
      uint32_t kk[CAP / NT];
      float ww[CAP / NT];
      int m = 0;
      for (int i = tid; i < n; i += NT) {
        const uint32_t key = s.cand_key[i];
        const uint32_t pre = level == 0 ? key >> 21 : key >> 10;
        if (pre == prefix) {
          kk[m] = key;
          ww[m] = s.cand_w[i];
          ++m;
        }
      }
      __syncthreads();
      const int base = atomicAdd(&s.found, m);
      for (int q = 0; q < m; ++q) {
        s.cand_key[base + q] = kk[q];
        s.cand_w[base + q] = ww[q];
      }
      __syncthreads();
      if (tid == 0) s.n_cand = static_cast<uint32_t>(s.found);
      __syncthreads();
    }
  }
  return prefix;
}

// Random stream of a row: (row or row_seq[row], offset + row_pos[row]).
__device__ __forceinline__ uint4 row_draw(const SampleArgs &a, int row, uint32_t group) {
  const uint32_t stream_id = static_cast<uint32_t>(a.row_seq != nullptr ? a.row_seq[row] : row);
  const uint32_t stream_pos = static_cast<uint32_t>(a.row_pos != nullptr ? a.row_pos[row] : 0);
  return philox(make_uint4(group, stream_id, a.off_lo + stream_pos, a.off_hi), a.seed_lo, a.seed_hi);
}
__device__ __forceinline__ uint32_t word(const uint4 r, int j) {
  return j == 0 ? r.x : (j == 1 ? r.y : (j == 2 ? r.z : r.w));
}

__device__ __forceinline__ uint32_t block_sum_u(SampleSmem &s, uint32_t v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) s.red_i[threadIdx.x >> 5] = static_cast<int>(v);
  __syncthreads();
  uint32_t t = 0u;
  for (int i = 0; i < NW; ++i) t += static_cast<uint32_t>(s.red_i[i]);
  __syncthreads();
  return t;
}

// Window pre-filter.  For a ladder of windows [zmax - D, zmax] the element
// count and softmax mass are taken in one pass; the smallest window that must
// contain the kept set (top-k: at least k elements, so every element of the
// k-th largest key's group; top-p alone: at least top_p of the total mass) is
// collected into a list of at most CAP elements, and the exact selections and
// the draw run on that list.  The kept set is a prefix of the descending order,
// and so is every window, which is why the selection on the list equals the
// selection on the row.
constexpr int NJ = 8;  // window ladder: D = 0.5 * 2^j (j < NJ - 1), then everything
__device__ __forceinline__ float window_d(int j) { return j < NJ - 1 ? 0.5f * static_cast<float>(1 << j) : INFINITY; }

// Smallest window index whose (count, mass) totals admit the kept set and
// whose count fits the list, or -1.
__device__ __forceinline__ int pick_window(const SampleArgs &a, const uint32_t *ct, const float *mt, float Zt) {
  const bool use_k = a.top_k > 0 && a.top_k < a.vocab;
  const bool use_p = a.top_p < 1.f;
  for (int j = 0; j < NJ; ++j) {
    const bool ok = (use_k ? ct[j] >= static_cast<uint32_t>(a.top_k) : (!use_p || mt[j] >= a.top_p * Zt)) &&
                    ct[j] <= static_cast<uint32_t>(CAP);
    if (ok && ct[j] > 0u) return j;
  }
  return -1;
}

// Exact radix selection (as select_key) over the n-element list in
// s.cand_key / s.cand_w (z), restricted to keys >= floor_key.
template <bool MASS>
__device__ uint32_t list_select(SampleSmem &s, int n, uint32_t floor_key, float target_f, uint32_t target_u,
                                float zmax) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0;
  for (int level = 0; level < 3; ++level) {
    const int nb = nbins(level);
    for (int b = tid; b < nb; b += NT) {
      s.cnt[b] = 0u;
      s.mass[b] = 0.f;
    }
    __syncthreads();
    for (int i = tid; i < n; i += NT) {
      const uint32_t key = s.cand_key[i];
      if (key >= floor_key && above(key, level) == prefix) {
        const uint32_t d = digit(key, level);
        atomicAdd(&s.cnt[d], 1u);
        if (MASS) atomicAdd(&s.mass[d], expf(s.cand_w[i] - zmax));
      }
    }
    __syncthreads();
    const int bin = find_bin<MASS>(s, nb, target_f, target_u);
    if (bin < 0) return floor_key;
    target_f -= s.before_f;
    target_u -= s.before_u;
    prefix = compose(prefix, level, static_cast<uint32_t>(bin));
  }
  return prefix;
}

// Top-k / top-p thresholds and the Gumbel-max draw on the n-element window
// list (keys, z and indices in s); writes the token and kept_min.  Z_all is
// the softmax mass of the whole row (used when top-k is off).
__device__ void finish_list(SampleSmem &s, const SampleArgs &a, int row, int n, float zmax, float Z_all) {
  const int tid = threadIdx.x;
  const bool use_k = a.top_k > 0 && a.top_k < a.vocab;
  const bool use_p = a.top_p < 1.f;
  uint32_t floor_key = 0u;
  if (use_k) floor_key = list_select<false>(s, n, 0u, 0.f, static_cast<uint32_t>(a.top_k), zmax);
  if (use_p) {
    float Z = Z_all;
    if (use_k) {
      float part = 0.f;
      for (int i = tid; i < n; i += NT)
        if (s.cand_key[i] >= floor_key) part += expf(s.cand_w[i] - zmax);
      Z = block_sum(s, part);
    }
    floor_key = list_select<true>(s, n, floor_key, a.top_p * Z, 0u, zmax);
  }
  if (floor_key == 0u) {  // rounding left the top-p target unreached: the whole list is kept
    float m = -INFINITY;
    for (int i = tid; i < n; i += NT) m = fmaxf(m, -s.cand_w[i]);
    floor_key = fkey(-block_max(s, m));
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < n; i += NT) {
    if (s.cand_key[i] >= floor_key) {
      const int idx = s.cand_i[i];
      better(bv, bi, s.cand_w[i] + gumbel(word(row_draw(a, row, static_cast<uint32_t>(idx >> 2)), idx & 3)), idx);
    }
  }
  const int tok = block_argmax(s, bv, bi);
  if (tid == 0) {
    a.out[row] = tok;
    if (a.kept_min != nullptr) a.kept_min[row] = floor_key == 0u ? -INFINITY : kval(floor_key);
  }
}

// One row by one CTA, reading the row from global memory for every pass.
__device__ void sample_row(SampleSmem &s, const SampleArgs &a, int row) {
  const int tid = threadIdx.x;
  const float *lg = a.logits + static_cast<size_t>(row) * a.ld;
  const int V = a.vocab;

  if (a.temperature <= 0.f || a.top_k == 1) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for_row(a, lg, [&](int i, float z, uint32_t) { better(bv, bi, z, i); });
    const int tok = block_argmax(s, bv, bi);
    if (tid == 0) {
      a.out[row] = tok;
      if (a.kept_min != nullptr)
        a.kept_min[row] = a.temperature > 0.f ? __fdiv_rn(lg[tok], a.temperature) : lg[tok];
    }
    return;
  }

  const bool use_k = a.top_k > 0 && a.top_k < V;
  const bool use_p = a.top_p < 1.f;
  uint32_t floor_key = 0u;
  float zmax = -INFINITY;
  if (use_k || use_p) {
    float m = -INFINITY;
    for_row(a, lg, [&](int, float z, uint32_t) { m = fmaxf(m, z); });
    zmax = block_max(s, m);
    // Window pre-filter: one pass for the ladder's counts and masses, one to
    // collect the chosen window; the selections then run on the list.
    uint32_t cnt[NJ];
    float mass[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      cnt[j] = 0u;
      mass[j] = 0.f;
    }
    for_row(a, lg, [&](int, float z, uint32_t) {
      const float d = zmax - z;
      const float w = expf(-d);
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        if (d <= window_d(j)) {
          ++cnt[j];
          mass[j] += w;
        }
      }
    });
    uint32_t ct[NJ];
    float mt[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      mt[j] = block_sum(s, mass[j]);
      ct[j] = block_sum_u(s, cnt[j]);
    }
    const int js = pick_window(a, ct, mt, mt[NJ - 1]);
    if (js >= 0) {
      const float dsel = window_d(js);
      if (tid == 0) s.n_cand = 0u;
      __syncthreads();
      for_row(a, lg, [&](int i, float z, uint32_t key) {
        if (zmax - z <= dsel) {
          const uint32_t slot = atomicAdd(&s.n_cand, 1u);
          s.cand_key[slot] = key;
          s.cand_w[slot] = z;
          s.cand_i[slot] = i;
        }
      });
      __syncthreads();
      finish_list(s, a, row, static_cast<int>(s.n_cand), zmax, mt[NJ - 1]);
      return;
    }
  }
  if (use_k)
    floor_key = select_key<false>(s, a, lg, 0u, 0.f, static_cast<uint32_t>(a.top_k),
                                  [](float) { return 0.f; });
  if (use_p) {
    float part = 0.f;
    for_row(a, lg, [&](int, float z, uint32_t key) {
      if (key >= floor_key) part += expf(z - zmax);
    });
    const float Z = block_sum(s, part);
    floor_key = select_key<true>(s, a, lg, floor_key, a.top_p * Z, 0u,
                                 [&](float z) { return expf(z - zmax); });
  }

  // Gumbel-max over the kept set.
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int g = tid; 4 * g < V; g += NT) {
    const uint4 r = row_draw(a, row, static_cast<uint32_t>(g));
    const uint32_t rv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * g + j;
      if (i < V) {
        const float z = __fdiv_rn(lg[i], a.temperature);
        if (fkey(z) >= floor_key) better(bv, bi, z + gumbel(rv[j]), i);
      }
    }
  }
  const int tok = block_argmax(s, bv, bi);
  if (tid == 0) {
    a.out[row] = tok;
    if (a.kept_min != nullptr) a.kept_min[row] = floor_key == 0u ? -INFINITY : kval(floor_key);
  }
}

__global__ void __launch_bounds__(NT, 1) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  sample_row(*reinterpret_cast<SampleSmem *>(smem_raw), a, blockIdx.x);
}

// ------------------------------------------------------ cluster-per-row path
// A cluster of CL CTAs holds one row in shared memory (a slice of at most
// SLICE elements per CTA, read from global memory once).  The CTAs publish
// per-slice statistics (max, and for a ladder of windows [zmax - D, zmax]
// the element count and softmax mass); every CTA derives the same smallest
// window that must contain the kept set (top-k: at least k elements; top-p
// alone: at least top_p of the total mass), collects its window elements, and
// rank 0 gathers them through distributed shared memory and runs the exact
// selection and the draw on that list.  The kept set, the random stream and
// hence the token are those of the one-CTA path.  A row whose window would
// not fit the list falls back to the one-CTA path on rank 0.
constexpr int CL = 8;
constexpr int SLICE = 19200;

struct ClusterSmem {
  SampleSmem hs;       // histograms; hs.cand_key / cand_w / cand_i hold the list's key, z and index
  float zs[SLICE];     // this CTA's slice of z
  float st_max, st_min, st_val;
  int st_idx;
  uint32_t st_cnt[NJ];
  float st_mass[NJ];
  float st_Z;
  uint32_t st_n;       // window elements collected by this CTA
  float zmax;
  int jsel;
  uint32_t red_u[NW];
};

__global__ void __launch_bounds__(NT, 1) sample_cluster_kernel(SampleArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  ClusterSmem &c = *reinterpret_cast<ClusterSmem *>(smem_raw);
  const int rank = static_cast<int>(cluster.block_rank()), row = blockIdx.y, tid = threadIdx.x;
  const int V = a.vocab;
  const int slice = ((V + CL - 1) / CL + 3) & ~3;  // multiple of 4: draw groups stay in one CTA
  const int lo = min(V, rank * slice), n = min(V, lo + slice) - lo;
  const float *lg = a.logits + static_cast<size_t>(row) * a.ld + lo;
  const bool greedy = a.temperature <= 0.f || a.top_k == 1;
  float mx = -INFINITY, mn = INFINITY, bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < n; i += NT) {
    const float z = greedy ? lg[i] : __fdiv_rn(lg[i], a.temperature);
    c.zs[i] = z;
    mx = fmaxf(mx, z);
    mn = fminf(mn, z);
    if (greedy) better(bv, bi, z, lo + i);
  }
  mx = block_max(c.hs, mx);
  mn = -block_max(c.hs, -mn);
  const bool all = !greedy && (a.top_k == 0 || a.top_k >= V) && a.top_p >= 1.f;
  if (all) {  // temperature only: Gumbel-max over the whole slice
    for (int g = tid; 4 * g < n; g += NT) {
      const uint4 r = row_draw(a, row, static_cast<uint32_t>((lo >> 2) + g));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * g + j;
        if (i < n) better(bv, bi, c.zs[i] + gumbel(word(r, j)), lo + i);
      }
    }
  }
  if (greedy || all) {
    const int idx = block_argmax(c.hs, bv, bi);
    if (tid == 0) {
      // The winner's score, recomputed from its index (same arithmetic as above).
      float v = -INFINITY;
      if (idx >= lo && idx < lo + n)
        v = greedy ? c.zs[idx - lo]
                   : c.zs[idx - lo] + gumbel(word(row_draw(a, row, static_cast<uint32_t>(idx >> 2)), idx & 3));
      c.st_val = v;
      c.st_idx = idx;
      c.st_min = mn;
    }
    cluster.sync();
    if (rank == 0 && tid == 0) {
      float best = -INFINITY, lowest = INFINITY;
      int bidx = 0x7fffffff;
      for (int r = 0; r < CL; ++r) {
        ClusterSmem *o = cluster.map_shared_rank(&c, r);
        better(best, bidx, o->st_val, o->st_idx);
        lowest = fminf(lowest, o->st_min);
      }
      a.out[row] = bidx;
      if (a.kept_min != nullptr) a.kept_min[row] = greedy ? best : lowest;
    }
    cluster.sync();
    return;
  }
  // Window statistics of this slice.
  if (tid == 0) c.st_max = mx;
  cluster.sync();
  if (tid == 0) {
    float zm = -INFINITY;
    for (int r = 0; r < CL; ++r) zm = fmaxf(zm, cluster.map_shared_rank(&c, r)->st_max);
    c.zmax = zm;
  }
  __syncthreads();
  const float zmax = c.zmax;
  uint32_t cnt[NJ];
  float mass[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    cnt[j] = 0u;
    mass[j] = 0.f;
  }
  for (int i = tid; i < n; i += NT) {
    const float d = zmax - c.zs[i];
    const float w = expf(-d);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      if (d <= window_d(j)) {
        ++cnt[j];
        mass[j] += w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float m = block_sum(c.hs, mass[j]);
    uint32_t u = cnt[j];
    for (int o = 16; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
    if ((tid & 31) == 0) c.red_u[tid >> 5] = u;
    __syncthreads();
    if (tid == 0) {
      uint32_t t = 0;
      for (int w = 0; w < NW; ++w) t += c.red_u[w];
      c.st_cnt[j] = t;
      c.st_mass[j] = m;
    }
    __syncthreads();
  }
  cluster.sync();
  if (tid == 0) {
    uint32_t ct[NJ];
    float mt[NJ];
    for (int j = 0; j < NJ; ++j) {
      ct[j] = 0u;
      mt[j] = 0.f;
      for (int r = 0; r < CL; ++r) {
        ClusterSmem *o = cluster.map_shared_rank(&c, r);
        ct[j] += o->st_cnt[j];
        mt[j] += o->st_mass[j];
      }
    }
    c.jsel = pick_window(a, ct, mt, mt[NJ - 1]);
    c.st_Z = mt[NJ - 1];
  }
  __syncthreads();
  const int js = c.jsel;
  if (js < 0) {  // window does not fit the list: the one-CTA path on rank 0
    cluster.sync();
    if (rank == 0) sample_row(c.hs, a, row);
    return;
  }
  // Collect this slice's window elements.
  if (tid == 0) c.st_n = 0u;
  __syncthreads();
  const float dsel = window_d(js);
  for (int i = tid; i < n; i += NT) {
    const float z = c.zs[i];
    if (zmax - z <= dsel) {
      const uint32_t slot = atomicAdd(&c.st_n, 1u);
      c.hs.cand_key[slot] = fkey(z);
      c.hs.cand_w[slot] = z;
      c.hs.cand_i[slot] = lo + i;
    }
  }
  cluster.sync();
  // Rank 0 appends the other ranks' lists to its own.
  int total = 0;
  if (rank == 0) {
    total = static_cast<int>(c.st_n);
    for (int r = 1; r < CL; ++r) {
      ClusterSmem *o = cluster.map_shared_rank(&c, r);
      const int m = static_cast<int>(o->st_n);
      for (int i = tid; i < m; i += NT) {
        c.hs.cand_key[total + i] = o->hs.cand_key[i];
        c.hs.cand_w[total + i] = o->hs.cand_w[i];
        c.hs.cand_i[total + i] = o->hs.cand_i[i];
      }
      total += m;
    }
  }
  cluster.sync();  // the other ranks' shared memory is no longer read
  if (rank != 0) return;
  finish_list(c.hs, a, row, total, zmax, c.st_Z);
}

int g_attr_done[64];
int g_cluster_ok[64];  // 0 unknown, 1 usable, -1 not

}  // namespace

extern "C" int qwen_b200_sample(const float *logits, long long ld, int rows, int vocab, float temperature,
                                int top_k, float top_p, unsigned long long seed, unsigned long long offset,
                                const int *row_seq, const int *row_pos, int *out_tokens, float *kept_min,
                                void *stream) {
  qb200_clear_error();
  char msg[256];
  if (rows < 0 || vocab < 1 || ld < vocab) {
    snprintf(msg, sizeof msg, "bad shape: rows=%d vocab=%d ld=%lld", rows, vocab, ld);
    return qb200_set_error(40, msg);
  }
  if (!(temperature >= 0.f) || top_k < 0 || !(top_p > 0.f && top_p <= 1.f)) {
    snprintf(msg, sizeof msg, "bad sampling parameters: temperature=%g top_k=%d top_p=%g (need temperature >= 0, "
             "top_k >= 0, 0 < top_p <= 1)", temperature, top_k, top_p);
    return qb200_set_error(40, msg);
  }
  if (rows == 0) return 0;
  if (logits == nullptr || out_tokens == nullptr) return qb200_set_error(40, "null logits or output pointer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return qb200_set_error(41, "cudaGetDevice failed");
  const size_t smem = sizeof(SampleSmem);
  if (!g_attr_done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) {
      snprintf(msg, sizeof msg, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return qb200_set_error(41, msg);
    }
    g_attr_done[dev] = 1;
  }
  SampleArgs a;
  a.logits = logits;
  a.ld = ld;
  a.vocab = vocab;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.seed_lo = static_cast<uint32_t>(seed);
  a.seed_hi = static_cast<uint32_t>(seed >> 32);
  a.off_lo = static_cast<uint32_t>(offset);
  a.off_hi = static_cast<uint32_t>(offset >> 32);
  a.row_seq = row_seq;
  a.row_pos = row_pos;
  a.out = out_tokens;
  a.kept_min = kept_min;
  // Cluster-per-row path when the row fits CL slices, clusters of CL such CTAs
  // can be co-scheduled on this device and the rows are few; else one CTA per row.
  const int slice = ((vocab + CL - 1) / CL + 3) & ~3;
  if (slice <= SLICE && g_cluster_ok[dev] == 0) {
    const int csmem = static_cast<int>(sizeof(ClusterSmem));
    cudaError_t ce = cudaFuncSetAttribute(sample_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, csmem);
    int nclusters = 0;
    if (ce == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(CL, 1, 1);
      cfg.blockDim = dim3(NT, 1, 1);
      cfg.dynamicSmemBytes = csmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = CL;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      ce = cudaOccupancyMaxActiveClusters(&nclusters, sample_cluster_kernel, &cfg);
    }
    g_cluster_ok[dev] = (ce == cudaSuccess && nclusters > 0) ? 1 : -1;
    cudaGetLastError();  // a refused probe leaves no sticky error
  }
  cudaError_t e;
  // 18 clusters of 8 run at a time on 148 SMs and one takes ~35 us, while the
  // one-CTA path runs 148 rows at a time in ~200 us: clusters up to ~100 rows.
  if (slice <= SLICE && g_cluster_ok[dev] == 1 && rows <= 96) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, static_cast<unsigned>(rows), 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = sizeof(ClusterSmem);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, sample_cluster_kernel, a);
  } else {
    sample_kernel<<<rows, NT, smem, static_cast<cudaStream_t>(stream)>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    snprintf(msg, sizeof msg, "sample kernel launch: %s", cudaGetErrorString(e));
    return qb200_set_error(41, msg);
  }
  return 0;
}

extern "C" void qwen_b200_sample_set_cluster(int enable) {
  for (int d = 0; d < 64; ++d)
    if (!enable) g_cluster_ok[d] = -1;
    else if (g_cluster_ok[d] == -1) g_cluster_ok[d] = 0;
}
