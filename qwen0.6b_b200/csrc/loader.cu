// Native safetensors reader: header parsing, validation, host reads and
// device loads with on-device BF16/F32 -> F16 conversion.  C ABI in
// include/qwen_b200_loader.h.
//
// Upstream obtains the same tensors through transformers
// (Model/Qwen06B_architecture.py:122-127: from_pretrained(torch_dtype=float16)
// then state_dict()), i.e. torch's dtype cast applied to the checkpoint's
// tensors.  The cast here is the same IEEE round-to-nearest-even of the exact
// fp32 value, so the loaded fp16 bits equal torch's for every finite input.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "host_err.h"
#include "qwen_b200_loader.h"

namespace {

constexpr int ERR_IO = 20, ERR_FORMAT = 21, ERR_ARG = 22, ERR_CUDA = 23;
constexpr long long MAX_HEADER = 100LL << 20;  // the format's own header limit
constexpr size_t CHUNK = 16u << 20;            // bytes per pinned staging buffer

int fail(int code, const std::string &msg) { return qb200_set_error(code, msg.c_str()); }

// ------------------------------------------------------------------ JSON
// Just enough JSON for a safetensors header: objects, arrays, strings with
// escapes, integers, true/false/null.  Fractions and exponents are rejected
// (no header field uses them).
struct JVal {
  enum Kind { NUL, BOOL, INT, STR, ARR, OBJ } kind = NUL;
  long long i = 0;
  std::string s;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
};

class JParser {
 public:
  JParser(const char *p, size_t n) : p_(p), end_(p + n) {}
  bool parse(JVal &v, std::string &err) {
    if (!value(v, 0)) {
      err = err_.empty() ? "malformed JSON" : err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      err = "trailing bytes after the JSON header";
      return false;
    }
    return true;
  }

 private:
  const char *p_, *end_;
  std::string err_;

  bool bad(const char *m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char *w) {
    const size_t n = strlen(w);
    if (static_cast<size_t>(end_ - p_) < n || memcmp(p_, w, n) != 0) return bad("bad literal");
    p_ += n;
    return true;
  }
  static void put_utf8(std::string &o, uint32_t cp) {
    if (cp < 0x80) {
      o += static_cast<char>(cp);
    } else if (cp < 0x800) {
      o += static_cast<char>(0xC0 | (cp >> 6));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += static_cast<char>(0xE0 | (cp >> 12));
      o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      o += static_cast<char>(0xF0 | (cp >> 18));
      o += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t &cp) {
    if (end_ - p_ < 4) return bad("short \\u escape");
    cp = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p_++;
      cp <<= 4;
      if (c >= '0' && c <= '9') cp |= c - '0';
      else if (c >= 'a' && c <= 'f') cp |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') cp |= c - 'A' + 10;
      else return bad("bad \\u escape");
    }
    return true;
  }
  bool str(std::string &o) {
    if (p_ >= end_ || *p_ != '"') return bad("expected a string");
    ++p_;
    while (p_ < end_ && *p_ != '"') {
      const unsigned char c = static_cast<unsigned char>(*p_++);
      if (c < 0x20) return bad("control character in a string");
      if (c != '\\') {
        o += static_cast<char>(c);
        continue;
      }
      if (p_ >= end_) return bad("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return bad("lone surrogate");
            p_ += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return bad("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return bad("lone surrogate");
          }
          put_utf8(o, cp);
          break;
        }
        default: return bad("unknown escape");
      }
    }
    if (p_ >= end_) return bad("unterminated string");
    ++p_;
    return true;
  }
  bool num(long long &v) {
    bool neg = false;
    if (p_ < end_ && *p_ == '-') {
      neg = true;
      ++p_;
    }
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return bad("expected a number");
    unsigned long long u = 0;
    while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
      const unsigned d = *p_++ - '0';
      if (u > (static_cast<unsigned long long>(INT64_MAX) - d) / 10) return bad("integer overflow");
      u = u * 10 + d;
    }
    if (p_ < end_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) return bad("non-integer number");
    v = neg ? -static_cast<long long>(u) : static_cast<long long>(u);
    return true;
  }
  bool value(JVal &v, int depth) {
    if (depth > 16) return bad("JSON nested too deeply");
    ws();
    if (p_ >= end_) return bad("unexpected end of header");
    const char c = *p_;
    if (c == '{') {
      v.kind = JVal::OBJ;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::pair<std::string, JVal> kv;
        if (!str(kv.first)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return bad("expected ':'");
        ++p_;
        if (!value(kv.second, depth + 1)) return false;
        v.obj.push_back(std::move(kv));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return bad("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = JVal::ARR;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        JVal e;
        if (!value(e, depth + 1)) return false;
        v.arr.push_back(std::move(e));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return bad("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = JVal::STR;
      return str(v.s);
    }
    if (c == 't') {
      v.kind = JVal::BOOL;
      v.i = 1;
      return lit("true");
    }
    if (c == 'f') {
      v.kind = JVal::BOOL;
      return lit("false");
    }
    if (c == 'n') return lit("null");
    v.kind = JVal::INT;
    return num(v.i);
  }
};

const JVal *member(const JVal &o, const char *k) {
  for (const auto &kv : o.obj)
    if (kv.first == k) return &kv.second;
  return nullptr;
}

// ------------------------------------------------------------- conversion
// In place: each element is read and written by the same thread.
__global__ void bf16_to_f16_kernel(uint16_t *p, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long n8 = n / 8;
  uint4 *p8 = reinterpret_cast<uint4 *>(p);
  for (long long j = i; j < n8; j += stride) {
    uint4 v = p8[j];
    uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = __uint_as_float((w[k] & 0xFFFFu) << 16);
      const float hi = __uint_as_float(w[k] & 0xFFFF0000u);
      const __half2 h = __halves2half2(__float2half_rn(lo), __float2half_rn(hi));
      w[k] = *reinterpret_cast<const uint32_t *>(&h);
    }
    p8[j] = v;
  }
  for (long long j = n8 * 8 + i; j < n; j += stride) {
    const __half h = __float2half_rn(__uint_as_float(static_cast<uint32_t>(p[j]) << 16));
    p[j] = __half_as_ushort(h);
  }
}

__global__ void f32_to_f16_kernel(const float *src, __half *dst, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long n4 = n / 4;
  for (long long j = i; j < n4; j += stride) {
    const float4 v = reinterpret_cast<const float4 *>(src)[j];
    const __half2 a = __halves2half2(__float2half_rn(v.x), __float2half_rn(v.y));
    const __half2 b = __halves2half2(__float2half_rn(v.z), __float2half_rn(v.w));
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t *>(&a);
    o.y = *reinterpret_cast<const uint32_t *>(&b);
    reinterpret_cast<uint2 *>(dst)[j] = o;
  }
  for (long long j = n4 * 4 + i; j < n; j += stride) dst[j] = __float2half_rn(src[j]);
}

int grid_for(long long n) {
  const long long want = (n / 8 + 255) / 256;
  return static_cast<int>(want < 1 ? 1 : (want > 148 * 8 ? 148 * 8 : want));
}

}  // namespace

struct QwenStTensor {
  std::string name;
  int dtype = QWEN_ST_OTHER;
  int esize = 0;
  std::vector<long long> shape;
  long long begin = 0, end = 0;  // relative to data_start
};

struct QwenStFile {
  int fd = -1;
  std::string path;
  long long file_size = 0, data_start = 0;
  std::vector<QwenStTensor> t;
  std::map<std::string, int> index;
  std::vector<std::pair<std::string, std::string>> meta;
  void *pinned[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool ev_live[2] = {false, false};
  void *stage = nullptr;  // device staging for F32 sources
  int stage_dev = -1;

  ~QwenStFile() {
    for (int b = 0; b < 2; ++b) {
      if (ev[b] != nullptr) {
        if (ev_live[b]) cudaEventSynchronize(ev[b]);
        cudaEventDestroy(ev[b]);
      }
      if (pinned[b] != nullptr) cudaFreeHost(pinned[b]);
    }
    if (stage != nullptr) {
      int cur = -1;
      cudaGetDevice(&cur);
      cudaSetDevice(stage_dev);
      cudaFree(stage);
      if (cur >= 0) cudaSetDevice(cur);
    }
    if (fd >= 0) close(fd);
  }
};

namespace {

bool read_exact(int fd, void *dst, size_t n, long long off) {
  char *p = static_cast<char *>(dst);
  while (n > 0) {
    const ssize_t r = pread(fd, p, n, off);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    p += r;
    n -= static_cast<size_t>(r);
    off += r;
  }
  return true;
}

int dtype_of(const std::string &s, int *esize) {
  if (s == "F16") { *esize = 2; return QWEN_ST_F16; }
  if (s == "BF16") { *esize = 2; return QWEN_ST_BF16; }
  if (s == "F32") { *esize = 4; return QWEN_ST_F32; }
  static const std::map<std::string, int> other = {
      {"BOOL", 1}, {"U8", 1}, {"I8", 1}, {"F8_E4M3", 1}, {"F8_E5M2", 1}, {"I16", 2}, {"U16", 2},
      {"I32", 4}, {"U32", 4}, {"F64", 8}, {"I64", 8}, {"U64", 8}};
  const auto it = other.find(s);
  *esize = it == other.end() ? 0 : it->second;
  return QWEN_ST_OTHER;
}

int parse_header(QwenStFile &f, const std::string &hdr) {
  JVal root;
  std::string err;
  JParser jp(hdr.data(), hdr.size());
  if (!jp.parse(root, err)) return fail(ERR_FORMAT, f.path + ": header: " + err);
  if (root.kind != JVal::OBJ) return fail(ERR_FORMAT, f.path + ": header is not a JSON object");
  const long long data_size = f.file_size - f.data_start;
  for (const auto &kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind != JVal::OBJ) return fail(ERR_FORMAT, f.path + ": __metadata__ is not an object");
      for (const auto &m : kv.second.obj) {
        if (m.second.kind != JVal::STR)
          return fail(ERR_FORMAT, f.path + ": __metadata__ value of '" + m.first + "' is not a string");
        f.meta.emplace_back(m.first, m.second.s);
      }
      continue;
    }
    const std::string &name = kv.first;
    const JVal &d = kv.second;
    const JVal *dt = d.kind == JVal::OBJ ? member(d, "dtype") : nullptr;
    const JVal *sh = d.kind == JVal::OBJ ? member(d, "shape") : nullptr;
    const JVal *off = d.kind == JVal::OBJ ? member(d, "data_offsets") : nullptr;
    if (dt == nullptr || sh == nullptr || off == nullptr || dt->kind != JVal::STR ||
        sh->kind != JVal::ARR || off->kind != JVal::ARR || off->arr.size() != 2)
      return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' needs dtype, shape and data_offsets[2]");
    QwenStTensor t;
    t.name = name;
    t.dtype = dtype_of(dt->s, &t.esize);
    if (t.esize == 0) return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' has unknown dtype " + dt->s);
    if (sh->arr.size() > 8) return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' has rank > 8");
    long long numel = 1;
    for (const JVal &e : sh->arr) {
      if (e.kind != JVal::INT || e.i < 0)
        return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' has a bad shape entry");
      if (e.i > 0 && numel > (INT64_MAX / t.esize) / e.i)
        return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' is too large");
      numel *= e.i;
      t.shape.push_back(e.i);
    }
    if (off->arr[0].kind != JVal::INT || off->arr[1].kind != JVal::INT)
      return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' has non-integer data_offsets");
    t.begin = off->arr[0].i;
    t.end = off->arr[1].i;
    if (t.begin < 0 || t.end < t.begin || t.end > data_size)
      return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' lies outside the file");
    if (t.end - t.begin != numel * t.esize)
      return fail(ERR_FORMAT, f.path + ": tensor '" + name + "' byte size does not match its shape");
    if (f.index.count(name)) return fail(ERR_FORMAT, f.path + ": duplicate tensor '" + name + "'");
    f.index[name] = static_cast<int>(f.t.size());
    f.t.push_back(std::move(t));
  }
  return 0;
}

int check_index(const QwenStFile *f, int i) {
  if (f == nullptr) return fail(ERR_ARG, "null safetensors handle");
  if (i < 0 || i >= static_cast<int>(f->t.size()))
    return fail(ERR_ARG, "tensor index " + std::to_string(i) + " out of range");
  return 0;
}

int cuda_fail(const char *what, cudaError_t e) {
  return fail(ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int qwen_b200_st_open(const char *path, QwenStFile **out) {
  qb200_clear_error();
  if (path == nullptr || out == nullptr) return fail(ERR_ARG, "null path or handle pointer");
  *out = nullptr;
  std::unique_ptr<QwenStFile> f(new QwenStFile());
  f->path = path;
  f->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f->fd < 0) return fail(ERR_IO, f->path + ": " + strerror(errno));
  struct stat stt;
  if (fstat(f->fd, &stt) != 0) return fail(ERR_IO, f->path + ": " + strerror(errno));
  f->file_size = static_cast<long long>(stt.st_size);
  unsigned char lenb[8];
  if (f->file_size < 8 || !read_exact(f->fd, lenb, 8, 0))
    return fail(ERR_FORMAT, f->path + ": shorter than the 8-byte header length");
  unsigned long long n = 0;
  for (int k = 7; k >= 0; --k) n = (n << 8) | lenb[k];
  if (n > static_cast<unsigned long long>(MAX_HEADER) || static_cast<long long>(n) > f->file_size - 8)
    return fail(ERR_FORMAT, f->path + ": header length " + std::to_string(n) + " is invalid");
  std::string hdr(n, '\0');
  if (n > 0 && !read_exact(f->fd, &hdr[0], n, 8)) return fail(ERR_IO, f->path + ": short read of the header");
  f->data_start = 8 + static_cast<long long>(n);
  if (const int rc = parse_header(*f, hdr)) return rc;
  posix_fadvise(f->fd, 0, 0, POSIX_FADV_SEQUENTIAL);
  *out = f.release();
  return 0;
}

void qwen_b200_st_close(QwenStFile *f) { delete f; }

int qwen_b200_st_num_tensors(const QwenStFile *f) { return f == nullptr ? 0 : static_cast<int>(f->t.size()); }

int qwen_b200_st_find(const QwenStFile *f, const char *name) {
  if (f == nullptr || name == nullptr) return -1;
  const auto it = f->index.find(name);
  return it == f->index.end() ? -1 : it->second;
}

int qwen_b200_st_info(const QwenStFile *f, int i, const char **name, int *dtype, int *ndim,
                      long long shape[8], long long *nbytes) {
  qb200_clear_error();
  if (const int rc = check_index(f, i)) return rc;
  const QwenStTensor &t = f->t[i];
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = static_cast<int>(t.shape.size());
  if (shape)
    for (size_t k = 0; k < t.shape.size(); ++k) shape[k] = t.shape[k];
  if (nbytes) *nbytes = t.end - t.begin;
  return 0;
}

const char *qwen_b200_st_metadata(const QwenStFile *f, const char *key) {
  if (f == nullptr || key == nullptr) return nullptr;
  for (const auto &kv : f->meta)
    if (kv.first == key) return kv.second.c_str();
  return nullptr;
}

int qwen_b200_st_read_host(const QwenStFile *f, int i, void *dst, long long cap) {
  qb200_clear_error();
  if (const int rc = check_index(f, i)) return rc;
  const QwenStTensor &t = f->t[i];
  const long long n = t.end - t.begin;
  if (dst == nullptr && n > 0) return fail(ERR_ARG, "null destination");
  if (cap < n) return fail(ERR_ARG, "destination holds " + std::to_string(cap) + " bytes, tensor '" + t.name +
                                        "' needs " + std::to_string(n));
  if (n > 0 && !read_exact(f->fd, dst, static_cast<size_t>(n), f->data_start + t.begin))
    return fail(ERR_IO, f->path + ": short read of tensor '" + t.name + "'");
  return 0;
}

int qwen_b200_st_load_f16(QwenStFile *f, int i, void *dst, cudaStream_t stream) {
  qb200_clear_error();
  if (const int rc = check_index(f, i)) return rc;
  const QwenStTensor &t = f->t[i];
  if (t.dtype == QWEN_ST_OTHER)
    return fail(ERR_ARG, "tensor '" + t.name + "' is not F16, BF16 or F32");
  const long long n = t.end - t.begin;
  if (n == 0) return 0;
  if (dst == nullptr || reinterpret_cast<uintptr_t>(dst) % 16 != 0)
    return fail(ERR_ARG, "destination of tensor '" + t.name + "' must be a 16-byte aligned device pointer");
  cudaError_t e;
  for (int b = 0; b < 2; ++b) {
    if (f->pinned[b] == nullptr) {
      if ((e = cudaHostAlloc(&f->pinned[b], CHUNK, cudaHostAllocPortable)) != cudaSuccess) {
        f->pinned[b] = nullptr;
        return cuda_fail("cudaHostAlloc", e);
      }
    }
    if (f->ev[b] == nullptr) {
      if ((e = cudaEventCreateWithFlags(&f->ev[b], cudaEventDisableTiming)) != cudaSuccess) {
        f->ev[b] = nullptr;
        return cuda_fail("cudaEventCreate", e);
      }
    }
  }
  if (t.dtype == QWEN_ST_F32) {
    int dev = -1;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail("cudaGetDevice", e);
    if (f->stage != nullptr && f->stage_dev != dev) {
      // Staging belongs to another device: let its copies finish first.
      for (int b = 0; b < 2; ++b)
        if (f->ev_live[b]) cudaEventSynchronize(f->ev[b]);
      cudaSetDevice(f->stage_dev);
      cudaFree(f->stage);
      cudaSetDevice(dev);
      f->stage = nullptr;
    }
    // The staging buffer may still be read by a conversion enqueued on
    // another stream by an earlier call.
    for (int b = 0; b < 2; ++b)
      if (f->ev_live[b]) {
        if ((e = cudaEventSynchronize(f->ev[b])) != cudaSuccess) return cuda_fail("cudaEventSynchronize", e);
        f->ev_live[b] = false;
      }
    if (f->stage == nullptr) {
      if ((e = cudaMalloc(&f->stage, CHUNK)) != cudaSuccess) {
        f->stage = nullptr;
        return cuda_fail("cudaMalloc(staging)", e);
      }
      f->stage_dev = dev;
    }
  }
  char *out = static_cast<char *>(dst);
  long long done = 0;
  for (int k = 0; done < n; ++k) {
    const int b = k & 1;
    const size_t len = static_cast<size_t>(n - done < static_cast<long long>(CHUNK) ? n - done : CHUNK);
    if (f->ev_live[b]) {
      if ((e = cudaEventSynchronize(f->ev[b])) != cudaSuccess) return cuda_fail("cudaEventSynchronize", e);
      f->ev_live[b] = false;
    }
    if (!read_exact(f->fd, f->pinned[b], len, f->data_start + t.begin + done))
      return fail(ERR_IO, f->path + ": short read of tensor '" + t.name + "'");
    if (t.dtype == QWEN_ST_F32) {
      if ((e = cudaMemcpyAsync(f->stage, f->pinned[b], len, cudaMemcpyHostToDevice, stream)) != cudaSuccess)
        return cuda_fail("cudaMemcpyAsync", e);
      const long long elems = static_cast<long long>(len / 4);
      f32_to_f16_kernel<<<grid_for(elems), 256, 0, stream>>>(static_cast<const float *>(f->stage),
                                                            reinterpret_cast<__half *>(out + done / 2), elems);
    } else {
      if ((e = cudaMemcpyAsync(out + done, f->pinned[b], len, cudaMemcpyHostToDevice, stream)) != cudaSuccess)
        return cuda_fail("cudaMemcpyAsync", e);
      if (t.dtype == QWEN_ST_BF16) {
        const long long elems = static_cast<long long>(len / 2);
        bf16_to_f16_kernel<<<grid_for(elems), 256, 0, stream>>>(reinterpret_cast<uint16_t *>(out + done), elems);
      }
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail("conversion kernel launch", e);
    if ((e = cudaEventRecord(f->ev[b], stream)) != cudaSuccess) return cuda_fail("cudaEventRecord", e);
    f->ev_live[b] = true;
    done += static_cast<long long>(len);
  }
  return 0;
}

}  // extern "C"
