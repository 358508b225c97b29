// safetensors.cpp -- reader of safetensors checkpoints for the per-layer
// packed-weight binding (the MLX layout is used as stored: uint32 packed
// words, bf16 scales / biases, stacked experts [E, N, ...]).
//
// Behaviour follows the reference's header reader
// (Sources/MLXFastCore/Safetensors.swift:75-180): an 8-byte little-endian
// header length, a JSON object of tensors {dtype, shape, data_offsets} plus
// an optional "__metadata__" object; the header is limited to 100,000,000
// bytes; offsets must be ordered and inside the data section. The file is
// mapped read-only; tensors are copied to host memory or to device memory
// (cudaMemcpyAsync from the mapping on the caller's stream, synchronised
// before returning so the mapping may be closed afterwards).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "host.hpp"

namespace b2q {
namespace {

constexpr uint64_t kMaxHeader = 100000000ull;

struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets inside the data section
};

struct StFile {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  const uint8_t* data = nullptr;  // start of the data section
  uint64_t data_bytes = 0;
  std::map<std::string, TensorInfo> tensors;
  std::vector<std::string> names;  // in file order of the header
};

// ---- a small JSON reader: the subset a safetensors header uses ----------------
struct Json {
  const char* p;
  const char* e;
  bool fail = false;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return fail = true, false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return fail = true, false;
        char q = *p++;
        switch (q) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {  // keep BMP code points as UTF-8
            if (e - p < 4) return fail = true, false;
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else return fail = true, false;
            }
            if (v < 0x80) out += (char)v;
            else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 0x3F)); }
            else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 0x3F)); out += (char)(0x80 | (v & 0x3F)); }
            break;
          }
          default: return fail = true, false;
        }
      } else {
        out += c;
      }
    }
    if (p >= e) return fail = true, false;
    ++p;
    return true;
  }
  // non-negative integers only (shapes and offsets)
  bool integer(int64_t& v) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return fail = true, false;
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      if (v > (INT64_MAX - 9) / 10) return fail = true, false;
      v = v * 10 + (*p++ - '0');
    }
    if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return fail = true, false;
    return true;
  }
  bool int_array(std::vector<int64_t>& out) {
    out.clear();
    if (!eat('[')) return fail = true, false;
    if (eat(']')) return true;
    do {
      int64_t v;
      if (!integer(v)) return false;
      out.push_back(v);
    } while (eat(','));
    if (!eat(']')) return fail = true, false;
    return true;
  }
  // skip any value
  bool skip() {
    ws();
    if (p >= e) return fail = true, false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = (*p == '{') ? '}' : ']';
      const bool obj = (*p == '{');
      ++p;
      if (eat(close)) return true;
      do {
        if (obj) {
          std::string k;
          if (!str(k) || !eat(':')) return fail = true, false;
        }
        if (!skip()) return false;
      } while (eat(','));
      if (!eat(close)) return fail = true, false;
      return true;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n' && *p != '\r' && *p != '\t') ++p;
    return true;
  }
};

int parse_header(StFile& f, const char* h, size_t n, const char* path) {
  Json j{h, h + n};
  if (!j.eat('{')) return set_error(B2Q_EINVAL, "safetensors header must be a JSON object: %s", path);
  if (j.eat('}')) return B2Q_OK;
  do {
    std::string name;
    if (!j.str(name) || !j.eat(':')) return set_error(B2Q_EINVAL, "invalid safetensors header JSON in %s", path);
    if (name == "__metadata__") {
      if (!j.skip()) return set_error(B2Q_EINVAL, "invalid safetensors header JSON in %s", path);
      continue;
    }
    if (!j.eat('{')) return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
    TensorInfo t;
    bool has_dtype = false, has_shape = false, has_off = false;
    std::vector<int64_t> off;
    if (!j.eat('}')) {
      do {
        std::string key;
        if (!j.str(key) || !j.eat(':'))
          return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
        if (key == "dtype") {
          if (!j.str(t.dtype)) return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
          has_dtype = true;
        } else if (key == "shape") {
          if (!j.int_array(t.shape)) return set_error(B2Q_EINVAL, "invalid shape for %s in %s", name.c_str(), path);
          has_shape = true;
        } else if (key == "data_offsets") {
          if (!j.int_array(off)) return set_error(B2Q_EINVAL, "invalid data_offsets for %s in %s", name.c_str(), path);
          has_off = true;
        } else if (!j.skip()) {
          return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
        }
      } while (j.eat(','));
      if (!j.eat('}')) return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
    }
    if (!has_dtype || !has_shape || !has_off || off.size() != 2)
      return set_error(B2Q_EINVAL, "invalid tensor header for %s in %s", name.c_str(), path);
    if (off[1] < off[0]) return set_error(B2Q_EINVAL, "invalid data_offsets for %s in %s", name.c_str(), path);
    if ((uint64_t)off[1] > f.data_bytes)
      return set_error(B2Q_EINVAL, "data_offsets for %s exceed safetensors file size in %s", name.c_str(), path);
    t.begin = (uint64_t)off[0];
    t.end = (uint64_t)off[1];
    if (!f.tensors.count(name)) f.names.push_back(name);
    f.tensors[name] = t;
  } while (j.eat(','));
  if (!j.eat('}') || j.fail) return set_error(B2Q_EINVAL, "invalid safetensors header JSON in %s", path);
  return B2Q_OK;
}

void close_file(StFile* f) {
  if (!f) return;
  if (f->map) munmap(const_cast<uint8_t*>(f->map), f->size);
  if (f->fd >= 0) close(f->fd);
  delete f;
}

}  // namespace
}  // namespace b2q

using namespace b2q;

extern "C" {

int b2q_st_open(const char* path, void** handle) {
  clear_error();
  if (!path || !handle) return set_error(B2Q_EINVAL, "st_open: null argument");
  *handle = nullptr;
  StFile* f = new StFile();
  f->fd = open(path, O_RDONLY);
  if (f->fd < 0) {
    delete f;
    return set_error(B2Q_EINVAL, "cannot open safetensors file: %s", path);
  }
  struct stat sb;
  if (fstat(f->fd, &sb) != 0 || sb.st_size < 8) {
    close_file(f);
    return set_error(B2Q_EINVAL, "safetensors file is too small: %s", path);
  }
  f->size = (size_t)sb.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    f->map = nullptr;
    close_file(f);
    return set_error(B2Q_EINVAL, "cannot map safetensors file: %s", path);
  }
  f->map = static_cast<const uint8_t*>(m);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | f->map[i];  // little endian
  int rc = B2Q_OK;
  if (hlen == 0) rc = set_error(B2Q_EINVAL, "safetensors header is empty: %s", path);
  else if (hlen > kMaxHeader) rc = set_error(B2Q_EINVAL, "safetensors header exceeds %llu bytes: %s", (unsigned long long)kMaxHeader, path);
  else if (hlen > f->size - 8) rc = set_error(B2Q_EINVAL, "truncated safetensors header: %s", path);
  if (rc == B2Q_OK) {
    f->data = f->map + 8 + hlen;
    f->data_bytes = f->size - 8 - hlen;
    rc = parse_header(*f, reinterpret_cast<const char*>(f->map + 8), (size_t)hlen, path);
  }
  if (rc) {
    close_file(f);
    return rc;
  }
  *handle = f;
  return B2Q_OK;
}

int b2q_st_close(void* handle) {
  close_file(static_cast<StFile*>(handle));
  return B2Q_OK;
}

int b2q_st_count(void* handle) {
  clear_error();
  if (!handle) return set_error(B2Q_EINVAL, "st_count: null handle");
  return (int)static_cast<StFile*>(handle)->names.size();
}

// Name of tensor i (header order) copied into buf (NUL-terminated); its length, or < 0.
int b2q_st_name(void* handle, int i, char* buf, size_t buf_bytes) {
  clear_error();
  StFile* f = static_cast<StFile*>(handle);
  if (!f || i < 0 || i >= (int)f->names.size()) return set_error(B2Q_EINVAL, "st_name: bad handle or index");
  const std::string& n = f->names[i];
  if (buf && buf_bytes) {
    const size_t c = std::min(buf_bytes - 1, n.size());
    std::memcpy(buf, n.data(), c);
    buf[c] = 0;
  }
  return (int)n.size();
}

int b2q_st_info(void* handle, const char* name, char* dtype, size_t dtype_bytes, int64_t* shape, int max_dims,
                int* ndim, uint64_t* nbytes) {
  clear_error();
  StFile* f = static_cast<StFile*>(handle);
  if (!f || !name) return set_error(B2Q_EINVAL, "st_info: null argument");
  auto it = f->tensors.find(name);
  if (it == f->tensors.end()) return set_error(B2Q_EINVAL, "tensor not found in safetensors file: %s", name);
  const TensorInfo& t = it->second;
  if (dtype && dtype_bytes) {
    const size_t c = std::min(dtype_bytes - 1, t.dtype.size());
    std::memcpy(dtype, t.dtype.data(), c);
    dtype[c] = 0;
  }
  if (ndim) *ndim = (int)t.shape.size();
  if (shape)
    for (int d = 0; d < max_dims && d < (int)t.shape.size(); ++d) shape[d] = t.shape[d];
  if (nbytes) *nbytes = t.end - t.begin;
  return B2Q_OK;
}

// Copy tensor `name` (its bytes as stored) to dst: host memory when to_device == 0,
// device memory otherwise (cudaMemcpyAsync on stream, then a stream synchronise).
int b2q_st_read(void* handle, const char* name, void* dst, size_t dst_bytes, int to_device, void* stream) {
  clear_error();
  StFile* f = static_cast<StFile*>(handle);
  if (!f || !name || !dst) return set_error(B2Q_EINVAL, "st_read: null argument");
  auto it = f->tensors.find(name);
  if (it == f->tensors.end()) return set_error(B2Q_EINVAL, "tensor not found in safetensors file: %s", name);
  const TensorInfo& t = it->second;
  const size_t n = (size_t)(t.end - t.begin);
  if (dst_bytes < n) return set_error(B2Q_EINVAL, "st_read: %s needs %zu bytes, got %zu", name, n, dst_bytes);
  const uint8_t* src = f->data + t.begin;
  if (!to_device) {
    std::memcpy(dst, src, n);
    return B2Q_OK;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2Q_TRY_CUDA(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, st));
  B2Q_TRY_CUDA(cudaStreamSynchronize(st));
  return B2Q_OK;
}

}  // extern "C"
