// Safetensors reader (host only): the checkpoint format the reference loads
// its NVFP4 / FP8 weights from (crates/firepit/src/checkpoint.rs:57-213,
// SafetensorsFile over the `safetensors` crate's Metadata / TensorInfo).
//
// File layout (the safetensors format): an 8-byte little-endian header
// length N, N bytes of UTF-8 JSON (an object: tensor name -> {"dtype",
// "shape", "data_offsets": [begin, end]} relative to the data buffer, plus an
// optional "__metadata__" object of string -> string), then the data buffer.
// The header is parsed by a small JSON reader of our own; every tensor's byte
// range is checked against its dtype and shape and against the file size,
// and reads use pread, like the reference's read_exact_at.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

struct fpb_safetensors {
  struct Tensor {
    int dtype = 0;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
  };
  int fd = -1;
  uint64_t data_start = 0;
  std::vector<std::string> names;  // in data-offset order
  std::map<std::string, Tensor> tensors;
  std::map<std::string, std::string> metadata;
};

namespace fpb {
namespace {

// Element size in bytes of each dtype code (FPB_ST_*), 0 = unknown.
constexpr struct {
  const char *name;
  int bytes;
} kStDtypes[] = {{"BOOL", 1}, {"U8", 1},  {"I8", 1},   {"F8_E5M2", 1}, {"F8_E4M3", 1},
                 {"I16", 2},  {"U16", 2}, {"F16", 2},  {"BF16", 2},    {"I32", 4},
                 {"U32", 4},  {"F32", 4}, {"F64", 8},  {"I64", 8},     {"U64", 8}};
constexpr int kStDtypeCount = sizeof(kStDtypes) / sizeof(kStDtypes[0]);

// ---- a minimal JSON reader (objects, arrays, strings, numbers, literals) ----
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  bool integral = false;
  int64_t i = 0;
  std::string str;
  std::vector<Json> items;                             // Array
  std::vector<std::pair<std::string, Json>> members;  // Object, in file order
};

struct Parser {
  const char *p, *end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail_at(const char *what) {
    if (err.empty()) err = what;
    return false;
  }
  static void put_utf8(std::string &s, uint32_t c) {
    if (c < 0x80) {
      s += (char)c;
    } else if (c < 0x800) {
      s += (char)(0xC0 | (c >> 6));
      s += (char)(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      s += (char)(0xE0 | (c >> 12));
      s += (char)(0x80 | ((c >> 6) & 0x3F));
      s += (char)(0x80 | (c & 0x3F));
    } else {
      s += (char)(0xF0 | (c >> 18));
      s += (char)(0x80 | ((c >> 12) & 0x3F));
      s += (char)(0x80 | ((c >> 6) & 0x3F));
      s += (char)(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t &v) {
    if (end - p < 4) return fail_at("truncated \\u escape");
    v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail_at("bad \\u escape");
    }
    return true;
  }
  bool string(std::string &s) {
    if (p >= end || *p != '"') return fail_at("expected a string");
    ++p;
    while (p < end && *p != '"') {
      const unsigned char c = (unsigned char)*p++;
      if (c < 0x20) return fail_at("control character in a string");
      if (c != '\\') {
        s += (char)c;
        continue;
      }
      if (p >= end) return fail_at("truncated escape");
      const char e = *p++;
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2;
            if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail_at("lone surrogate");
            p += 2;
            if (!hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000) return fail_at("bad surrogate pair");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          put_utf8(s, c1);
          break;
        }
        default: return fail_at("bad escape");
      }
    }
    if (p >= end) return fail_at("unterminated string");
    ++p;
    return true;
  }
  bool number(Json &v) {
    const char *s = p;
    if (p < end && *p == '-') ++p;
    bool frac = false;
    while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-')) {
      if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
      ++p;
    }
    if (p == s) return fail_at("expected a value");
    const std::string t(s, p);
    char *stop = nullptr;
    v.kind = Json::Number;
    v.num = strtod(t.c_str(), &stop);
    if (!stop || *stop) return fail_at("bad number");
    if (!frac) {
      errno = 0;
      const long long i = strtoll(t.c_str(), &stop, 10);
      if (errno == 0 && stop && !*stop) {
        v.integral = true;
        v.i = i;
      }
    }
    return true;
  }
  bool value(Json &v) {
    if (++depth > 64) return fail_at("nesting too deep");
    ws();
    if (p >= end) return fail_at("unexpected end of header");
    bool ok = true;
    if (*p == '{') {
      ++p;
      v.kind = Json::Object;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string key;
          if (!string(key)) return false;
          ws();
          if (p >= end || *p != ':') return fail_at("expected ':'");
          ++p;
          v.members.emplace_back(std::move(key), Json());
          if (!value(v.members.back().second)) return false;
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          return fail_at("expected ',' or '}'");
        }
      }
    } else if (*p == '[') {
      ++p;
      v.kind = Json::Array;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          v.items.emplace_back();
          if (!value(v.items.back())) return false;
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          return fail_at("expected ',' or ']'");
        }
      }
    } else if (*p == '"') {
      v.kind = Json::String;
      ok = string(v.str);
    } else if (end - p >= 4 && !memcmp(p, "true", 4)) {
      v.kind = Json::Bool, v.b = true, p += 4;
    } else if (end - p >= 5 && !memcmp(p, "false", 5)) {
      v.kind = Json::Bool, v.b = false, p += 5;
    } else if (end - p >= 4 && !memcmp(p, "null", 4)) {
      v.kind = Json::Null, p += 4;
    } else {
      ok = number(v);
    }
    --depth;
    return ok;
  }
};

const Json *member(const Json &o, const char *key) {
  for (const auto &m : o.members)
    if (m.first == key) return &m.second;
  return nullptr;
}

int dtype_code(const std::string &s) {
  for (int i = 0; i < kStDtypeCount; ++i)
    if (s == kStDtypes[i].name) return i;
  return -1;
}

bool read_at(int fd, void *dst, uint64_t bytes, uint64_t offset) {
  uint8_t *d = static_cast<uint8_t *>(dst);
  while (bytes > 0) {
    const ssize_t r = pread(fd, d, (size_t)std::min<uint64_t>(bytes, 1ull << 30), (off_t)offset);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    d += r;
    bytes -= (uint64_t)r;
    offset += (uint64_t)r;
  }
  return true;
}

const fpb_safetensors::Tensor *find(const fpb_safetensors *f, const char *name) {
  if (!f || !name) return nullptr;
  auto it = f->tensors.find(name);
  return it == f->tensors.end() ? nullptr : &it->second;
}

}  // namespace
}  // namespace fpb

using namespace fpb;

// SafetensorsFile::open (checkpoint.rs:63-76).
extern "C" int fpb_safetensors_open(const char *path, fpb_safetensors **out) {
  if (!path || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_safetensors_open: null pointer");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(FPB_ERR_IO, "%s: %s", path, strerror(errno));
  auto *f = new fpb_safetensors();
  f->fd = fd;
  auto bad = [&](int status, const char *fmt, const char *detail) {
    close(fd);
    delete f;
    return fail(status, fmt, path, detail);
  };
  struct stat st;
  if (fstat(fd, &st) != 0) return bad(FPB_ERR_IO, "%s: %s", strerror(errno));
  const uint64_t size = (uint64_t)st.st_size;
  uint8_t len8[8];
  if (size < 8 || !read_at(fd, len8, 8, 0)) return bad(FPB_ERR_FORMAT, "%s: %s", "shorter than a header");
  uint64_t n = 0;
  for (int k = 7; k >= 0; --k) n = (n << 8) | len8[k];
  if (n > 100000000ull || n > size - 8) return bad(FPB_ERR_FORMAT, "%s: %s", "header length out of range");
  std::string json((size_t)n, '\0');
  if (!read_at(fd, &json[0], n, 8)) return bad(FPB_ERR_IO, "%s: %s", "header read failed");
  f->data_start = 8 + n;
  const uint64_t data_bytes = size - f->data_start;

  Parser ps{json.data(), json.data() + json.size()};
  Json root;
  if (!ps.value(root)) return bad(FPB_ERR_FORMAT, "%s: header JSON: %s", ps.err.c_str());
  ps.ws();
  if (ps.p != ps.end) return bad(FPB_ERR_FORMAT, "%s: header JSON: %s", "trailing characters");
  if (root.kind != Json::Object) return bad(FPB_ERR_FORMAT, "%s: %s", "header is not an object");

  std::vector<std::pair<uint64_t, std::string>> order;
  for (const auto &m : root.members) {
    if (m.first == "__metadata__") {
      if (m.second.kind != Json::Object) return bad(FPB_ERR_FORMAT, "%s: %s", "__metadata__ is not an object");
      for (const auto &kv : m.second.members) {
        if (kv.second.kind != Json::String) return bad(FPB_ERR_FORMAT, "%s: %s", "__metadata__ value is not a string");
        f->metadata[kv.first] = kv.second.str;
      }
      continue;
    }
    const Json &t = m.second;
    const Json *dt = t.kind == Json::Object ? member(t, "dtype") : nullptr;
    const Json *sh = t.kind == Json::Object ? member(t, "shape") : nullptr;
    const Json *off = t.kind == Json::Object ? member(t, "data_offsets") : nullptr;
    if (!dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off || off->kind != Json::Array ||
        off->items.size() != 2)
      return bad(FPB_ERR_FORMAT, "%s: tensor %s has no dtype, shape and data_offsets", m.first.c_str());
    fpb_safetensors::Tensor info;
    info.dtype = dtype_code(dt->str);
    if (info.dtype < 0) return bad(FPB_ERR_FORMAT, "%s: unsupported dtype %s", dt->str.c_str());
    uint64_t numel = 1;
    for (const auto &d : sh->items) {
      if (d.kind != Json::Number || !d.integral || d.i < 0) return bad(FPB_ERR_FORMAT, "%s: bad shape of %s", m.first.c_str());
      info.shape.push_back(d.i);
      if (d.i != 0 && numel > UINT64_MAX / (uint64_t)d.i) return bad(FPB_ERR_FORMAT, "%s: shape of %s overflows", m.first.c_str());
      numel *= (uint64_t)d.i;
    }
    for (const auto &o : off->items)
      if (o.kind != Json::Number || !o.integral || o.i < 0)
        return bad(FPB_ERR_FORMAT, "%s: bad data_offsets of %s", m.first.c_str());
    info.begin = (uint64_t)off->items[0].i;
    info.end = (uint64_t)off->items[1].i;
    const uint64_t esz = (uint64_t)kStDtypes[info.dtype].bytes;
    if (info.begin > info.end || info.end > data_bytes || (numel && esz > UINT64_MAX / numel) ||
        info.end - info.begin != numel * esz)
      return bad(FPB_ERR_FORMAT, "%s: data_offsets of %s disagree with its dtype, shape or the file size",
                 m.first.c_str());
    if (f->tensors.count(m.first)) return bad(FPB_ERR_FORMAT, "%s: duplicate tensor %s", m.first.c_str());
    f->tensors.emplace(m.first, std::move(info));
    order.emplace_back(f->tensors[m.first].begin, m.first);
  }
  std::stable_sort(order.begin(), order.end(),
                   [](const auto &a, const auto &b) { return a.first < b.first; });
  for (auto &o : order) f->names.push_back(std::move(o.second));
  *out = f;
  return FPB_OK;
}

extern "C" void fpb_safetensors_close(fpb_safetensors *f) {
  if (!f) return;
  if (f->fd >= 0) close(f->fd);
  delete f;
}

extern "C" size_t fpb_safetensors_count(const fpb_safetensors *f) { return f ? f->names.size() : 0; }

extern "C" const char *fpb_safetensors_name(const fpb_safetensors *f, size_t i) {
  return (f && i < f->names.size()) ? f->names[i].c_str() : nullptr;
}

// SafetensorsFile::has_tensor (checkpoint.rs:86-88).
extern "C" int fpb_safetensors_has(const fpb_safetensors *f, const char *name) { return find(f, name) != nullptr; }

// SafetensorsFile::metadata (checkpoint.rs:78-84): NULL when absent.
extern "C" const char *fpb_safetensors_metadata(const fpb_safetensors *f, const char *key) {
  if (!f || !key) return nullptr;
  auto it = f->metadata.find(key);
  return it == f->metadata.end() ? nullptr : it->second.c_str();
}

extern "C" const char *fpb_safetensors_dtype_name(int dtype) {
  return (dtype >= 0 && dtype < kStDtypeCount) ? kStDtypes[dtype].name : nullptr;
}

// TensorInfo of a tensor (checkpoint.rs:187-191, Checkpoint::stored).
extern "C" int fpb_safetensors_info(const fpb_safetensors *f, const char *name, int *dtype, int64_t *shape,
                                    int max_dims, int *ndim, size_t *nbytes) {
  const fpb_safetensors::Tensor *t = find(f, name);
  if (!t) return fail(FPB_ERR_FORMAT, "unknown tensor %s", name ? name : "(null)");
  if (dtype) *dtype = t->dtype;
  if (ndim) *ndim = (int)t->shape.size();
  if (nbytes) *nbytes = (size_t)(t->end - t->begin);
  if (shape) {
    if ((int)t->shape.size() > max_dims)
      return fail(FPB_ERR_INVALID_ARGUMENT, "%s has %zu dimensions (room for %d)", name, t->shape.size(), max_dims);
    for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
  }
  return FPB_OK;
}

// SafetensorsFile::bytes (checkpoint.rs:158-167): the tensor's raw bytes, after
// checking its stored dtype (FPB_ERR_FORMAT "expected X, got Y" otherwise).
// Bytes [byte_begin, byte_begin + bytes) of the tensor's range are read, so
// that a caller can take rows (SafetensorsFile::row, :169-185) or stream a
// large tensor in pieces.
extern "C" int fpb_safetensors_read(const fpb_safetensors *f, const char *name, int dtype, size_t byte_begin,
                                    void *dst, size_t bytes) {
  const fpb_safetensors::Tensor *t = find(f, name);
  if (!t) return fail(FPB_ERR_FORMAT, "unknown tensor %s", name ? name : "(null)");
  if (dtype != t->dtype)
    return fail(FPB_ERR_FORMAT, "%s: expected %s, got %s", name,
                fpb_safetensors_dtype_name(dtype) ? fpb_safetensors_dtype_name(dtype) : "?",
                kStDtypes[t->dtype].name);
  if (bytes == 0) return FPB_OK;
  if (!dst) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_safetensors_read: null destination");
  const uint64_t len = t->end - t->begin;
  if (byte_begin > len || bytes > len - byte_begin)
    return fail(FPB_ERR_SHAPE, "%s: bytes [%zu, %zu) outside its %llu", name, byte_begin, byte_begin + bytes,
                (unsigned long long)len);
  if (!read_at(f->fd, dst, bytes, f->data_start + t->begin + byte_begin))
    return fail(FPB_ERR_IO, "%s: read failed (%s)", name, strerror(errno));
  return FPB_OK;
}
