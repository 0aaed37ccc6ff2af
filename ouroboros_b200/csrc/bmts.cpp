// bmts.cpp -- reader of BMTS v1 shard files (the reference's model tensor shard
// format, cluster/src/bmts.rs:1-14, 171-209) and their upload to the device.
//
// Layout (little-endian): magic u32 0x4F55524F ("OURO"), version u16 (1),
// node u16, n_tensors u32, meta_len u32, meta = JSON array of
// {name, shape[], dtype, offset, length}, then the data section. The file is
// memory-mapped; tensor spans are views into the mapping, as the reference's
// Payload::Mapped. Version 2 (Cap'n Proto meta) is refused, as the reference
// does without its capnp2 feature. Errors follow bmts.rs's messages.
#include "ouroq.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

struct BmtsEntry {
  std::string name;
  std::vector<uint64_t> shape;
  uint32_t dtype = 0;
  uint64_t offset = 0, length = 0;
};

struct ouroq_bmts {
  std::string path;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint16_t node = 0;
  uint64_t data_start = 0;
  std::vector<BmtsEntry> tensors;
};

namespace {

constexpr uint32_t kBmtsMagic = 0x4F55524Fu;
constexpr uint16_t kBmtsVersion = 1;
constexpr size_t kBmtsHeaderLen = 16;
constexpr uint32_t kDtypeTq1 = 34;   // QuantKind::Tq1_0 (dequant.rs:344)
constexpr uint32_t kDtypeTl1 = 143;  // QuantKind::Tl1 (dequant.rs:345)
constexpr uint32_t kDtypeF16 = 1;    // QuantKind::F16 (dequant.rs:337)
constexpr uint32_t kDtypeBf16 = 30;  // QuantKind::Bf16 (dequant.rs:338)

void set_err(char* err, size_t len, const char* fmt, ...) {
  if (!err || !len) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, len, fmt, ap);
  va_end(ap);
}

// Whole-table UTF-8 check: the reference parses the table with serde_json from
// bytes, which refuses invalid UTF-8 (overlong forms, surrogates, code points
// past U+10FFFF, truncated sequences).
bool valid_utf8(const uint8_t* p, const uint8_t* e) {
  while (p < e) {
    const uint8_t c = *p++;
    if (c < 0x80) continue;
    int n;
    uint32_t v;
    if (c >= 0xC2 && c <= 0xDF) n = 1, v = c & 0x1F;
    else if (c >= 0xE0 && c <= 0xEF) n = 2, v = c & 0x0F;
    else if (c >= 0xF0 && c <= 0xF4) n = 3, v = c & 0x07;
    else return false;
    if (e - p < n) return false;
    for (int i = 0; i < n; ++i) {
      if ((p[i] & 0xC0) != 0x80) return false;
      v = (v << 6) | (p[i] & 0x3F);
    }
    p += n;
    if ((n == 2 && v < 0x800) || (n == 3 && v < 0x10000) || v > 0x10FFFF ||
        (v >= 0xD800 && v <= 0xDFFF))
      return false;
  }
  return true;
}

void put_utf8(std::string& s, uint32_t v) {
  if (v < 0x80) {
    s += (char)v;
  } else if (v < 0x800) {
    s += (char)(0xC0 | (v >> 6));
    s += (char)(0x80 | (v & 0x3F));
  } else if (v < 0x10000) {
    s += (char)(0xE0 | (v >> 12));
    s += (char)(0x80 | ((v >> 6) & 0x3F));
    s += (char)(0x80 | (v & 0x3F));
  } else {
    s += (char)(0xF0 | (v >> 18));
    s += (char)(0x80 | ((v >> 12) & 0x3F));
    s += (char)(0x80 | ((v >> 6) & 0x3F));
    s += (char)(0x80 | (v & 0x3F));
  }
}

// Minimal JSON reader for the tensor table: an array of objects whose values
// are strings, unsigned integers or arrays of unsigned integers. Unknown keys
// are skipped (any JSON value, nested at most kMaxDepth deep). Strings follow
// the JSON grammar: no raw control characters, the eight escapes, \u with
// surrogate pairs.
constexpr int kMaxDepth = 128;
struct Json {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool expect(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    err = std::string("expected '") + c + "'";
    return false;
  }
  bool peek(char c) {
    ws();
    return p < e && *p == c;
  }
  bool hex4(uint32_t* v) {
    if (e - p < 4) return (err = "bad \\u escape"), false;
    *v = 0;
    for (int i = 0; i < 4; ++i) {
      const char h = *p++;
      *v <<= 4;
      if (h >= '0' && h <= '9') *v |= (uint32_t)(h - '0');
      else if (h >= 'a' && h <= 'f') *v |= (uint32_t)(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') *v |= (uint32_t)(h - 'A' + 10);
      else return (err = "bad \\u escape"), false;
    }
    return true;
  }
  bool string(std::string* out) {
    if (!expect('"')) return false;
    std::string s;
    while (p < e && *p != '"') {
      const char c = *p++;
      if ((unsigned char)c < 0x20) return (err = "control character in a string"), false;
      if (c != '\\') {
        s += c;
        continue;
      }
      if (p >= e) break;
      const char x = *p++;
      switch (x) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'n': s += '\n'; break;
        case 't': s += '\t'; break;
        case 'r': s += '\r'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'u': {
          uint32_t v;
          if (!hex4(&v)) return false;
          if (v >= 0xDC00 && v <= 0xDFFF) return (err = "lone surrogate in \\u escape"), false;
          if (v >= 0xD800 && v <= 0xDBFF) {
            uint32_t lo;
            if (e - p < 2 || p[0] != '\\' || p[1] != 'u')
              return (err = "lone surrogate in \\u escape"), false;
            p += 2;
            if (!hex4(&lo)) return false;
            if (lo < 0xDC00 || lo > 0xDFFF) return (err = "lone surrogate in \\u escape"), false;
            v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(s, v);
          break;
        }
        default:
          return (err = "invalid escape in a string"), false;
      }
    }
    if (!expect('"')) return false;
    if (out) *out = s;
    return true;
  }
  bool uint(uint64_t* out) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return (err = "expected an unsigned integer"), false;
    uint64_t v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p++ - '0');
      if (v > (UINT64_MAX - d) / 10) return (err = "integer overflow"), false;
      v = v * 10 + d;
    }
    if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return (err = "expected an integer"), false;
    *out = v;
    return true;
  }
  bool literal(const char* word) {
    const size_t n = std::strlen(word);
    if ((size_t)(e - p) < n || std::memcmp(p, word, n) != 0) return (err = "bad value"), false;
    p += n;
    return true;
  }
  // JSON number: -?(0|[1-9][0-9]*)(.[0-9]+)?([eE][+-]?[0-9]+)?
  bool number() {
    auto digits = [&]() {
      const char* s = p;
      while (p < e && *p >= '0' && *p <= '9') ++p;
      return p > s;
    };
    if (p < e && *p == '-') ++p;
    if (p < e && *p == '0') {
      ++p;
    } else if (!digits()) {
      return (err = "bad value"), false;
    }
    if (p < e && *p == '.') {
      ++p;
      if (!digits()) return (err = "bad number"), false;
    }
    if (p < e && (*p == 'e' || *p == 'E')) {
      ++p;
      if (p < e && (*p == '+' || *p == '-')) ++p;
      if (!digits()) return (err = "bad number"), false;
    }
    return true;
  }
  bool skip_value(int depth = 0) {
    ws();
    if (p >= e) return (err = "truncated"), false;
    if (depth > kMaxDepth) return (err = "values nested too deep"), false;
    if (*p == '"') return string(nullptr);
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      if (peek(close)) return ++p, true;
      for (;;) {
        if (open == '{') {
          if (!string(nullptr) || !expect(':')) return false;
        }
        if (!skip_value(depth + 1)) return false;
        if (peek(',')) {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    if (*p == 't') return literal("true");
    if (*p == 'f') return literal("false");
    if (*p == 'n') return literal("null");
    return number();
  }
  bool uint_array(std::vector<uint64_t>* out) {
    if (!expect('[')) return false;
    if (peek(']')) return ++p, true;
    for (;;) {
      uint64_t v;
      if (!uint(&v)) return false;
      out->push_back(v);
      if (peek(',')) {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
  bool table(std::vector<BmtsEntry>* out) {
    if (!expect('[')) return false;
    if (peek(']')) return ++p, true;
    for (;;) {
      if (!expect('{')) return false;
      BmtsEntry t;
      bool have[5] = {false, false, false, false, false};
      if (!peek('}')) {
        for (;;) {
          std::string key;
          if (!string(&key) || !expect(':')) return false;
          uint64_t v = 0;
          if (key == "name") {
            if (!string(&t.name)) return false;
            if (t.name.find('\0') != std::string::npos)
              return (err = "tensor name holds a NUL character"), false;
            have[0] = true;
          } else if (key == "shape") {
            if (!uint_array(&t.shape)) return false;
            have[1] = true;
          } else if (key == "dtype") {
            if (!uint(&v)) return false;
            if (v > UINT32_MAX) return (err = "dtype out of range"), false;
            t.dtype = (uint32_t)v;
            have[2] = true;
          } else if (key == "offset") {
            if (!uint(&t.offset)) return false;
            have[3] = true;
          } else if (key == "length") {
            if (!uint(&t.length)) return false;
            have[4] = true;
          } else if (!skip_value()) {
            return false;
          }
          if (peek(',')) {
            ++p;
            continue;
          }
          break;
        }
      }
      if (!expect('}')) return false;
      for (bool h : have)
        if (!h) return (err = "tensor entry lacks a field"), false;
      out->push_back(std::move(t));
      if (peek(',')) {
        ++p;
        continue;
      }
      if (!expect(']')) return false;
      ws();
      if (p != e) return (err = "trailing bytes after the tensor table"), false;
      return true;
    }
  }
};

uint32_t rd32(const uint8_t* b) {
  return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}
uint16_t rd16(const uint8_t* b) { return (uint16_t)(b[0] | (b[1] << 8)); }

const BmtsEntry* find(const ouroq_bmts* f, const char* name) {
  for (const BmtsEntry& t : f->tensors)
    if (t.name == name) return &t;
  return nullptr;
}

}  // namespace

extern "C" {

ouroq_status ouroq_bmts_open(const char* path, ouroq_bmts** out, char* err, size_t err_len) {
  if (!path || !out) return OUROQ_ERR_BAD_ARG;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) {
    set_err(err, err_len, "cannot open %s", path);
    return OUROQ_ERR_BAD_ARG;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    set_err(err, err_len, "cannot stat %s", path);
    return OUROQ_ERR_BAD_ARG;
  }
  const size_t size = (size_t)st.st_size;
  if (size < kBmtsHeaderLen) {
    close(fd);
    set_err(err, err_len, "BMTS file too short: %s", path);
    return OUROQ_ERR_BAD_SHAPE;
  }
  void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    set_err(err, err_len, "cannot map %s", path);
    return OUROQ_ERR_BAD_ARG;
  }
  const uint8_t* b = static_cast<const uint8_t*>(m);
  auto bail = [&](ouroq_status s) {
    munmap(m, size);
    return s;
  };
  const uint32_t magic = rd32(b);
  if (magic != kBmtsMagic) {
    set_err(err, err_len, "bad BMTS magic %#010x in %s", magic, path);
    return bail(OUROQ_ERR_BAD_SHAPE);
  }
  const uint16_t version = rd16(b + 4);
  const uint16_t node = rd16(b + 6);
  const uint32_t n_tensors = rd32(b + 8);
  const uint32_t meta_len = rd32(b + 12);
  if (size < kBmtsHeaderLen + (size_t)meta_len) {
    set_err(err, err_len, "BMTS meta truncated: %s", path);
    return bail(OUROQ_ERR_BAD_SHAPE);
  }
  if (version != kBmtsVersion) {
    set_err(err, err_len,
            "unsupported BMTS version %u in %s (only v1, JSON meta, is read here)", version, path);
    return bail(OUROQ_ERR_UNSUPPORTED);
  }
  if (!valid_utf8(b + kBmtsHeaderLen, b + kBmtsHeaderLen + meta_len)) {
    set_err(err, err_len, "BMTS meta is not valid UTF-8: %s", path);
    return bail(OUROQ_ERR_BAD_SHAPE);
  }
  ouroq_bmts* f = new (std::nothrow) ouroq_bmts;
  if (!f) return bail(OUROQ_ERR_OOM);
  Json j{reinterpret_cast<const char*>(b + kBmtsHeaderLen),
         reinterpret_cast<const char*>(b + kBmtsHeaderLen + meta_len), {}};
  if (!j.table(&f->tensors)) {
    set_err(err, err_len, "BMTS meta is not a tensor table (%s): %s", j.err.c_str(), path);
    delete f;
    return bail(OUROQ_ERR_BAD_SHAPE);
  }
  if (f->tensors.size() != n_tensors) {
    set_err(err, err_len, "BMTS tensor count mismatch: header %u vs meta %zu", n_tensors,
            f->tensors.size());
    delete f;
    return bail(OUROQ_ERR_BAD_SHAPE);
  }
  f->path = path;
  f->map = b;
  f->size = size;
  f->node = node;
  f->data_start = kBmtsHeaderLen + meta_len;
  *out = f;
  return OUROQ_OK;
}

ouroq_status ouroq_bmts_close(ouroq_bmts* f) {
  if (!f) return OUROQ_ERR_BAD_ARG;
  if (f->map) munmap(const_cast<uint8_t*>(f->map), f->size);
  delete f;
  return OUROQ_OK;
}

ouroq_status ouroq_bmts_info(const ouroq_bmts* f, int* node, int* n_tensors, uint64_t* data_start,
                             uint64_t* data_len) {
  if (!f) return OUROQ_ERR_BAD_ARG;
  if (node) *node = f->node;
  if (n_tensors) *n_tensors = (int)f->tensors.size();
  if (data_start) *data_start = f->data_start;
  if (data_len) {
    uint64_t n = 0;
    for (const BmtsEntry& t : f->tensors) n += t.length;
    *data_len = n;
  }
  return OUROQ_OK;
}

ouroq_status ouroq_bmts_tensor(const ouroq_bmts* f, int i, const char** name, int* rank,
                               uint64_t* shape4, uint32_t* dtype, uint64_t* offset,
                               uint64_t* length) {
  if (!f || i < 0 || i >= (int)f->tensors.size()) return OUROQ_ERR_BAD_ARG;
  const BmtsEntry& t = f->tensors[i];
  if (name) *name = t.name.c_str();
  if (rank) *rank = (int)t.shape.size();
  if (shape4)
    for (int k = 0; k < 4; ++k) shape4[k] = k < (int)t.shape.size() ? t.shape[k] : 0;
  if (dtype) *dtype = t.dtype;
  if (offset) *offset = t.offset;
  if (length) *length = t.length;
  return OUROQ_OK;
}

ouroq_status ouroq_bmts_span(const ouroq_bmts* f, const char* name, uint64_t offset,
                             uint64_t length, const void** out, char* err, size_t err_len) {
  if (!f || !name || !out) return OUROQ_ERR_BAD_ARG;
  *out = nullptr;
  const BmtsEntry* t = find(f, name);
  if (!t) {
    set_err(err, err_len, "tensor %s not in shard", name);
    return OUROQ_ERR_BAD_ARG;
  }
  if (offset > t->length || length > t->length - offset) {
    set_err(err, err_len, "span [%llu, %llu) exceeds tensor %s of %llu bytes",
            (unsigned long long)offset, (unsigned long long)(offset + length), name,
            (unsigned long long)t->length);
    return OUROQ_ERR_BAD_SHAPE;
  }
  uint64_t start = 0;
  if (__builtin_add_overflow(f->data_start, t->offset, &start) ||
      __builtin_add_overflow(start, offset, &start) || start > f->size ||
      length > f->size - start) {
    set_err(err, err_len, "tensor %s range exceeds file %s", name, f->path.c_str());
    return OUROQ_ERR_BAD_SHAPE;
  }
  *out = f->map + start;
  return OUROQ_OK;
}

ouroq_status ouroq_bmts_upload(ouroq_ctx* ctx, const ouroq_bmts* f, const char* name,
                               ouroq_weight** out, char* err, size_t err_len) {
  if (!ctx || !f || !name || !out) return OUROQ_ERR_BAD_ARG;
  *out = nullptr;
  const BmtsEntry* t = find(f, name);
  if (!t) {
    set_err(err, err_len, "tensor %s not in shard", name);
    return OUROQ_ERR_BAD_ARG;
  }
  ouroq_format fmt;
  if (t->dtype == kDtypeTl1) {
    fmt = OUROQ_FMT_PTQ1_0;
  } else if (t->dtype == kDtypeTq1) {
    fmt = OUROQ_FMT_TQ1_0;
  } else if (t->dtype == kDtypeF16) {
    fmt = OUROQ_FMT_F16;
  } else if (t->dtype == kDtypeBf16) {
    fmt = OUROQ_FMT_BF16;
  } else {
    set_err(err, err_len,
            "tensor %s: dtype %u is not a matmul format here (1 F16, 30 BF16, 34 TQ1_0, 143 Tl1)",
            name, t->dtype);
    return OUROQ_ERR_UNSUPPORTED;
  }
  // GGUF order [in, out] (infer/mod.rs:118-122): in_len = shape[0], out_len = shape[1]
  if (t->shape.size() != 2 || t->shape[0] == 0 || t->shape[1] == 0 || t->shape[0] > INT32_MAX ||
      t->shape[1] > INT32_MAX) {
    set_err(err, err_len, "tensor %s: expected a rank-2 shape", name);
    return OUROQ_ERR_BAD_SHAPE;
  }
  const int K = (int)t->shape[0], M = (int)t->shape[1];
  const uint64_t rb = fmt == OUROQ_FMT_PTQ1_0 ? (uint64_t)K / 128 * 28
                      : fmt == OUROQ_FMT_TQ1_0 ? (uint64_t)K / 256 * 54
                                               : (uint64_t)K * 2;
  if (rb * (uint64_t)M != t->length) {
    set_err(err, err_len, "tensor %s: %llu bytes, %d x %d needs %llu", name,
            (unsigned long long)t->length, M, K, (unsigned long long)(rb * (uint64_t)M));
    return OUROQ_ERR_BAD_SHAPE;
  }
  const void* p = nullptr;
  ouroq_status st = ouroq_bmts_span(f, name, 0, t->length, &p, err, err_len);
  if (st != OUROQ_OK) return st;
  st = ouroq_weight_upload(ctx, fmt, p, M, K, nullptr, 1.0f, out);
  if (st != OUROQ_OK) set_err(err, err_len, "upload of %s: %s", name, ouroq_last_error(ctx));
  return st;
}

}  // extern "C"
