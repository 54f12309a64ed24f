// Memory-mapped safetensors reader (host side of the loader, crates/tts-nn/src/lib.rs:153-373,
// which maps the file through candle's MmapedSafetensors): an 8-byte little-endian header
// length, a JSON header {name: {"dtype", "shape", "data_offsets": [begin, end]}, optional
// "__metadata__"}, then the tensors' bytes. Tensors are handed out as views into the mapping;
// casts, transposes and folds are the caller's load-time work.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "tts_cuda.h"

namespace tts {
void set_error(const std::string& msg);
}

struct tts_safetensors {
  void* map = nullptr;
  size_t size = 0;
  const uint8_t* data = nullptr;  // start of the tensor bytes
  std::vector<std::string> names;
  struct Info {
    int dtype = TTS_DT_OTHER;
    int ndim = 0;
    long long shape[8] = {0};
    size_t begin = 0, end = 0;
  };
  std::vector<Info> info;
  std::unordered_map<std::string, int> index;
};

namespace {

using tts::set_error;

// A JSON reader for the header's subset: objects, arrays, strings, integers; other values
// (true/false/null/floats in the metadata) are skipped.
struct Json {
  const char* p;
  const char* e;
  bool ok = true;

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
  bool str(std::string* out) {
    ws();
    if (p >= e || *p != '"') return ok = false;
    ++p;
    std::string s;
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return ok = false;
        const char x = *p++;
        switch (x) {
          case '"': s += '"'; break;
          case '\\': s += '\\'; break;
          case '/': s += '/'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            if (e - p < 4) return ok = false;
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= unsigned(h - '0');
              else if (h >= 'a' && h <= 'f') cp |= unsigned(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') cp |= unsigned(h - 'A' + 10);
              else return ok = false;
            }
            // UTF-8 of a basic-plane code point (names here are ASCII in practice)
            if (cp < 0x80) {
              s += char(cp);
            } else if (cp < 0x800) {
              s += char(0xC0 | (cp >> 6));
              s += char(0x80 | (cp & 0x3F));
            } else {
              s += char(0xE0 | (cp >> 12));
              s += char(0x80 | ((cp >> 6) & 0x3F));
              s += char(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: return ok = false;
        }
      } else {
        s += c;
      }
    }
    if (p >= e) return ok = false;
    ++p;  // closing quote
    if (out) *out = std::move(s);
    return true;
  }
  bool integer(long long* out) {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= e || *p < '0' || *p > '9') return ok = false;
    unsigned long long v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const unsigned long long d = unsigned(*p++ - '0');
      if (v > (~0ull - d) / 10) return ok = false;  // overflow
      v = v * 10 + d;
    }
    if (v > (1ull << 62)) return ok = false;
    *out = neg ? -(long long)v : (long long)v;
    return true;
  }
  bool skip() {  // any value
    ws();
    if (p >= e) return ok = false;
    if (*p == '"') return str(nullptr);
    if (*p == '{') {
      ++p;
      if (eat('}')) return true;
      do {
        if (!str(nullptr) || !eat(':') || !skip()) return ok = false;
      } while (eat(','));
      return eat('}') || (ok = false);
    }
    if (*p == '[') {
      ++p;
      if (eat(']')) return true;
      do {
        if (!skip()) return ok = false;
      } while (eat(','));
      return eat(']') || (ok = false);
    }
    // number or literal: up to the next delimiter
    const char* q = p;
    while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n' &&
           *p != '\r' && *p != '\t')
      ++p;
    return p > q || (ok = false);
  }
};

int dtype_of(const std::string& s, size_t* bytes) {
  struct D {
    const char* n;
    int code;
    size_t b;
  };
  static const D table[] = {{"F32", TTS_DT_F32, 4},  {"F16", TTS_DT_F16, 2},
                            {"BF16", TTS_DT_BF16, 2}, {"I32", TTS_DT_I32, 4},
                            {"I64", TTS_DT_I64, 8},  {"U8", TTS_DT_U8, 1},
                            {"F64", TTS_DT_F64, 8},  {"I8", TTS_DT_I8, 1},
                            {"I16", TTS_DT_I16, 2},  {"BOOL", TTS_DT_BOOL, 1}};
  for (const D& d : table)
    if (s == d.n) {
      *bytes = d.b;
      return d.code;
    }
  *bytes = 0;
  return TTS_DT_OTHER;
}

tts_status parse(tts_safetensors* f, const char* path) {
  const uint8_t* base = static_cast<const uint8_t*>(f->map);
  if (f->size < 8) {
    set_error(std::string("safetensors: ") + path + " is shorter than its header length");
    return TTS_ERR_INVALID_ARG;
  }
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
  if (hlen > f->size - 8 || hlen > (size_t(100) << 20)) {
    set_error(std::string("safetensors: ") + path + " header length out of range");
    return TTS_ERR_INVALID_ARG;
  }
  f->data = base + 8 + hlen;
  const size_t data_size = f->size - 8 - size_t(hlen);
  Json j{reinterpret_cast<const char*>(base + 8), reinterpret_cast<const char*>(base + 8 + hlen)};
  auto bad = [&](const std::string& what) {
    set_error(std::string("safetensors: ") + path + ": " + what);
    return TTS_ERR_INVALID_ARG;
  };
  if (!j.eat('{')) return bad("header is not a JSON object");
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(&name) || !j.eat(':')) return bad("malformed header");
      if (name == "__metadata__") {
        if (!j.skip()) return bad("malformed __metadata__");
        continue;
      }
      if (!j.eat('{')) return bad("tensor entry " + name + " is not an object");
      tts_safetensors::Info in;
      std::string dt;
      bool has_dt = false, has_shape = false, has_off = false;
      size_t esize = 0;
      do {
        std::string key;
        if (!j.str(&key) || !j.eat(':')) return bad("malformed entry " + name);
        if (key == "dtype") {
          if (!j.str(&dt)) return bad("dtype of " + name);
          in.dtype = dtype_of(dt, &esize);
          has_dt = true;
        } else if (key == "shape") {
          if (!j.eat('[')) return bad("shape of " + name);
          if (!j.eat(']')) {
            do {
              long long v = 0;
              if (!j.integer(&v) || v < 0 || in.ndim >= 8) return bad("shape of " + name);
              in.shape[in.ndim++] = v;
            } while (j.eat(','));
            if (!j.eat(']')) return bad("shape of " + name);
          }
          has_shape = true;
        } else if (key == "data_offsets") {
          long long b = 0, en = 0;
          if (!j.eat('[') || !j.integer(&b) || !j.eat(',') || !j.integer(&en) || !j.eat(']'))
            return bad("data_offsets of " + name);
          if (b < 0 || en < b || size_t(en) > data_size) return bad("data_offsets of " + name + " outside the file");
          in.begin = size_t(b);
          in.end = size_t(en);
          has_off = true;
        } else if (!j.skip()) {
          return bad("entry " + name);
        }
      } while (j.eat(','));
      if (!j.eat('}')) return bad("entry " + name);
      if (!has_dt || !has_shape || !has_off) return bad("entry " + name + " lacks dtype, shape or data_offsets");
      if (esize) {
        size_t n = 1;
        for (int d = 0; d < in.ndim; ++d) n *= size_t(in.shape[d]);
        if (n * esize != in.end - in.begin) return bad("size of " + name + " does not match its shape");
      }
      if (f->index.count(name)) return bad("tensor " + name + " appears twice");
      f->index[name] = int(f->names.size());
      f->names.push_back(name);
      f->info.push_back(in);
    } while (j.eat(','));
    if (!j.eat('}')) return bad("malformed header");
  }
  if (!j.ok) return bad("malformed header");
  return TTS_OK;
}

void view(const tts_safetensors* f, int i, tts_tensor_view* out) {
  const auto& in = f->info[size_t(i)];
  out->name = f->names[size_t(i)].c_str();
  out->dtype = in.dtype;
  out->ndim = in.ndim;
  for (int d = 0; d < 8; ++d) out->shape[d] = d < in.ndim ? in.shape[d] : 0;
  out->data = f->data + in.begin;
  out->nbytes = in.end - in.begin;
}

}  // namespace

extern "C" {

tts_status tts_safetensors_open(const char* path, tts_safetensors** out) {
  if (!path || !out) {
    set_error("safetensors_open: NULL argument");
    return TTS_ERR_INVALID_ARG;
  }
  const int fd = open(path, O_RDONLY);
  if (fd < 0) {
    set_error(std::string("safetensors_open: cannot open ") + path);
    return TTS_ERR_INVALID_ARG;
  }
  struct stat sb {};
  if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
    close(fd);
    set_error(std::string("safetensors_open: cannot stat ") + path + " or it is empty");
    return TTS_ERR_INVALID_ARG;
  }
  void* m = mmap(nullptr, size_t(sb.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    set_error(std::string("safetensors_open: cannot map ") + path);
    return TTS_ERR_INVALID_ARG;
  }
  auto* f = new tts_safetensors();
  f->map = m;
  f->size = size_t(sb.st_size);
  const tts_status rc = parse(f, path);
  if (rc != TTS_OK) {
    tts_safetensors_close(f);
    return rc;
  }
  *out = f;
  return TTS_OK;
}

int tts_safetensors_count(const tts_safetensors* f) { return f ? int(f->names.size()) : 0; }

tts_status tts_safetensors_at(const tts_safetensors* f, int i, tts_tensor_view* out) {
  if (!f || !out || i < 0 || i >= int(f->names.size())) {
    set_error("safetensors_at: index out of range");
    return TTS_ERR_INVALID_ARG;
  }
  view(f, i, out);
  return TTS_OK;
}

tts_status tts_safetensors_find(const tts_safetensors* f, const char* name, tts_tensor_view* out) {
  if (!f || !name || !out) {
    set_error("safetensors_find: NULL argument");
    return TTS_ERR_INVALID_ARG;
  }
  const auto it = f->index.find(name);
  if (it == f->index.end()) {
    set_error(std::string("missing tensor ") + name);
    return TTS_ERR_INVALID_ARG;
  }
  view(f, it->second, out);
  return TTS_OK;
}

tts_status tts_safetensors_close(tts_safetensors* f) {
  if (!f) return TTS_OK;
  if (f->map) munmap(f->map, f->size);
  delete f;
  return TTS_OK;
}

}  // extern "C"
