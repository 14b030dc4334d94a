// Safetensors reader: mmap, header parsing, name mapping (host code only).
#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace iam {
namespace {

// A small JSON reader for safetensors headers: objects, arrays, strings,
// integers; other scalars (floats, true/false/null) are skipped.
struct Json {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const std::string& m) {
    if (err.empty()) err = m;
    return false;
  }
  bool expect(char c) {
    ws();
    if (p >= e || *p != c) return fail(std::string("expected '") + c + "'");
    ++p;
    return true;
  }
  bool peek(char c) {
    ws();
    return p < e && *p == c;
  }
  bool string(std::string& out) {
    ws();
    if (p >= e || *p != '"') return fail("expected a string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return fail("bad escape");
        const char x = *p++;
        switch (x) {
          case 'n': c = '\n'; break;
          case 't': c = '\t'; break;
          case 'r': c = '\r'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'u':  // tensor names are ASCII; keep the code point's low byte
            if (e - p < 4) return fail("bad \\u escape");
            c = static_cast<char>(std::strtol(std::string(p, 4).c_str(), nullptr, 16) & 0xFF);
            p += 4;
            break;
          default: c = x;
        }
      }
      out.push_back(c);
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool integer(int64_t& v) {
    ws();
    const char* s = p;
    if (p < e && *p == '-') ++p;
    if (p >= e || *p < '0' || *p > '9') return fail("expected an integer");
    while (p < e && *p >= '0' && *p <= '9') ++p;
    v = std::strtoll(std::string(s, p).c_str(), nullptr, 10);
    return true;
  }
  bool skip_value(int depth = 0) {
    if (depth > 32) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("unexpected end");
    if (*p == '"') {
      std::string s;
      return string(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (peek(close)) {
        ++p;
        return true;
      }
      for (;;) {
        if (obj) {
          std::string k;
          if (!string(k) || !expect(':')) return false;
        }
        if (!skip_value(depth + 1)) return false;
        if (peek(',')) {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;  // number, true, false, null
    return true;
  }
  bool int_array(std::vector<int64_t>& out) {
    out.clear();
    if (!expect('[')) return false;
    if (peek(']')) {
      ++p;
      return true;
    }
    for (;;) {
      int64_t v;
      if (!integer(v)) return false;
      out.push_back(v);
      if (peek(',')) {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
};

size_t dtype_size(const std::string& d) {
  if (d == "U8" || d == "I8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  return 0;
}

}  // namespace

bool st_parse_header(const char* json, size_t len, int file, std::vector<StTensor>& out, std::string& err) {
  Json j{json, json + len, {}};
  if (!j.expect('{')) {
    err = "header: " + j.err;
    return false;
  }
  if (j.peek('}')) return true;
  for (;;) {
    std::string name;
    if (!j.string(name) || !j.expect(':')) break;
    if (name == "__metadata__") {
      if (!j.skip_value()) break;
    } else {
      StTensor t;
      t.name = name;
      t.file = file;
      bool have_dtype = false, have_shape = false, have_off = false;
      if (!j.expect('{')) break;
      bool ok = true;
      if (!j.peek('}')) {
        for (;;) {
          std::string key;
          if (!j.string(key) || !j.expect(':')) {
            ok = false;
            break;
          }
          if (key == "dtype") {
            ok = j.string(t.dtype);
            have_dtype = true;
          } else if (key == "shape") {
            ok = j.int_array(t.shape);
            have_shape = true;
          } else if (key == "data_offsets") {
            std::vector<int64_t> o;
            ok = j.int_array(o);
            if (ok && (o.size() != 2 || o[0] < 0 || o[1] < o[0])) ok = j.fail("bad data_offsets of " + name);
            if (ok) {
              t.begin = static_cast<uint64_t>(o[0]);
              t.end = static_cast<uint64_t>(o[1]);
            }
            have_off = true;
          } else {
            ok = j.skip_value();
          }
          if (!ok) break;
          if (j.peek(',')) {
            ++j.p;
            continue;
          }
          ok = j.expect('}');
          break;
        }
      } else {
        ++j.p;
      }
      if (!ok) break;
      if (!have_dtype || !have_shape || !have_off) {
        err = "header: tensor " + name + " lacks dtype, shape or data_offsets";
        return false;
      }
      size_t n = 1;
      for (int64_t d : t.shape) {
        if (d < 0) {
          err = "header: negative dimension in " + name;
          return false;
        }
        n *= static_cast<size_t>(d);
      }
      const size_t es = dtype_size(t.dtype);
      if (es == 0) {
        err = "header: unknown dtype " + t.dtype + " of " + name;
        return false;
      }
      if (n * es != t.bytes()) {
        err = "header: " + name + " has " + std::to_string(t.bytes()) + " bytes for " + std::to_string(n) +
              " elements of " + t.dtype;
        return false;
      }
      out.push_back(t);
    }
    if (j.peek(',')) {
      ++j.p;
      continue;
    }
    if (!j.expect('}')) break;
    return true;
  }
  err = "header: " + (j.err.empty() ? std::string("malformed") : j.err);
  return false;
}

std::string st_engine_name(const std::string& name) {
  std::string n = name;
  for (const char* pre : {"model.language_model.", "language_model.model.", "language_model."}) {
    const size_t l = std::strlen(pre);
    if (n.compare(0, l, pre) == 0) {
      n = (std::strcmp(pre, "language_model.") == 0 ? "" : "model.") + n.substr(l);
      break;
    }
  }
  for (const char* keep : {"model.layers.", "model.embed_tokens.", "model.norm.", "lm_head."})
    if (n.compare(0, std::strlen(keep), keep) == 0) return n;
  return std::string();
}

StCheckpoint::~StCheckpoint() {
  for (auto& f : files)
    if (f.base) munmap(const_cast<unsigned char*>(f.base), f.size);
}

bool st_open(const std::vector<std::string>& paths, StCheckpoint& ck, std::string& err) {
  for (size_t i = 0; i < paths.size(); ++i) {
    StFile f;
    f.path = paths[i];
    const int fd = open(paths[i].c_str(), O_RDONLY);
    if (fd < 0) {
      err = "cannot open " + paths[i] + ": " + std::strerror(errno);
      return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
      close(fd);
      err = paths[i] + ": not a safetensors file (too short)";
      return false;
    }
    f.size = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
      err = "mmap " + paths[i] + ": " + std::strerror(errno);
      return false;
    }
    f.base = static_cast<const unsigned char*>(m);
    ck.files.push_back(f);
    uint64_t hlen = 0;
    for (int b = 0; b < 8; ++b) hlen |= static_cast<uint64_t>(f.base[b]) << (8 * b);
    if (hlen > f.size - 8) {
      err = paths[i] + ": header length beyond the file";
      return false;
    }
    ck.files.back().data_off = 8 + static_cast<size_t>(hlen);
    std::vector<StTensor> ts;
    if (!st_parse_header(reinterpret_cast<const char*>(f.base + 8), static_cast<size_t>(hlen), static_cast<int>(i),
                         ts, err)) {
      err = paths[i] + ": " + err;
      return false;
    }
    const size_t data = f.size - 8 - static_cast<size_t>(hlen);
    for (auto& t : ts) {
      if (t.end > data) {
        err = paths[i] + ": " + t.name + " lies beyond the end of the file";
        return false;
      }
      const std::string n = st_engine_name(t.name);
      if (n.empty()) {
        ck.ignored.push_back(t.name);
        continue;
      }
      if (ck.tensors.count(n)) {
        err = "tensor " + t.name + " appears twice (" + ck.files[ck.tensors[n].file].path + ", " + paths[i] + ")";
        return false;
      }
      ck.tensors[n] = t;
    }
  }
  return true;
}

}  // namespace iam
