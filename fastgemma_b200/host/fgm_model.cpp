// .fgm model files: see fgm_model.hpp.

#include "fgm_model.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "fgm_cuda.h"

namespace fgm_core {

namespace k = fgm_kernels;

namespace {

[[noreturn]] void bad(const std::string &msg) { throw k::Error(FGM_CUDA_EINVAL, msg); }

// Recursive-descent JSON reader over [p, end).
class JsonReader {
 public:
  JsonReader(const char *p, size_t n) : p_(p), end_(p + n) {}

  Json document() {
    Json v = value(0);
    ws();
    if (p_ != end_) bad("fgm header: trailing bytes after the JSON value");
    return v;
  }

 private:
  static constexpr int kMaxDepth = 64;
  const char *p_, *end_;

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
  }
  char peek() {
    ws();
    if (p_ >= end_) bad("fgm header: unexpected end of JSON");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) bad(std::string("fgm header: expected '") + c + "'");
    p_++;
  }
  void literal(const char *word) {
    const size_t n = std::strlen(word);
    if ((size_t)(end_ - p_) < n || std::memcmp(p_, word, n) != 0) bad("fgm header: bad literal");
    p_ += n;
  }

  Json value(int depth) {
    if (depth > kMaxDepth) bad("fgm header: JSON nested too deeply");
    Json v;
    switch (peek()) {
      case '{': {
        p_++;
        v.kind = Json::Object;
        if (peek() == '}') {
          p_++;
          return v;
        }
        for (;;) {
          if (peek() != '"') bad("fgm header: object key must be a string");
          std::string key = string();
          expect(':');
          v.obj[key] = value(depth + 1);
          const char c = peek();
          p_++;
          if (c == '}') return v;
          if (c != ',') bad("fgm header: expected ',' or '}'");
        }
      }
      case '[': {
        p_++;
        v.kind = Json::Array;
        if (peek() == ']') {
          p_++;
          return v;
        }
        for (;;) {
          v.arr.push_back(value(depth + 1));
          const char c = peek();
          p_++;
          if (c == ']') return v;
          if (c != ',') bad("fgm header: expected ',' or ']'");
        }
      }
      case '"':
        v.kind = Json::String;
        v.str = string();
        return v;
      case 't':
        literal("true");
        v.kind = Json::Bool;
        v.b = true;
        return v;
      case 'f':
        literal("false");
        v.kind = Json::Bool;
        return v;
      case 'n':
        literal("null");
        return v;
      default:
        v.kind = Json::Number;
        v.num = number();
        return v;
    }
  }

  double number() {
    const char *s = p_;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) p_++;
    while (p_ < end_ && (std::isdigit((unsigned char)*p_) || *p_ == '.' || *p_ == 'e' ||
                         *p_ == 'E' || *p_ == '-' || *p_ == '+'))
      p_++;
    const std::string text(s, p_);
    if (text.empty()) bad("fgm header: unexpected character in JSON");
    char *stop = nullptr;
    const double d = std::strtod(text.c_str(), &stop);
    if (stop != text.c_str() + text.size()) bad("fgm header: bad number '" + text + "'");
    return d;
  }

  static void utf8(std::string &out, uint32_t cp) {
    if (cp < 0x80) {
      out += (char)cp;
    } else if (cp < 0x800) {
      out += (char)(0xC0 | (cp >> 6));
      out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += (char)(0xE0 | (cp >> 12));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    } else {
      out += (char)(0xF0 | (cp >> 18));
      out += (char)(0x80 | ((cp >> 12) & 0x3F));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    }
  }

  uint32_t hex4() {
    if (end_ - p_ < 4) bad("fgm header: short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; i++) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else bad("fgm header: bad \\u escape");
    }
    return v;
  }

  std::string string() {
    expect('"');
    std::string out;
    for (;;) {
      if (p_ >= end_) bad("fgm header: unterminated string");
      const char c = *p_++;
      if (c == '"') return out;
      if ((unsigned char)c < 0x20) bad("fgm header: control character in string");
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= end_) bad("fgm header: unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') bad("fgm header: lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) bad("fgm header: bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(out, cp);
          break;
        }
        default:
          bad("fgm header: bad escape");
      }
    }
  }
};

size_t as_size(const Json &v, const std::string &what) {
  if (v.kind != Json::Number || v.num < 0 || v.num != std::floor(v.num) || v.num > 9.0e15)
    bad("fgm header: " + what + " is not a non-negative integer");
  return (size_t)v.num;
}

// meta[key] as an unsigned integer, or `dflt` when absent (model.rs:173-175)
size_t meta_uint(const Json &meta, const char *key, size_t dflt) {
  const Json *v = meta.find(key);
  if (!v || v->kind != Json::Number || v->num < 0) return dflt;
  return (size_t)v->num;
}

}  // namespace

const Json *Json::find(const std::string &key) const {
  if (kind != Object) return nullptr;
  auto it = obj.find(key);
  return it == obj.end() ? nullptr : &it->second;
}

Json Json::parse(const char *text, size_t len) { return JsonReader(text, len).document(); }

std::unique_ptr<Model> Model::open(const std::string &path) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) throw k::Error(FGM_CUDA_EINVAL, path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int e = errno;
    ::close(fd);
    throw k::Error(FGM_CUDA_EINVAL, path + ": " + std::strerror(e));
  }
  const size_t size = (size_t)st.st_size;
  if (size < 12) {
    ::close(fd);
    bad(path + ": not a .fgm file (too short)");
  }
  void *m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  const int merr = errno;
  ::close(fd);  // the mapping keeps the file
  if (m == MAP_FAILED) throw k::Error(FGM_CUDA_EINVAL, path + ": mmap: " + std::strerror(merr));
  std::unique_ptr<Model> model(new Model());
  model->base_ = static_cast<const uint8_t *>(m);
  model->size_ = size;

  const uint8_t *b = model->base_;
  if (std::memcmp(b, "FASTGEM1", 8) != 0) bad(path + ": not a .fgm file");
  const uint32_t hlen = (uint32_t)b[8] | ((uint32_t)b[9] << 8) | ((uint32_t)b[10] << 16) |
                        ((uint32_t)b[11] << 24);
  if ((size_t)hlen > size - 12) bad(path + ": header length past the end of the file");
  const Json h = Json::parse(reinterpret_cast<const char *>(b + 12), hlen);
  if (h.kind != Json::Object) bad(path + ": header is not a JSON object");
  const Json *cfg = h.find("config");
  if (!cfg) bad(path + ": header has no config");
  model->config_ = *cfg;
  if (const Json *meta = h.find("meta")) model->meta_ = *meta;
  const Json *tensors = h.find("tensors");
  if (!tensors || tensors->kind != Json::Object) bad(path + ": header has no tensors object");
  for (const auto &kv : tensors->obj) {
    const Json &t = kv.second;
    TensorEntry e;
    const Json *dt = t.find("dtype"), *sh = t.find("shape"), *off = t.find("offset"),
               *nb = t.find("nbytes");
    if (!dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off || !nb)
      bad(path + ": tensor " + kv.first + " lacks dtype / shape / offset / nbytes");
    e.dtype = dt->str;
    for (const Json &d : sh->arr) e.shape.push_back(as_size(d, kv.first + " shape"));
    e.offset = as_size(*off, kv.first + " offset");
    e.nbytes = as_size(*nb, kv.first + " nbytes");
    if (e.offset > size || e.nbytes > size - e.offset)
      bad(path + ": tensor " + kv.first + " lies past the end of the file");
    if (const Json *meta = t.find("meta")) e.meta = *meta;
    model->tensors_.emplace(kv.first, std::move(e));
  }
  return model;
}

Model::~Model() {
  if (base_) munmap(const_cast<uint8_t *>(base_), size_);
}

bool Model::has(const std::string &name) const { return tensors_.count(name) != 0; }

const TensorEntry &Model::entry(const std::string &name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) bad("missing tensor " + name);
  return it->second;
}

const std::vector<size_t> &Model::shape(const std::string &name) const {
  return entry(name).shape;
}

const uint8_t *Model::raw(const std::string &name, size_t *nbytes) const {
  const TensorEntry &e = entry(name);
  *nbytes = e.nbytes;
  return base_ + e.offset;
}

k::Slice<const uint8_t> Model::u8s(const std::string &name) const {
  size_t n;
  const uint8_t *p = raw(name, &n);
  return {p, n};
}

k::Slice<const int8_t> Model::i8s(const std::string &name) const {
  size_t n;
  const uint8_t *p = raw(name, &n);
  return {reinterpret_cast<const int8_t *>(p), n};
}

k::Slice<const k::f16> Model::f16s(const std::string &name) const {
  size_t n;
  const uint8_t *p = raw(name, &n);
  return {reinterpret_cast<const k::f16 *>(p), n / 2};
}

k::Slice<const float> Model::f32s(const std::string &name) const {
  size_t n;
  const uint8_t *p = raw(name, &n);
  return {reinterpret_cast<const float *>(p), n / 4};
}

QLinear Model::linear(const std::string &name) const {
  const TensorEntry &e = entry(name);
  if (e.dtype != "q4g" && e.dtype != "q8c") bad("tensor " + name + " has non-linear dtype " + e.dtype);
  if (e.shape.size() < 2) bad("tensor " + name + " is not a matrix");
  QLinear w;
  w.n = e.shape[0];
  w.k = e.shape[1];
  w.hadamard = meta_uint(e.meta, "hadamard", 0);
  if (e.dtype == "q4g") {
    const auto q = u8s(name);
    const auto s = f16s(name + ".scale");
    w.bits = 4;
    w.q4 = q.ptr;
    w.q4_len = q.len;
    w.s4 = s.ptr;
    w.s4_len = s.len;
    w.group = meta_uint(e.meta, "group", 64);
  } else if (e.dtype == "q8c") {
    const auto q = i8s(name);
    const auto s = f32s(name + ".scale");
    w.bits = 8;
    w.q8 = q.ptr;
    w.q8_len = q.len;
    w.s8 = s.ptr;
    w.s8_len = s.len;
    w.group = 0;
  } else {
    bad("tensor " + name + " has non-linear dtype " + e.dtype);
  }
  return w;
}

DualW Model::dual(const std::string &name) const {
  const std::string alt = name + ".i8";
  if (!has(alt)) return DualW(linear(name));
  const QLinear hi = linear(alt);
  return DualW(linear(name), &hi);
}

size_t Model::total_bytes() const {
  size_t t = 0;
  for (const auto &kv : tensors_) t += kv.second.nbytes;
  return t;
}

size_t Model::register_linears() const {
  size_t bytes = 0;
  for (const auto &kv : tensors_) {
    const TensorEntry &e = kv.second;
    if (e.dtype != "q4g" && e.dtype != "q8c") continue;
    k::register_blob(base_ + e.offset, e.nbytes);
    bytes += e.nbytes;
    auto sc = tensors_.find(kv.first + ".scale");
    if (sc != tensors_.end()) {
      k::register_blob(base_ + sc->second.offset, sc->second.nbytes);
      bytes += sc->second.nbytes;
    }
  }
  return bytes;
}

void Model::unregister_linears() const {
  for (const auto &kv : tensors_) {
    const TensorEntry &e = kv.second;
    if (e.dtype != "q4g" && e.dtype != "q8c") continue;
    if (e.nbytes) k::unregister_blob(base_ + e.offset);
    auto sc = tensors_.find(kv.first + ".scale");
    if (sc != tensors_.end() && sc->second.nbytes) k::unregister_blob(base_ + sc->second.offset);
  }
}

}  // namespace fgm_core
