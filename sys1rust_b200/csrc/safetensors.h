// Host-side reader of `model.safetensors`: the checkpoint access of the reference's
// `laya_core::Weights` (runtime/crates/laya-core/src/weights.rs:10-77), behind the C ABI's
// s1c_weights_* entry points.
//
// The file is memory-mapped read-only. Opening validates the whole layout eagerly, so a file cut
// short (an interrupted download) fails at open with its path and length, never later: an 8-byte
// little-endian header length, a JSON object header of that length, and for every tensor a dtype,
// a shape and [begin, end) data offsets whose spans tile the data region exactly, in order, with
// end - begin = elements x element size. Tensor data are then views into the mapping.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace s1c {
namespace st {

// ---- a minimal JSON reader for the header (objects, arrays, strings, numbers, literals) ------
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool is_int = false;
  int64_t ival = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // insertion order
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  Json parse_document() {
    Json v = value(0);
    ws();
    if (p_ != end_) fail("trailing characters after the header object");
    return v;
  }

 private:
  const char* p_;
  const char* end_;
  [[noreturn]] void fail(const std::string& m) { throw std::runtime_error("invalid header JSON: " + m); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r')) ++p_;
  }
  char peek() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) fail(std::string("expected '") + c + "'");
    ++p_;
  }
  Json value(int depth) {
    if (depth > 64) fail("nesting too deep");
    const char c = peek();
    if (c == '{') return object(depth);
    if (c == '[') return array(depth);
    if (c == '"') {
      Json j;
      j.kind = Json::Str;
      j.str = string();
      return j;
    }
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    return literal();
  }
  Json object(int depth) {
    Json j;
    j.kind = Json::Obj;
    expect('{');
    if (peek() == '}') {
      ++p_;
      return j;
    }
    for (;;) {
      if (peek() != '"') fail("expected a key");
      std::string k = string();
      expect(':');
      j.obj.emplace_back(std::move(k), value(depth + 1));
      const char c = peek();
      ++p_;
      if (c == '}') return j;
      if (c != ',') fail("expected ',' or '}'");
    }
  }
  Json array(int depth) {
    Json j;
    j.kind = Json::Arr;
    expect('[');
    if (peek() == ']') {
      ++p_;
      return j;
    }
    for (;;) {
      j.arr.push_back(value(depth + 1));
      const char c = peek();
      ++p_;
      if (c == ']') return j;
      if (c != ',') fail("expected ',' or ']'");
    }
  }
  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (end_ - p_ < 4) fail("short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    expect('"');
    std::string s;
    for (;;) {
      if (p_ >= end_) fail("unterminated string");
      const char c = *p_++;
      if (c == '"') return s;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') {
        s += c;
        continue;
      }
      if (p_ >= end_) fail("unterminated escape");
      const char e = *p_++;
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
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') fail("lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(s, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
  }
  Json number() {
    const char* b = p_;
    bool integral = true;
    if (*p_ == '-') ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                         *p_ == '-')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integral = false;
      ++p_;
    }
    const std::string tok(b, p_);
    Json j;
    j.kind = Json::Num;
    try {
      size_t used = 0;
      j.num = std::stod(tok, &used);
      if (used != tok.size()) fail("bad number");
      if (integral) {
        j.ival = std::stoll(tok, &used);
        j.is_int = used == tok.size();
      }
    } catch (const std::logic_error&) {
      fail("bad number '" + tok + "'");
    }
    return j;
  }
  Json literal() {
    auto take = [&](const char* w) {
      const size_t n = std::strlen(w);
      if ((size_t)(end_ - p_) >= n && std::strncmp(p_, w, n) == 0) {
        p_ += n;
        return true;
      }
      return false;
    };
    Json j;
    if (take("true")) {
      j.kind = Json::Bool;
      j.num = 1;
    } else if (take("false")) {
      j.kind = Json::Bool;
    } else if (take("null")) {
      j.kind = Json::Null;
    } else {
      fail("unexpected character");
    }
    return j;
  }
};

// ---- the checkpoint ----------------------------------------------------------------------
struct Tensor {
  std::string name;
  std::string dtype;  // safetensors dtype name: F64, F32, F16, BF16, I64, ...
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;  // byte offsets in the data region
};

inline int dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

// Headers above this length are refused (the safetensors format's own limit is 100 MB).
constexpr uint64_t kMaxHeader = 100000000ull;

class File {
 public:
  File() = default;
  File(const File&) = delete;
  File& operator=(const File&) = delete;
  ~File() {
    if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
    if (fd_ >= 0) close(fd_);
  }

  // Maps `path` and validates its layout; throws std::runtime_error with the reason.
  void open(const std::string& path) {
    path_ = path;
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) throw std::runtime_error(std::string("cannot open: ") + std::strerror(errno));
    struct stat sb;
    if (fstat(fd_, &sb) != 0) throw std::runtime_error(std::string("cannot stat: ") + std::strerror(errno));
    size_ = (size_t)sb.st_size;
    if (size_ > 0) {
      map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
      if (map_ == MAP_FAILED) throw std::runtime_error(std::string("cannot map: ") + std::strerror(errno));
    }
    validate();
  }

  size_t size() const { return size_; }
  const std::vector<Tensor>& tensors() const { return tensors_; }
  const uint8_t* data(const Tensor& t) const { return static_cast<const uint8_t*>(map_) + data_off_ + t.begin; }

 private:
  std::string path_;
  int fd_ = -1;
  void* map_ = nullptr;
  size_t size_ = 0;
  size_t data_off_ = 0;
  std::vector<Tensor> tensors_;

  void validate() {
    if (size_ < 8) throw std::runtime_error("the 8-byte header length is incomplete");
    uint64_t n = 0;
    std::memcpy(&n, map_, 8);  // little-endian on every supported host
    if (n > kMaxHeader) throw std::runtime_error("header length " + std::to_string(n) + " is too large");
    if (8 + n > size_)
      throw std::runtime_error("header of " + std::to_string(n) + " bytes runs past the end of the file");
    const char* h = static_cast<const char*>(map_) + 8;
    Json root = Parser(h, (size_t)n).parse_document();
    if (root.kind != Json::Obj) throw std::runtime_error("header is not a JSON object");
    data_off_ = 8 + (size_t)n;
    const size_t data_len = size_ - data_off_;
    for (auto& kv : root.obj) {
      if (kv.first == "__metadata__") continue;
      const Json& e = kv.second;
      if (e.kind != Json::Obj) throw std::runtime_error(kv.first + ": entry is not an object");
      Tensor t;
      t.name = kv.first;
      const Json *dt = nullptr, *sh = nullptr, *off = nullptr;
      for (auto& f : e.obj) {
        if (f.first == "dtype") dt = &f.second;
        else if (f.first == "shape") sh = &f.second;
        else if (f.first == "data_offsets") off = &f.second;
      }
      if (!dt || dt->kind != Json::Str || !dtype_size(dt->str))
        throw std::runtime_error(kv.first + ": missing or unknown dtype");
      t.dtype = dt->str;
      if (!sh || sh->kind != Json::Arr) throw std::runtime_error(kv.first + ": missing shape");
      uint64_t numel = 1;
      for (auto& d : sh->arr) {
        if (d.kind != Json::Num || !d.is_int || d.ival < 0) throw std::runtime_error(kv.first + ": bad shape");
        t.shape.push_back(d.ival);
        if (d.ival != 0 && numel > UINT64_MAX / (uint64_t)d.ival) throw std::runtime_error(kv.first + ": shape overflows");
        numel *= (uint64_t)d.ival;
      }
      if (!off || off->kind != Json::Arr || off->arr.size() != 2 || off->arr[0].kind != Json::Num ||
          off->arr[1].kind != Json::Num || !off->arr[0].is_int || !off->arr[1].is_int || off->arr[0].ival < 0 ||
          off->arr[1].ival < off->arr[0].ival)
        throw std::runtime_error(kv.first + ": bad data_offsets");
      t.begin = (size_t)off->arr[0].ival;
      t.end = (size_t)off->arr[1].ival;
      if ((uint64_t)(t.end - t.begin) != numel * (uint64_t)dtype_size(t.dtype))
        throw std::runtime_error(kv.first + ": data_offsets do not match dtype x shape");
      tensors_.push_back(std::move(t));
    }
    // The spans must tile the data region: sorted by offset, each starts where the previous
    // ended, and the last ends at the end of the file.
    std::vector<const Tensor*> order;
    for (auto& t : tensors_) order.push_back(&t);
    std::sort(order.begin(), order.end(), [](const Tensor* a, const Tensor* b) { return a->begin < b->begin; });
    size_t at = 0;
    for (const Tensor* t : order) {
      if (t->begin != at) throw std::runtime_error(t->name + ": data_offsets leave a gap or overlap");
      at = t->end;
    }
    if (at != data_len)
      throw std::runtime_error("the header describes " + std::to_string(at) + " data bytes, the file holds " +
                               std::to_string(data_len));
  }
};

}  // namespace st
}  // namespace s1c
