// Checkpoints of a model's parameters, straight from and to its device
// buffers, in go-tensor's two formats:
//
//   safetensors  weights/safetensors/safetensors.go:55-175 (Decode, Encode)
//                with nn/state.go:84-126 (LoadStateDict) for loading by name;
//   GOTN v1      nn/serialize.go:11-89 (positional float64 values).
//
// The reference writes a checkpoint by copying every parameter to the host
// as float64 (Tensor.Float64s) and encoding from there; here the flat
// parameter buffer comes back in one device-to-host copy in the model's dtype
// and is encoded directly, and loading decodes into one host buffer uploaded
// in the same way. The bytes written and the values loaded are the
// reference's: tensors in byte-sorted name order, the header as Go's
// encoding/json writes it, F32 values rounded from the parameters like
// float32(v).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "model.hpp"

namespace gotensor {

namespace {

// ---- Go's JSON string escaping (encoding/json, HTML-safe, Go 1.23) ----------

std::string go_json_string(const std::string& s) {
  static const char* hex = "0123456789abcdef";
  std::string out = "\"";
  size_t i = 0;
  while (i < s.size()) {
    const unsigned char c = (unsigned char)s[i];
    if (c < 0x80) {
      switch (c) {
        case '"': out += "\\\""; break;
        case '\\': out += "\\\\"; break;
        case '\b': out += "\\b"; break;
        case '\f': out += "\\f"; break;
        case '\n': out += "\\n"; break;
        case '\r': out += "\\r"; break;
        case '\t': out += "\\t"; break;
        default:
          if (c < 0x20 || c == '<' || c == '>' || c == '&') {
            out += "\\u00";
            out += hex[c >> 4];
            out += hex[c & 15];
          } else {
            out += (char)c;
          }
      }
      i++;
      continue;
    }
    // one well-formed UTF-8 sequence, else U+FFFD for this byte
    int n = (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 0;
    uint32_t cp = n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
    bool ok = n > 0 && i + n <= s.size();
    for (int k = 1; ok && k < n; k++) {
      const unsigned char d = (unsigned char)s[i + k];
      ok = (d & 0xC0) == 0x80;
      cp = (cp << 6) | (d & 0x3F);
    }
    if (ok) {  // reject overlong forms, surrogates and values past U+10FFFF
      ok = !((n == 2 && cp < 0x80) || (n == 3 && cp < 0x800) || (n == 4 && cp < 0x10000) ||
             (cp >= 0xD800 && cp <= 0xDFFF) || cp > 0x10FFFF);
    }
    if (!ok) {
      out += "\\ufffd";
      i++;
      continue;
    }
    if (cp == 0x2028 || cp == 0x2029) {
      out += cp == 0x2028 ? "\\u2028" : "\\u2029";
    } else {
      out.append(s, i, n);
    }
    i += n;
  }
  return out + "\"";
}

// ---- a JSON reader for safetensors headers ----------------------------------

struct JVal {
  enum Kind { OBJ, ARR, STR, NUM, LIT } kind = LIT;
  std::string str;                              // STR, or NUM's text
  std::vector<std::pair<std::string, JVal>> obj;  // in file order
  std::vector<JVal> arr;
};

class JsonReader {
 public:
  JsonReader(const char* p, const char* end) : p_(p), end_(end) {}
  JVal parse_document() {
    JVal v = value(0);
    ws();
    if (p_ != end_) fail("trailing data after the header object");
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const std::string& what) { throw Error("safetensors: header: " + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
  }
  char peek() {
    ws();
    if (p_ >= end_) fail("unexpected end of JSON input");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) fail(std::string("expected '") + c + "'");
    p_++;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (end_ - p_ < 4) fail("bad \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; k++) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    expect('"');
    std::string o;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      const char c = *p_++;
      if (c == '"') return o;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p_ >= end_) fail("unterminated string");
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
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            const char* save = p_;
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo >= 0xDC00 && lo < 0xE000) {
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            } else {
              p_ = save;
              cp = 0xFFFD;
            }
          } else if (cp >= 0xD800 && cp < 0xE000) {
            cp = 0xFFFD;
          }
          put_utf8(o, cp);
          break;
        }
        default: fail("bad escape in string");
      }
    }
  }
  JVal value(int depth) {
    if (depth > 64) fail("nesting too deep");
    JVal v;
    const char c = peek();
    if (c == '{') {
      p_++;
      v.kind = JVal::OBJ;
      if (peek() == '}') {
        p_++;
        return v;
      }
      while (true) {
        std::string k = string();
        expect(':');
        v.obj.emplace_back(std::move(k), value(depth + 1));
        const char d = peek();
        p_++;
        if (d == '}') return v;
        if (d != ',') fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      p_++;
      v.kind = JVal::ARR;
      if (peek() == ']') {
        p_++;
        return v;
      }
      while (true) {
        v.arr.push_back(value(depth + 1));
        const char d = peek();
        p_++;
        if (d == ']') return v;
        if (d != ',') fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = JVal::STR;
      v.str = string();
      return v;
    }
    if (c == '-' || (c >= '0' && c <= '9')) {
      v.kind = JVal::NUM;
      const char* s = p_;
      if (*p_ == '-') p_++;
      while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                           *p_ == '-'))
        p_++;
      v.str.assign(s, p_);
      return v;
    }
    for (const char* lit : {"true", "false", "null"}) {
      const size_t n = strlen(lit);
      if ((size_t)(end_ - p_) >= n && memcmp(p_, lit, n) == 0) {
        p_ += n;
        v.kind = JVal::LIT;
        v.str = lit;
        return v;
      }
    }
    fail("invalid character in header");
  }
};

// An integer JSON number (Go rejects fractions and exponents for int fields).
int64_t json_int(const JVal& v, const std::string& what) {
  if (v.kind != JVal::NUM) throw Error(what + ": not a number");
  const std::string& t = v.str;
  size_t i = t[0] == '-' ? 1 : 0;
  if (i >= t.size()) throw Error(what + ": bad number " + t);
  for (size_t k = i; k < t.size(); k++)
    if (t[k] < '0' || t[k] > '9') throw Error(what + ": cannot read " + t + " as an integer");
  if (t.size() - i > 18) throw Error(what + ": number " + t + " out of range");
  return std::stoll(t);
}

// ---- element kinds (internal/dtype/dtype.go:41-128) -------------------------

int kind_size(const std::string& k) {
  if (k == "F64" || k == "I64" || k == "U64") return 8;
  if (k == "F32" || k == "I32" || k == "U32") return 4;
  if (k == "F16" || k == "BF16" || k == "I16" || k == "U16") return 2;
  if (k == "I8" || k == "U8" || k == "BOOL") return 1;
  return 0;
}

template <typename U>
U load_le(const unsigned char* p) {
  U v = 0;
  for (size_t b = 0; b < sizeof(U); b++) v |= (U)p[b] << (8 * b);
  return v;
}

double half_to_double(uint16_t h) {
  const int exp = (h >> 10) & 0x1F;
  const double frac = (double)(h & 0x3FF);
  double v;
  if (exp == 0) {
    v = std::ldexp(frac, -24);
  } else if (exp == 0x1F) {
    v = frac == 0 ? INFINITY : NAN;
  } else {
    v = std::ldexp(frac + 1024, exp - 25);
  }
  return (h & 0x8000) ? -v : v;
}

double decode_elem(const std::string& k, const unsigned char* p) {
  if (k == "F64") {
    const uint64_t b = load_le<uint64_t>(p);
    double d;
    memcpy(&d, &b, 8);
    return d;
  }
  if (k == "F32" || k == "BF16") {
    const uint32_t b = k == "F32" ? load_le<uint32_t>(p) : (uint32_t)load_le<uint16_t>(p) << 16;
    float f;
    memcpy(&f, &b, 4);
    return (double)f;
  }
  if (k == "F16") return half_to_double(load_le<uint16_t>(p));
  if (k == "I64") return (double)(int64_t)load_le<uint64_t>(p);
  if (k == "I32") return (double)(int32_t)load_le<uint32_t>(p);
  if (k == "I16") return (double)(int16_t)load_le<uint16_t>(p);
  if (k == "I8") return (double)(int8_t)p[0];
  if (k == "U64") return (double)load_le<uint64_t>(p);
  if (k == "U32") return (double)load_le<uint32_t>(p);
  if (k == "U16") return (double)load_le<uint16_t>(p);
  if (k == "U8") return (double)p[0];
  return p[0] != 0 ? 1.0 : 0.0;  // BOOL
}

static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "the file formats are little-endian, like this host");

// n elements of kind k at src, converted to T (through float64, as the
// reference converts); the kind is resolved once per tensor.
template <typename T>
void decode_into(const std::string& k, const unsigned char* src, int64_t n, T* dst) {
  if (k == "F32") {
    if (sizeof(T) == 4) {
      memcpy(dst, src, 4 * n);
    } else {
      for (int64_t i = 0; i < n; i++) {
        float f;
        memcpy(&f, src + 4 * i, 4);
        dst[i] = (T)(double)f;
      }
    }
  } else if (k == "F64") {
    if (sizeof(T) == 8) {
      memcpy(dst, src, 8 * n);
    } else {
      for (int64_t i = 0; i < n; i++) {
        double d;
        memcpy(&d, src + 8 * i, 8);
        dst[i] = (T)d;
      }
    }
  } else {
    const int sz = kind_size(k);
    for (int64_t i = 0; i < n; i++) dst[i] = (T)decode_elem(k, src + i * sz);
  }
}

constexpr uint64_t kMaxHeader = 100ull << 20;   // safetensors.go:18-19
constexpr int64_t kMaxElements = 1ll << 34;      // dtype.go:130-132

std::string shape_str(const std::vector<int64_t>& s) {  // Go's %v of a []int
  std::string o = "[";
  for (size_t i = 0; i < s.size(); i++) o += (i ? " " : "") + std::to_string(s[i]);
  return o + "]";
}

// A file mapped read-only (no copy of its bytes; tmpfs and page-cache pages
// are used in place).
class MappedFile {
 public:
  explicit MappedFile(const std::string& path) {
    const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw Error("open " + path + ": " + strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
      const int e = errno;
      close(fd);
      throw Error("stat " + path + ": " + strerror(e));
    }
    size_ = (size_t)st.st_size;
    if (size_ > 0) {
      void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
      if (p == MAP_FAILED) {
        const int e = errno;
        close(fd);
        throw Error("mmap " + path + ": " + strerror(e));
      }
      data_ = (const unsigned char*)p;
    }
    close(fd);
  }
  ~MappedFile() {
    if (data_) munmap((void*)data_, size_);
  }
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  const unsigned char* data() const { return data_; }
  size_t size() const { return size_; }

 private:
  const unsigned char* data_ = nullptr;
  size_t size_ = 0;
};

// A decoded safetensors file: entries point into the file's bytes.
struct StEntry {
  std::string kind;
  std::vector<int64_t> shape;
  int64_t numel = 0;
  const unsigned char* data = nullptr;
};

struct StFile {
  std::shared_ptr<MappedFile> file;
  std::map<std::string, StEntry> tensors;
  std::vector<std::pair<std::string, std::string>> metadata;
};

// Decode (safetensors.go:55-100): every entry is checked, used or not.
StFile st_decode(std::shared_ptr<MappedFile> b) {
  StFile f;
  f.file = std::move(b);
  const MappedFile& by = *f.file;
  if (by.size() < 8) throw Error("safetensors: file too short");
  const uint64_t n = load_le<uint64_t>(by.data());
  if (n > kMaxHeader || n > by.size() - 8) throw Error("safetensors: invalid header length " + std::to_string(n));
  JsonReader r((const char*)by.data() + 8, (const char*)by.data() + 8 + n);
  JVal root = r.parse_document();
  if (root.kind != JVal::OBJ) throw Error("safetensors: header: not a JSON object");
  const unsigned char* body = by.data() + 8 + n;
  const int64_t body_len = (int64_t)(by.size() - 8 - n);
  std::map<std::string, const JVal*> last;  // a repeated key: the last one counts
  for (auto& kv : root.obj) last[kv.first] = &kv.second;
  for (auto& kv : last) {
    const std::string& name = kv.first;
    const JVal& v = *kv.second;
    if (name == "__metadata__") {
      if (v.kind == JVal::LIT && v.str == "null") continue;
      if (v.kind != JVal::OBJ) throw Error("safetensors: __metadata__: not an object of strings");
      std::map<std::string, std::string> m;
      for (auto& e : v.obj) {
        if (e.second.kind != JVal::STR) throw Error("safetensors: __metadata__: not an object of strings");
        m[e.first] = e.second.str;
      }
      f.metadata.assign(m.begin(), m.end());
      continue;
    }
    const std::string q = "safetensors: tensor \"" + name + "\"";
    if (v.kind != JVal::OBJ) throw Error(q + ": not an object");
    StEntry e;
    const JVal *dt = nullptr, *shape = nullptr, *offs = nullptr;
    for (auto& field : v.obj) {
      if (field.first == "dtype") dt = &field.second;
      if (field.first == "shape") shape = &field.second;
      if (field.first == "data_offsets") offs = &field.second;
    }
    if (dt && dt->kind != JVal::STR && !(dt->kind == JVal::LIT && dt->str == "null"))
      throw Error(q + ": dtype is not a string");
    e.kind = dt && dt->kind == JVal::STR ? dt->str : "";
    const int size = kind_size(e.kind);
    if (!size) throw Error(q + " has unsupported dtype " + e.kind);
    if (shape && shape->kind == JVal::ARR)
      for (auto& d : shape->arr) e.shape.push_back(json_int(d, q + ": shape"));
    else if (shape && !(shape->kind == JVal::LIT && shape->str == "null"))
      throw Error(q + ": shape is not an array");
    int64_t numel = 1;
    for (int64_t d : e.shape) {
      if (d < 0) throw Error(q + ": negative dimension in shape " + shape_str(e.shape));
      if (d != 0 && numel > kMaxElements / d)
        throw Error(q + ": shape " + shape_str(e.shape) + " has more than " + std::to_string(kMaxElements) +
                    " elements");
      numel *= d;
    }
    e.numel = numel;
    int64_t start = 0, end = 0;
    if (offs && offs->kind == JVal::ARR) {
      if (offs->arr.size() > 0) start = json_int(offs->arr[0], q + ": data_offsets");
      if (offs->arr.size() > 1) end = json_int(offs->arr[1], q + ": data_offsets");
    } else if (offs && !(offs->kind == JVal::LIT && offs->str == "null")) {
      throw Error(q + ": data_offsets is not an array");
    }
    if (start < 0 || end < start || end > body_len || end - start != numel * size)
      throw Error(q + " has invalid data offsets [" + std::to_string(start) + " " + std::to_string(end) + "]");
    e.data = body + start;
    f.tensors[name] = std::move(e);
  }
  return f;
}

}  // namespace

char* Model::param_staging() {
  if (!staging_) check(gt_host_alloc(dev_params_ * es_, &staging_));
  return (char*)staging_;
}

namespace {

// Writes n values of a parameter (model dtype, es bytes each) as `size`-byte
// values: the bytes as they are when the widths match, else converted in
// chunks (float32(v) rounds to nearest).
void write_values(FILE* f, const char* src, int64_t n, size_t es, int size, const std::string& path) {
  if ((size_t)size == es) {
    if (n && fwrite(src, es, n, f) != (size_t)n) throw Error("write " + path + ": " + strerror(errno));
    return;
  }
  std::vector<unsigned char> buf(std::min<int64_t>(n, 1 << 16) * size);
  for (int64_t at = 0; at < n; at += 1 << 16) {
    const int64_t m = std::min<int64_t>(n - at, 1 << 16);
    for (int64_t i = 0; i < m; i++) {
      if (size == 8) {
        const double v = (double)((const float*)src)[at + i];
        memcpy(buf.data() + 8 * i, &v, 8);
      } else {
        const float v = (float)((const double*)src)[at + i];
        memcpy(buf.data() + 4 * i, &v, 4);
      }
    }
    if (fwrite(buf.data(), size, m, f) != (size_t)m) throw Error("write " + path + ": " + strerror(errno));
  }
}

}  // namespace

void Model::save_safetensors(const std::string& path, const std::string& dt,
                             const std::vector<std::pair<std::string, std::string>>& metadata) {
  if (dt != "F32" && dt != "F64") throw Error("safetensors: unsupported output dtype \"" + dt + "\"");
  std::vector<const ParamInfo*> order;
  for (auto& p : params_) {
    if (p.name == "__metadata__") throw Error("safetensors: \"__metadata__\" is a reserved name");
    order.push_back(&p);
  }
  std::sort(order.begin(), order.end(), [](const ParamInfo* a, const ParamInfo* b) { return a->name < b->name; });
  const int size = dt == "F64" ? 8 : 4;
  std::map<std::string, std::string> header;  // key -> JSON value; std::string order is byte order
  int64_t at = 0;
  for (const ParamInfo* p : order) {
    std::string shp;
    for (size_t d = 0; d < p->shape.size(); d++) shp += (d ? "," : "") + std::to_string(p->shape[d]);
    header[p->name] = "{\"dtype\":\"" + dt + "\",\"shape\":[" + shp + "],\"data_offsets\":[" + std::to_string(at) +
                      "," + std::to_string(at + p->numel * size) + "]}";
    at += p->numel * size;
  }
  if (!metadata.empty()) {
    std::map<std::string, std::string> m(metadata.begin(), metadata.end());
    std::string o = "{";
    for (auto& kv : m) o += (o.size() > 1 ? "," : "") + go_json_string(kv.first) + ":" + go_json_string(kv.second);
    header["__metadata__"] = o + "}";
  }
  std::string h = "{";
  for (auto& kv : header) h += (h.size() > 1 ? "," : "") + go_json_string(kv.first) + ":" + kv.second;
  h += "}";
  h.append((8 - h.size() % 8) % 8, ' ');
  std::string head(8, '\0');
  for (int k = 0; k < 8; k++) head[k] = (char)((uint64_t)h.size() >> (8 * k));
  char* stage = param_staging();
  check(gt_download(ctx_, stage, pbuf_.get(), dev_params_ * es_));  // one copy of the flat buffer
  std::unique_ptr<FILE, int (*)(FILE*)> f(fopen(path.c_str(), "wb"), fclose);
  if (!f) throw Error("open " + path + ": " + strerror(errno));
  head += h;
  if (fwrite(head.data(), 1, head.size(), f.get()) != head.size()) throw Error("write " + path + ": " + strerror(errno));
  for (const ParamInfo* p : order) write_values(f.get(), stage + p->dev_offset * es_, p->numel, es_, size, path);
  if (fflush(f.get()) != 0) throw Error("write " + path + ": " + strerror(errno));
}

void Model::load_safetensors(const std::string& path, bool strict) {
  StFile f;
  try {
    f = st_decode(std::make_shared<MappedFile>(path));
  } catch (const Error& e) {
    throw Error(path + ": " + e.what());
  }
  // LoadStateDict (nn/state.go:84-126): all or nothing.
  std::vector<std::string> missing;
  std::vector<std::pair<const ParamInfo*, const StEntry*>> load;
  for (auto& p : params_) {
    auto it = f.tensors.find(p.name);
    if (it == f.tensors.end()) {
      missing.push_back(p.name);
      continue;
    }
    if (it->second.shape != p.shape)
      throw Error("nn: " + p.name + " has shape " + shape_str(it->second.shape) + " in the state dict but " +
                  shape_str(p.shape) + " in the model");
    load.emplace_back(&p, &it->second);
  }
  if (strict) {
    std::vector<std::string> unexpected;
    for (auto& kv : f.tensors) {
      bool known = false;
      for (auto& p : params_) known |= p.name == kv.first;
      if (!known) unexpected.push_back(kv.first);  // std::map order: sorted
    }
    if (!missing.empty() || !unexpected.empty()) {
      std::string msg = "nn: state dict does not match model: ";
      auto join = [](const std::vector<std::string>& v) {
        std::string o;
        for (size_t i = 0; i < v.size(); i++) o += (i ? ", " : "") + v[i];
        return o;
      };
      if (!missing.empty()) msg += "missing keys: " + join(missing);
      if (!unexpected.empty()) msg += std::string(missing.empty() ? "" : "; ") + "unexpected keys: " + join(unexpected);
      throw Error(msg);
    }
  }
  char* stage = param_staging();
  check(gt_download(ctx_, stage, pbuf_.get(), dev_params_ * es_));  // what is not loaded keeps its value
  for (auto& pe : load) {
    const ParamInfo* p = pe.first;
    const StEntry* e = pe.second;
    if (dtype_ == GT_FLOAT64)
      decode_into(e->kind, e->data, p->numel, (double*)(stage + p->dev_offset * es_));
    else  // CopyFrom's cast to float32
      decode_into(e->kind, e->data, p->numel, (float*)(stage + p->dev_offset * es_));
  }
  check(gt_upload(ctx_, pbuf_.get(), stage, dev_params_ * es_));
}

void Model::save_gotn(const std::string& path) {
  char* stage = param_staging();
  check(gt_download(ctx_, stage, pbuf_.get(), dev_params_ * es_));
  std::unique_ptr<FILE, int (*)(FILE*)> f(fopen(path.c_str(), "wb"), fclose);
  if (!f) throw Error("open " + path + ": " + strerror(errno));
  auto put = [&](const void* b, size_t n) {
    if (fwrite(b, 1, n, f.get()) != n) throw Error("write " + path + ": " + strerror(errno));
  };
  auto u32 = [&](uint32_t v) { put(&v, 4); };
  put("GOTN", 4);
  u32(1);  // version
  u32((uint32_t)params_.size());
  for (auto& p : params_) {  // Parameters() order: rank, dims, float64 values
    u32((uint32_t)p.shape.size());
    for (int64_t d : p.shape) u32((uint32_t)d);
    write_values(f.get(), stage + p.dev_offset * es_, p.numel, es_, 8, path);
  }
  if (fflush(f.get()) != 0) throw Error("write " + path + ": " + strerror(errno));
}

void Model::load_gotn(const std::string& path) {
  const MappedFile file(path);
  const unsigned char* b = file.data();
  const size_t size = file.size();
  size_t at = 0;
  auto take = [&](size_t n, const std::string& what) {
    if (size - at < n) throw Error(what + ": unexpected EOF");
    const unsigned char* p = b + at;
    at += n;
    return p;
  };
  if (size < 4) throw Error("nn: read header: unexpected EOF");
  if (memcmp(b, "GOTN", 4) != 0) throw Error("nn: not a go-tensor model file");
  at = 4;
  const uint32_t version = load_le<uint32_t>(take(4, "nn"));
  if (version != 1) throw Error("nn: unsupported model file version " + std::to_string(version));
  const uint32_t count = load_le<uint32_t>(take(4, "nn"));
  if (count != params_.size())
    throw Error("nn: file has " + std::to_string(count) + " parameters, module has " +
                std::to_string(params_.size()));
  // Every record is checked before any value is used: nothing changes unless
  // the whole file is good.
  std::vector<const unsigned char*> values(params_.size());
  for (size_t i = 0; i < params_.size(); i++) {
    const ParamInfo& p = params_[i];
    const uint32_t rank = load_le<uint32_t>(take(4, "nn: parameter " + std::to_string(i)));
    std::vector<int64_t> dims;
    const unsigned char* dp = take(4ull * rank, "nn: parameter " + std::to_string(i));
    for (uint32_t d = 0; d < rank; d++) dims.push_back(load_le<uint32_t>(dp + 4 * d));
    if (dims != p.shape)
      throw Error("nn: parameter " + std::to_string(i) + " has shape " + shape_str(dims) + " in file, " +
                  shape_str(p.shape) + " in module");
    values[i] = take(8ull * p.numel, "nn: parameter " + std::to_string(i));
  }
  char* stage = param_staging();
  check(gt_download(ctx_, stage, pbuf_.get(), dev_params_ * es_));
  for (size_t i = 0; i < params_.size(); i++) {
    const ParamInfo& p = params_[i];
    if (dtype_ == GT_FLOAT64)
      decode_into("F64", values[i], p.numel, (double*)(stage + p.dev_offset * es_));
    else
      decode_into("F64", values[i], p.numel, (float*)(stage + p.dev_offset * es_));
  }
  check(gt_upload(ctx_, pbuf_.get(), stage, dev_params_ * es_));
}

}  // namespace gotensor

using gotensor::Error;

extern "C" {

GT_API char* gth_safetensors_read(const char* path, const char* name, double* out, int64_t cap, int64_t* shape,
                                  int shape_cap, int* ndim, int64_t* numel) {
  try {
    if (!path || !name) throw Error("gth_safetensors_read: null path or name");
    gotensor::StFile f;
    try {
      f = gotensor::st_decode(std::make_shared<gotensor::MappedFile>(path));
    } catch (const Error& e) {
      throw Error(std::string(path) + ": " + e.what());
    }
    auto it = f.tensors.find(name);
    if (it == f.tensors.end()) throw Error(std::string("safetensors: no tensor \"") + name + "\" in " + path);
    const auto& e = it->second;
    const int64_t n = e.shape.empty() ? 1 : e.numel;  // a scalar holds one value
    if (numel) *numel = n;
    if (ndim) *ndim = (int)e.shape.size();
    if (shape)
      for (size_t d = 0; d < e.shape.size() && (int)d < shape_cap; d++) shape[d] = e.shape[d];
    if (out) {
      if (cap < n) throw Error("gth_safetensors_read: output holds " + std::to_string(cap) + " of " +
                               std::to_string(n) + " values");
      gotensor::decode_into(e.kind, e.data, n, out);
    }
    return nullptr;
  } catch (const std::exception& ex) {
    char* m = (char*)malloc(strlen(ex.what()) + 1);
    if (m) strcpy(m, ex.what());
    return m;
  }
}

GT_API char* gth_safetensors_metadata(const char* path, const char* key, char* value, int cap, int* len) {
  try {
    if (!path || !key) throw Error("gth_safetensors_metadata: null path or key");
    gotensor::StFile f;
    try {
      f = gotensor::st_decode(std::make_shared<gotensor::MappedFile>(path));
    } catch (const Error& e) {
      throw Error(std::string(path) + ": " + e.what());
    }
    for (auto& kv : f.metadata) {
      if (kv.first != key) continue;
      if (len) *len = (int)kv.second.size();
      if (value && cap > 0) {
        const size_t n = std::min<size_t>(kv.second.size(), (size_t)cap - 1);
        memcpy(value, kv.second.data(), n);
        value[n] = 0;
      }
      return nullptr;
    }
    throw Error(std::string("safetensors: no metadata \"") + key + "\" in " + path);
  } catch (const std::exception& ex) {
    char* m = (char*)malloc(strlen(ex.what()) + 1);
    if (m) strcpy(m, ex.what());
    return m;
  }
}

}  // extern "C"
