// Checkpoint intake on the host: config.json and safetensors shards of a model
// directory, the way the reference reads them (src/config.rs:142-189,
// src/weights.rs:14-489), feeding the C-ABI loaders (qasr_load_embed / qasr_load_layer).
//
// Shards are memory-mapped read-only and every tensor's byte range is checked against
// the file and against dtype x shape before anything reads it.  Float tensors narrow to
// f16 with round-to-nearest-even (bf16 -> f32 is exact, then one rounding: the values
// RawTensor::narrow_f16_into produces, src/weights.rs:55-80); I8 tensors dequantise as
// f16(f32(q) * s) with their `<name without .weight>.weight_scale` (src/weights.rs:394-417)
// or, for an INT8_F32 context, go to the device as the file's own bytes and f32 scales
// (PackedInt8, src/weights.rs:309-356).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "abi_guard.h"
#include "ctx_internal.h"
#include "f16_host.h"
#include "qasr_b200.h"
#include "qasr_b200_audio.h"

namespace {

// ------------------------------------------------------------------ JSON (RFC 8259)
// Enough of JSON for config.json, model.safetensors.index.json and safetensors headers:
// objects keep their key order, numbers keep an exact int64 when they are integers.
struct JValue {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  bool is_int = false;
  long long i = 0;
  std::string str;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;

  const JValue* get(const char* key) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(JValue* out, std::string* err) {
    ws();
    if (!value(out, 0)) {
      *err = "JSON: " + err_ + " at byte " + std::to_string(pos());
      return false;
    }
    ws();
    if (p_ != end_) {
      *err = "JSON: trailing bytes at " + std::to_string(pos());
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* start_ = p_;
  const char* end_;
  std::string err_;

  size_t pos() const { return static_cast<size_t>(p_ - start_); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool fail(const char* m) {
    err_ = m;
    return false;
  }
  bool lit(const char* s) {
    const size_t n = std::strlen(s);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, s, n) != 0) return fail("bad literal");
    p_ += n;
    return true;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) {
      o += static_cast<char>(c);
    } else if (c < 0x800) {
      o += static_cast<char>(0xC0 | (c >> 6));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      o += static_cast<char>(0xE0 | (c >> 12));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else {
      o += static_cast<char>(0xF0 | (c >> 18));
      o += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t* v) {
    if (end_ - p_ < 4) return fail("short \\u escape");
    *v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p_++;
      *v <<= 4;
      if (c >= '0' && c <= '9') *v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') *v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') *v |= static_cast<uint32_t>(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool string(std::string* o) {
    ++p_;  // opening quote
    while (true) {
      if (p_ >= end_) return fail("unterminated string");
      const char c = *p_++;
      if (c == '"') return true;
      if (static_cast<unsigned char>(c) < 0x20) return fail("control character in string");
      if (c != '\\') {
        *o += c;
        continue;
      }
      if (p_ >= end_) return fail("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': *o += '"'; break;
        case '\\': *o += '\\'; break;
        case '/': *o += '/'; break;
        case 'b': *o += '\b'; break;
        case 'f': *o += '\f'; break;
        case 'n': *o += '\n'; break;
        case 'r': *o += '\r'; break;
        case 't': *o += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(&c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate");
            p_ += 2;
            if (!hex4(&c2) || c2 < 0xDC00 || c2 >= 0xE000) return fail("bad surrogate pair");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          utf8(*o, c1);
          break;
        }
        default: return fail("bad escape");
      }
    }
  }
  bool number(JValue* v) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    bool frac = false;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                         *p_ == '-')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') frac = true;
      ++p_;
    }
    if (p_ == s || (p_ == s + 1 && *s == '-')) return fail("bad number");
    const std::string t(s, p_);
    char* endp = nullptr;
    v->kind = JValue::Num;
    v->num = std::strtod(t.c_str(), &endp);
    if (endp != t.c_str() + t.size()) return fail("bad number");
    if (!frac) {
      errno = 0;
      const long long i = std::strtoll(t.c_str(), &endp, 10);
      if (errno == 0 && endp == t.c_str() + t.size()) {
        v->is_int = true;
        v->i = i;
      }
    }
    return true;
  }
  bool value(JValue* v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    if (p_ >= end_) return fail("unexpected end");
    const char c = *p_;
    if (c == '{') {
      v->kind = JValue::Obj;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        if (p_ >= end_ || *p_ != '"') return fail("expected key");
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        ws();
        v->obj.emplace_back(std::move(key), JValue{});
        if (!value(&v->obj.back().second, depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v->kind = JValue::Arr;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        v->arr.emplace_back();
        if (!value(&v->arr.back(), depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->kind = JValue::Str;
      return string(&v->str);
    }
    if (c == 't') {
      v->kind = JValue::Bool;
      v->b = true;
      return lit("true");
    }
    if (c == 'f') {
      v->kind = JValue::Bool;
      return lit("false");
    }
    if (c == 'n') return lit("null");
    return number(v);
  }
};

bool read_file(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = !std::ferror(f);
  std::fclose(f);
  return ok;
}

bool file_exists(const std::string& path) {
  struct stat st;
  return ::stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

void set_err(char* err, int errlen, const std::string& m) {
  if (err && errlen > 0) std::snprintf(err, static_cast<size_t>(errlen), "%s", m.c_str());
}

// ------------------------------------------------------------------ tensors
struct Tensor {
  std::string dtype;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

// bytes per element of the safetensors dtypes; 0 for ones without a fixed size here
size_t dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

// remap_hf_weight_name (src/weights.rs:173-187)
std::string remap_hf(const std::string& n) {
  auto starts = [&](const char* p) { return n.compare(0, std::strlen(p), p) == 0; };
  if (starts("model.multi_modal_projector.linear_1"))
    return "thinker.audio_tower.proj1" + n.substr(std::strlen("model.multi_modal_projector.linear_1"));
  if (starts("model.multi_modal_projector.linear_2"))
    return "thinker.audio_tower.proj2" + n.substr(std::strlen("model.multi_modal_projector.linear_2"));
  if (starts("model.audio_tower.")) return "thinker.audio_tower." + n.substr(std::strlen("model.audio_tower."));
  if (starts("model.language_model.")) return "thinker.model." + n.substr(std::strlen("model.language_model."));
  return n;
}

float to_f32_elem(const Tensor& t, int64_t i) {
  const uint8_t* p = t.data;
  if (t.dtype == "F32") {
    float f;
    std::memcpy(&f, p + 4 * i, 4);
    return f;
  }
  uint16_t h;
  std::memcpy(&h, p + 2 * i, 2);
  if (t.dtype == "BF16") {
    const uint32_t x = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &x, 4);
    return f;
  }
  return qasr::f16_bits_to_f32(h);  // F16
}

}  // namespace

struct qasr_checkpoint {
  std::vector<std::pair<void*, size_t>> maps;
  std::unordered_map<std::string, Tensor> tensors;
  std::string err;

  ~qasr_checkpoint() {
    for (auto& m : maps) ::munmap(m.first, m.second);
  }
  qasr_status fail(qasr_status s, const std::string& m) {
    err = m;
    return s;
  }
  const Tensor* find(const std::string& name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
  }

  // load_shard (src/weights.rs:203-228)
  qasr_status add_shard(const std::string& path, std::unordered_map<std::string, Tensor>* out) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail(QASR_ERR_INVALID_ARG, "open " + path + ": " + std::strerror(errno));
    struct stat st;
    if (::fstat(fd, &st) != 0) {
      ::close(fd);
      return fail(QASR_ERR_INVALID_ARG, "stat " + path);
    }
    const size_t size = static_cast<size_t>(st.st_size);
    if (size < 8) {
      ::close(fd);
      return fail(QASR_ERR_INVALID_ARG, path + ": shorter than a safetensors header");
    }
    void* m = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) return fail(QASR_ERR_OOM, "mmap " + path + ": " + std::strerror(errno));
    maps.emplace_back(m, size);
    const uint8_t* base = static_cast<const uint8_t*>(m);
    uint64_t hlen = 0;
    for (int k = 0; k < 8; ++k) hlen |= static_cast<uint64_t>(base[k]) << (8 * k);  // little-endian
    if (hlen > size - 8) return fail(QASR_ERR_INVALID_ARG, path + ": header length past the end of the file");
    JValue h;
    std::string jerr;
    if (!JParser(reinterpret_cast<const char*>(base + 8), hlen).parse(&h, &jerr))
      return fail(QASR_ERR_INVALID_ARG, path + ": " + jerr);
    if (h.kind != JValue::Obj) return fail(QASR_ERR_INVALID_ARG, path + ": header is not an object");
    const uint8_t* data = base + 8 + hlen;
    const size_t dlen = size - 8 - hlen;
    for (const auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      const JValue& e = kv.second;
      const JValue* dt = e.get("dtype");
      const JValue* sh = e.get("shape");
      const JValue* off = e.get("data_offsets");
      if (!dt || dt->kind != JValue::Str || !sh || sh->kind != JValue::Arr || !off || off->kind != JValue::Arr ||
          off->arr.size() != 2 || !off->arr[0].is_int || !off->arr[1].is_int)
        return fail(QASR_ERR_INVALID_ARG, path + ": malformed entry " + kv.first);
      Tensor t;
      t.dtype = dt->str;
      for (const JValue& d : sh->arr) {
        if (!d.is_int || d.i < 0) return fail(QASR_ERR_INVALID_ARG, path + ": bad shape of " + kv.first);
        t.shape.push_back(d.i);
      }
      const long long b = off->arr[0].i, en = off->arr[1].i;
      if (b < 0 || en < b || static_cast<unsigned long long>(en) > dlen)
        return fail(QASR_ERR_INVALID_ARG, path + ": data_offsets of " + kv.first + " outside the file");
      t.data = data + b;
      t.nbytes = static_cast<size_t>(en - b);
      const size_t es = dtype_size(t.dtype);
      // element count and byte size without wrap-around: a shape whose product overflows
      // (e.g. [2^33, 2^31]) would otherwise wrap to a small count and pass the size check
      uint64_t count = 1, bytes = 0;
      for (int64_t d : t.shape)
        if (__builtin_mul_overflow(count, static_cast<uint64_t>(d), &count) || count > (1ull << 62))
          return fail(QASR_ERR_INVALID_ARG, path + ": shape of " + kv.first + " overflows");
      if (es != 0 && (__builtin_mul_overflow(count, static_cast<uint64_t>(es), &bytes) || bytes != t.nbytes))
        return fail(QASR_ERR_INVALID_ARG, path + ": " + kv.first + " holds " + std::to_string(t.nbytes) +
                                              " bytes for " + std::to_string(t.numel()) + " x " + t.dtype);
      (*out)[kv.first] = std::move(t);
    }
    return QASR_OK;
  }

  // load_tensors (src/weights.rs:150-171) + normalize_hf_weight_names (:189-201)
  qasr_status open_dir(const std::string& dir) {
    std::unordered_map<std::string, Tensor> all;
    const std::string index = dir + "/model.safetensors.index.json";
    if (file_exists(index)) {
      std::string text;
      if (!read_file(index, &text)) return fail(QASR_ERR_INVALID_ARG, "read " + index);
      JValue j;
      std::string jerr;
      if (!JParser(text.data(), text.size()).parse(&j, &jerr)) return fail(QASR_ERR_INVALID_ARG, index + ": " + jerr);
      const JValue* wm = j.get("weight_map");
      if (!wm || wm->kind != JValue::Obj) return fail(QASR_ERR_INVALID_ARG, "invalid index.json: no weight_map");
      std::vector<std::string> shards;
      for (const auto& kv : wm->obj)
        if (kv.second.kind == JValue::Str) shards.push_back(kv.second.str);
      std::sort(shards.begin(), shards.end());
      shards.erase(std::unique(shards.begin(), shards.end()), shards.end());
      for (const std::string& s : shards) {
        if (s.find('/') != std::string::npos || s == "." || s == "..")
          return fail(QASR_ERR_INVALID_ARG, "index.json names a shard outside the directory: " + s);
        const qasr_status st = add_shard(dir + "/" + s, &all);
        if (st) return st;
      }
    } else {
      const qasr_status st = add_shard(dir + "/model.safetensors", &all);
      if (st) return st;
    }
    bool hf = false;
    for (const auto& kv : all)
      if (kv.first.rfind("model.audio_tower.", 0) == 0 || kv.first.rfind("model.language_model.", 0) == 0) hf = true;
    if (!hf) {
      tensors = std::move(all);
    } else {
      for (auto& kv : all) tensors[remap_hf(kv.first)] = std::move(kv.second);
    }
    return QASR_OK;
  }

  // scale_name (src/weights.rs:418-424)
  qasr_status scale_name(const std::string& w, std::string* out) {
    const std::string suf = ".weight";
    if (w.size() < suf.size() || w.compare(w.size() - suf.size(), suf.size(), suf) != 0)
      return fail(QASR_ERR_INVALID_ARG, "int8 weight " + w + " does not end in `.weight`");
    *out = w.substr(0, w.size() - suf.size()) + ".weight_scale";
    return QASR_OK;
  }

  // get_f16 (src/weights.rs:394-417): any float dtype narrowed, I8 dequantised
  qasr_status read_f16(const std::string& name, std::vector<uint16_t>* out, std::vector<int64_t>* shape) {
    const Tensor* t = find(name);
    if (!t) return fail(QASR_ERR_INVALID_ARG, "weight not found: " + name);
    const int64_t n = t->numel();
    out->resize(static_cast<size_t>(n));
    if (shape) *shape = t->shape;
    if (t->dtype == "F16") {
      std::memcpy(out->data(), t->data, static_cast<size_t>(n) * 2);
      return QASR_OK;
    }
    if (t->dtype == "BF16" || t->dtype == "F32") {
      uint16_t* o = out->data();
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < n; ++i) o[i] = qasr::f32_to_f16_bits(to_f32_elem(*t, i));
      return QASR_OK;
    }
    if (t->dtype == "I8") {
      std::string sn;
      qasr_status st = scale_name(name, &sn);
      if (st) return st;
      const Tensor* s = find(sn);
      if (!s) return fail(QASR_ERR_INVALID_ARG, "int8 weight " + name + " needs scale tensor " + sn);
      if (t->shape.size() != 2) return fail(QASR_ERR_INVALID_ARG, "expected 2D int8 weight " + name);
      if (s->dtype != "F32" && s->dtype != "F16" && s->dtype != "BF16")
        return fail(QASR_ERR_INVALID_ARG, "scale " + sn + " has dtype " + s->dtype);
      const int64_t rows = t->shape[0], cols = t->shape[1];
      if (s->numel() != rows)
        return fail(QASR_ERR_INVALID_ARG, "scale " + sn + " is " + std::to_string(s->numel()) + " for " +
                                              std::to_string(rows) + " rows");
      const int8_t* q = reinterpret_cast<const int8_t*>(t->data);
      uint16_t* o = out->data();
#pragma omp parallel for schedule(static)
      for (int64_t r = 0; r < rows; ++r) {
        const float sc = to_f32_elem(*s, r);
        for (int64_t c = 0; c < cols; ++c)
          o[r * cols + c] = qasr::f32_to_f16_bits(static_cast<float>(q[r * cols + c]) * sc);
      }
      return QASR_OK;
    }
    return fail(QASR_ERR_INVALID_ARG, "unsupported dtype " + t->dtype + " for " + name);
  }

  // get_int8 + PackedInt8::from_raw (src/weights.rs:479-489, 328-354)
  qasr_status int8(const std::string& name, int64_t rows, int64_t cols, const Tensor** w, const Tensor** s) {
    const Tensor* t = find(name);
    if (!t) return fail(QASR_ERR_INVALID_ARG, "weight not found: " + name);
    if (t->dtype != "I8") return fail(QASR_ERR_INVALID_ARG, name + " is " + t->dtype + ", not I8");
    std::string sn;
    qasr_status st = scale_name(name, &sn);
    if (st) return st;
    const Tensor* sc = find(sn);
    if (!sc) return fail(QASR_ERR_INVALID_ARG, "int8 weight " + name + " needs scale tensor " + sn);
    if (t->shape.size() != 2 || t->shape[0] != rows || t->shape[1] != cols)
      return fail(QASR_ERR_INVALID_ARG, name + ": expected [" + std::to_string(rows) + ", " + std::to_string(cols) + "]");
    if (cols % 4 != 0)
      return fail(QASR_ERR_INVALID_ARG, name + ": int8 cols " + std::to_string(cols) + " is not a multiple of 4");
    if (sc->dtype != "F32" || sc->shape.size() != 1 || sc->shape[0] != rows)
      return fail(QASR_ERR_INVALID_ARG, "int8 scale " + sn + " must be F32 [" + std::to_string(rows) + "]");
    *w = t;
    *s = sc;
    return QASR_OK;
  }
};

extern "C" {

static qasr_status read_model_config_body(const char* model_dir, qasr_model_config* out, char* err, int errlen) {
  if (!model_dir || !out) {
    set_err(err, errlen, "null argument");
    return QASR_ERR_INVALID_ARG;
  }
  const std::string path = std::string(model_dir) + "/config.json";
  std::string text;
  if (!read_file(path, &text)) {
    set_err(err, errlen, "read " + path);
    return QASR_ERR_INVALID_ARG;
  }
  JValue j;
  std::string jerr;
  if (!JParser(text.data(), text.size()).parse(&j, &jerr)) {
    set_err(err, errlen, path + ": " + jerr);
    return QASR_ERR_INVALID_ARG;
  }
  // AsrConfig::from_json_str (src/config.rs:148-173)
  const JValue* tc = nullptr;
  if (const JValue* th = j.get("thinker_config")) tc = th->get("text_config");
  else tc = j.get("text_config");
  if (!tc || tc->kind != JValue::Obj) {
    set_err(err, errlen, path + ": missing thinker_config and text_config");
    return QASR_ERR_INVALID_ARG;
  }
  auto geti = [&](const char* k, int def, int* v) {
    const JValue* x = tc->get(k);
    if (!x || x->kind == JValue::Null) {
      *v = def;
      return true;
    }
    if (!x->is_int || x->i <= 0 || x->i > (1 << 30)) return false;
    *v = static_cast<int>(x->i);
    return true;
  };
  qasr_model_config c{};
  int v[7];
  const char* keys[7] = {"vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                         "num_attention_heads", "num_key_value_heads", "head_dim"};
  const int defs[7] = {151936, 1024, 3072, 28, 16, 8, 128};  // src/config.rs:102-108
  for (int k = 0; k < 7; ++k)
    if (!geti(keys[k], defs[k], &v[k])) {
      set_err(err, errlen, path + ": text_config." + keys[k] + " is not a positive integer");
      return QASR_ERR_INVALID_ARG;
    }
  c.text.vocab_size = v[0];
  c.text.hidden_size = v[1];
  c.text.intermediate_size = v[2];
  c.text.num_hidden_layers = v[3];
  c.text.num_attention_heads = v[4];
  c.text.num_key_value_heads = v[5];
  c.text.head_dim = v[6];
  double eps = 1e-6, theta = 1000000.0;  // src/config.rs:109-110
  if (const JValue* x = tc->get("rms_norm_eps"); x && x->kind == JValue::Num) eps = x->num;
  if (const JValue* x = tc->get("rope_theta"); x && x->kind == JValue::Num) theta = x->num;
  if (const JValue* rp = tc->get("rope_parameters"); rp && rp->kind == JValue::Obj)
    if (const JValue* x = rp->get("rope_theta"); x && x->kind == JValue::Num) theta = x->num;
  c.text.rms_norm_eps = static_cast<float>(eps);
  c.rope_theta = theta;
  // mrope_section / mrope_interleaved (src/config.rs:175-189): defaults [24, 20, 20], true
  c.mrope_section[0] = 24;
  c.mrope_section[1] = 20;
  c.mrope_section[2] = 20;
  c.n_mrope_section = 3;
  c.mrope_interleaved = 1;
  if (const JValue* rs = tc->get("rope_scaling"); rs && rs->kind == JValue::Obj) {
    if (const JValue* ms = rs->get("mrope_section"); ms && ms->kind == JValue::Arr) {
      if (ms->arr.empty() || ms->arr.size() > 4) {
        set_err(err, errlen, path + ": rope_scaling.mrope_section must have 1 to 4 entries");
        return QASR_ERR_INVALID_ARG;
      }
      c.n_mrope_section = static_cast<int32_t>(ms->arr.size());
      for (size_t k = 0; k < ms->arr.size(); ++k) {
        if (!ms->arr[k].is_int || ms->arr[k].i < 0) {
          set_err(err, errlen, path + ": rope_scaling.mrope_section holds a non-integer");
          return QASR_ERR_INVALID_ARG;
        }
        c.mrope_section[k] = static_cast<int32_t>(ms->arr[k].i);
      }
    }
    bool il = false;
    if (const JValue* x = rs->get("mrope_interleaved"); x && x->kind == JValue::Bool) il = il || x->b;
    if (const JValue* x = rs->get("interleaved"); x && x->kind == JValue::Bool) il = il || x->b;
    c.mrope_interleaved = il ? 1 : 0;
  }
  *out = c;
  return QASR_OK;
}

static qasr_status read_audio_config_body(const char* model_dir, qasr_audio_config* out, char* err, int errlen) {
  if (!model_dir || !out) {
    set_err(err, errlen, "null argument");
    return QASR_ERR_INVALID_ARG;
  }
  const std::string path = std::string(model_dir) + "/config.json";
  std::string text;
  if (!read_file(path, &text)) {
    set_err(err, errlen, "read " + path);
    return QASR_ERR_INVALID_ARG;
  }
  JValue j;
  std::string jerr;
  if (!JParser(text.data(), text.size()).parse(&j, &jerr)) {
    set_err(err, errlen, path + ": " + jerr);
    return QASR_ERR_INVALID_ARG;
  }
  // AsrConfig::from_json_str (src/config.rs:148-173): thinker_config.audio_config, or the
  // HF layout's top-level audio_config
  const JValue* ac = nullptr;
  if (const JValue* th = j.get("thinker_config")) {
    ac = th->get("audio_config");
    if (!ac || ac->kind != JValue::Obj) {
      set_err(err, errlen, path + ": thinker_config has no audio_config");
      return QASR_ERR_INVALID_ARG;
    }
  } else {
    ac = j.get("audio_config");
    if (!ac || ac->kind != JValue::Obj) {
      set_err(err, errlen, path + ": missing thinker_config and audio_config");
      return QASR_ERR_INVALID_ARG;
    }
  }
  // AudioEncoderConfig and its defaults (src/config.rs:26-64)
  const char* keys[10] = {"d_model", "encoder_layers", "encoder_attention_heads", "encoder_ffn_dim", "num_mel_bins",
                          "downsample_hidden_size", "max_source_positions", "n_window", "n_window_infer",
                          "output_dim"};
  const int defs[10] = {896, 18, 14, 3584, 128, 480, 1500, 50, 800, 1024};
  int v[10];
  for (int k = 0; k < 10; ++k) {
    const JValue* x = ac->get(keys[k]);
    if (!x || x->kind == JValue::Null) {
      v[k] = defs[k];
    } else if (!x->is_int || x->i <= 0 || x->i > (1 << 30)) {
      set_err(err, errlen, path + ": audio_config." + keys[k] + " is not a positive integer");
      return QASR_ERR_INVALID_ARG;
    } else {
      v[k] = static_cast<int>(x->i);
    }
  }
  qasr_audio_config c{};
  c.d_model = v[0];
  c.encoder_layers = v[1];
  c.encoder_attention_heads = v[2];
  c.encoder_ffn_dim = v[3];
  c.num_mel_bins = v[4];
  c.downsample_hidden_size = v[5];
  c.max_source_positions = v[6];
  c.n_window = v[7];
  c.n_window_infer = v[8];
  c.output_dim = v[9];
  *out = c;
  return QASR_OK;
}

static qasr_status checkpoint_open_body(const char* model_dir, qasr_checkpoint** out, char* err, int errlen) {
  if (!model_dir || !out) {
    set_err(err, errlen, "null argument");
    return QASR_ERR_INVALID_ARG;
  }
  *out = nullptr;
  std::unique_ptr<qasr_checkpoint> ck(new (std::nothrow) qasr_checkpoint());  // freed on every early exit
  if (!ck) {
    set_err(err, errlen, "out of host memory");
    return QASR_ERR_OOM;
  }
  const qasr_status s = ck->open_dir(model_dir);
  if (s) {
    set_err(err, errlen, ck->err);
    return s;
  }
  *out = ck.release();
  return QASR_OK;
}

void qasr_checkpoint_close(qasr_checkpoint* ck) { delete ck; }

const char* qasr_checkpoint_last_error(const qasr_checkpoint* ck) { return ck ? ck->err.c_str() : "null checkpoint"; }

int64_t qasr_checkpoint_tensor_count(const qasr_checkpoint* ck) {
  return ck ? static_cast<int64_t>(ck->tensors.size()) : 0;
}

qasr_status qasr_checkpoint_tensor_info(qasr_checkpoint* ck, const char* name, char* dtype, int dtype_cap,
                                        int64_t* shape, int cap, int* ndim) {
  if (!ck || !name) return QASR_ERR_INVALID_ARG;
  const Tensor* t = ck->find(name);
  if (!t) return ck->fail(QASR_ERR_INVALID_ARG, std::string("weight not found: ") + name);
  if (dtype && dtype_cap > 0) std::snprintf(dtype, static_cast<size_t>(dtype_cap), "%s", t->dtype.c_str());
  if (ndim) *ndim = static_cast<int>(t->shape.size());
  for (int k = 0; shape && k < cap && k < static_cast<int>(t->shape.size()); ++k) shape[k] = t->shape[k];
  return QASR_OK;
}

qasr_status qasr_checkpoint_weight_format(qasr_checkpoint* ck, const char* prefix, int* weight_format) {
  if (!ck || !weight_format) return QASR_ERR_INVALID_ARG;
  const std::string name = std::string(prefix ? prefix : "thinker.model") + ".layers.0.self_attn.q_proj.weight";
  const Tensor* t = ck->find(name);
  if (!t) return ck->fail(QASR_ERR_INVALID_ARG, "weight not found: " + name);
  *weight_format = t->dtype == "I8" ? QASR_WEIGHTS_INT8_F32 : QASR_WEIGHTS_F16;
  return QASR_OK;
}

static qasr_status checkpoint_read_f16_body(qasr_checkpoint* ck, const char* name, uint16_t* out, int64_t count) {
  if (!ck || !name || !out) return QASR_ERR_INVALID_ARG;
  const Tensor* t = ck->find(name);
  if (!t) return ck->fail(QASR_ERR_INVALID_ARG, std::string("weight not found: ") + name);
  if (t->numel() != count)
    return ck->fail(QASR_ERR_INVALID_ARG, std::string(name) + " has " + std::to_string(t->numel()) +
                                              " elements, not " + std::to_string(count));
  std::vector<uint16_t> v;
  const qasr_status s = ck->read_f16(name, &v, nullptr);
  if (s) return s;
  std::memcpy(out, v.data(), v.size() * 2);
  return QASR_OK;
}

qasr_status qasr_checkpoint_read_f32(qasr_checkpoint* ck, const char* name, float* out, int64_t count) {
  if (!ck || !name || !out) return QASR_ERR_INVALID_ARG;
  const Tensor* t = ck->find(name);
  if (!t) return ck->fail(QASR_ERR_INVALID_ARG, std::string("weight not found: ") + name);
  if (t->numel() != count)
    return ck->fail(QASR_ERR_INVALID_ARG, std::string(name) + " has " + std::to_string(t->numel()) +
                                              " elements, not " + std::to_string(count));
  if (t->dtype != "F16" && t->dtype != "BF16" && t->dtype != "F32")
    return ck->fail(QASR_ERR_INVALID_ARG, std::string(name) + ": f32 read of dtype " + t->dtype);
  for (int64_t i = 0; i < count; ++i) out[i] = to_f32_elem(*t, i);
  return QASR_OK;
}

qasr_status qasr_checkpoint_rows_f16(qasr_checkpoint* ck, const char* name, const int32_t* rows, int n,
                                     uint16_t* out, int64_t count) {
  if (!ck || !name || !rows || !out || n < 0) return QASR_ERR_INVALID_ARG;
  const Tensor* t = ck->find(name);
  if (!t) return ck->fail(QASR_ERR_INVALID_ARG, std::string("weight not found: ") + name);
  if (t->shape.size() != 2) return ck->fail(QASR_ERR_INVALID_ARG, std::string(name) + " is not 2-D");
  const int64_t R = t->shape[0], C = t->shape[1];
  if (count != static_cast<int64_t>(n) * C)
    return ck->fail(QASR_ERR_INVALID_ARG, "out holds " + std::to_string(count) + " values, rows need " +
                                              std::to_string(static_cast<int64_t>(n) * C));
  if (t->dtype != "F16" && t->dtype != "BF16" && t->dtype != "F32")
    return ck->fail(QASR_ERR_INVALID_ARG, std::string(name) + ": row lookup of dtype " + t->dtype);
  for (int i = 0; i < n; ++i) {
    if (rows[i] < 0 || rows[i] >= R)
      return ck->fail(QASR_ERR_INVALID_ARG, "row " + std::to_string(rows[i]) + " of " + name + " is out of range");
    uint16_t* o = out + static_cast<int64_t>(i) * C;
    if (t->dtype == "F16") {
      std::memcpy(o, t->data + static_cast<size_t>(rows[i]) * C * 2, static_cast<size_t>(C) * 2);
    } else {
      for (int64_t c = 0; c < C; ++c) o[c] = qasr::f32_to_f16_bits(to_f32_elem(*t, static_cast<int64_t>(rows[i]) * C + c));
    }
  }
  return QASR_OK;
}

static qasr_status load_checkpoint_body(qasr_ctx* ctx, qasr_checkpoint* ck, const char* prefix_c) {
  if (!ctx || !ck) return QASR_ERR_INVALID_ARG;
  qasr_text_config cfg{};
  int fmt = 0;
  if (!qasr::ctx_shape(ctx, &cfg, &fmt)) return QASR_ERR_INVALID_ARG;
  const std::string prefix = prefix_c ? prefix_c : "thinker.model";
  auto bad = [&](qasr_status s, const std::string& m) { return qasr::ctx_fail(ctx, s, "checkpoint: " + m); };
  auto shape_is = [](const std::vector<int64_t>& sh, int64_t a, int64_t b) {
    return b < 0 ? (sh.size() == 1 && sh[0] == a) : (sh.size() == 2 && sh[0] == a && sh[1] == b);
  };
  const int hs = cfg.hidden_size, I = cfg.intermediate_size, hd = cfg.head_dim;
  const int qd = cfg.num_attention_heads * hd, kvd = cfg.num_key_value_heads * hd;

  // embed + final norm (src/decoder.rs:1253-1262; CpuTextDecoder::load src/cpu_decoder.rs:186-199)
  std::vector<uint16_t> embed, norm;
  std::vector<int64_t> sh;
  qasr_status s = ck->read_f16(prefix + ".embed_tokens.weight", &embed, &sh);
  if (s) return bad(s, ck->err);
  if (!shape_is(sh, cfg.vocab_size, hs))
    return bad(QASR_ERR_INVALID_ARG, "embed_tokens is not [" + std::to_string(cfg.vocab_size) + ", " +
                                         std::to_string(hs) + "]");
  if ((s = ck->read_f16(prefix + ".norm.weight", &norm, &sh))) return bad(s, ck->err);
  if (!shape_is(sh, hs, -1)) return bad(QASR_ERR_INVALID_ARG, "norm.weight is not [" + std::to_string(hs) + "]");
  if ((s = qasr_load_embed(ctx, embed.data(), norm.data()))) return s;
  embed.clear();
  embed.shrink_to_fit();

  static const char* lin_names[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                     "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
  const int64_t lin_shape[7][2] = {{qd, hs}, {kvd, hs}, {kvd, hs}, {hs, qd}, {I, hs}, {I, hs}, {hs, I}};
  for (int l = 0; l < cfg.num_hidden_layers; ++l) {
    const std::string lp = prefix + ".layers." + std::to_string(l) + ".";
    // norms (Layer::load src/cpu_decoder.rs:119-131: through f16, like every vector)
    std::vector<uint16_t> nv[4];
    const char* norm_names[4] = {"input_layernorm.weight", "post_attention_layernorm.weight",
                                 "self_attn.q_norm.weight", "self_attn.k_norm.weight"};
    const int norm_len[4] = {hs, hs, hd, hd};
    for (int k = 0; k < 4; ++k) {
      if ((s = ck->read_f16(lp + norm_names[k], &nv[k], &sh))) return bad(s, ck->err);
      if (!shape_is(sh, norm_len[k], -1))
        return bad(QASR_ERR_INVALID_ARG, lp + norm_names[k] + " is not [" + std::to_string(norm_len[k]) + "]");
    }
    qasr_layer_weights w{};
    std::vector<uint16_t> f16w[7];
    std::vector<uint16_t> s16[7];
    const void** lin_ptr[7] = {&w.q_proj, &w.k_proj, &w.v_proj, &w.o_proj, &w.gate_proj, &w.up_proj, &w.down_proj};
    const void** sc_ptr[7] = {&w.q_scale, &w.k_scale, &w.v_scale, &w.o_scale, &w.gate_scale, &w.up_scale, &w.down_scale};
    for (int k = 0; k < 7; ++k) {
      const std::string name = lp + lin_names[k] + ".weight";
      const int64_t rows = lin_shape[k][0], cols = lin_shape[k][1];
      if (fmt == QASR_WEIGHTS_F16) {  // get_matrix: narrowed, or I8 dequantised
        if ((s = ck->read_f16(name, &f16w[k], &sh))) return bad(s, ck->err);
        if (!shape_is(sh, rows, cols))
          return bad(QASR_ERR_INVALID_ARG, name + " is not [" + std::to_string(rows) + ", " + std::to_string(cols) + "]");
        *lin_ptr[k] = f16w[k].data();
      } else {  // get_int8: the file's bytes and scales
        const Tensor *tw = nullptr, *ts = nullptr;
        if ((s = ck->int8(name, rows, cols, &tw, &ts))) {
          const Tensor* t = ck->find(name);
          if (t && t->dtype != "I8")
            return bad(s, name + " is " + t->dtype + ": create the context with QASR_WEIGHTS_F16 for a float checkpoint");
          return bad(s, ck->err);
        }
        *lin_ptr[k] = tw->data;
        if (fmt == QASR_WEIGHTS_INT8_F32) {
          *sc_ptr[k] = ts->data;
        } else {  // f16 scales: only when every scale is an f16 value (no rounding)
          s16[k].resize(static_cast<size_t>(rows));
          for (int64_t r = 0; r < rows; ++r) {
            const float f = to_f32_elem(*ts, r);
            const uint16_t h = qasr::f32_to_f16_bits(f);
            if (qasr::f16_bits_to_f32(h) != f)
              return bad(QASR_ERR_INVALID_ARG, name + " has f32 scales that are not f16 values: use QASR_WEIGHTS_INT8_F32");
            s16[k][static_cast<size_t>(r)] = h;
          }
          *sc_ptr[k] = s16[k].data();
        }
      }
    }
    w.input_layernorm = nv[0].data();
    w.post_attention_layernorm = nv[1].data();
    w.q_norm = nv[2].data();
    w.k_norm = nv[3].data();
    if ((s = qasr_load_layer(ctx, l, &w))) return s;
  }
  return QASR_OK;
}

// The entry points above whose host buffers follow a file's contents, behind the guard
// that keeps C++ exceptions (a failed host allocation, most of all) inside the library.
qasr_status qasr_read_model_config(const char* model_dir, qasr_model_config* out, char* err, int errlen) {
  return qasr::guard([&] { return read_model_config_body(model_dir, out, err, errlen); },
                     [&](qasr_status s, const std::string& m) { set_err(err, errlen, m); return s; });
}

qasr_status qasr_read_audio_config(const char* model_dir, qasr_audio_config* out, char* err, int errlen) {
  return qasr::guard([&] { return read_audio_config_body(model_dir, out, err, errlen); },
                     [&](qasr_status s, const std::string& m) { set_err(err, errlen, m); return s; });
}

qasr_status qasr_checkpoint_open(const char* model_dir, qasr_checkpoint** out, char* err, int errlen) {
  return qasr::guard([&] { return checkpoint_open_body(model_dir, out, err, errlen); },
                     [&](qasr_status s, const std::string& m) { set_err(err, errlen, m); return s; });
}

qasr_status qasr_checkpoint_read_f16(qasr_checkpoint* ck, const char* name, uint16_t* out, int64_t count) {
  return qasr::guard([&] { return checkpoint_read_f16_body(ck, name, out, count); },
                     [&](qasr_status s, const std::string& m) { return ck ? ck->fail(s, m) : s; });
}

qasr_status qasr_load_checkpoint(qasr_ctx* ctx, qasr_checkpoint* ck, const char* prefix_c) {
  return qasr::guard([&] { return load_checkpoint_body(ctx, ck, prefix_c); },
                     [&](qasr_status s, const std::string& m) { return qasr::ctx_fail(ctx, s, "checkpoint: " + m); });
}

}  // extern "C"
