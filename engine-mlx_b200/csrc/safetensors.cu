// safetensors.cu — the safetensors container reader (host code only) and the
// host-only C entry point emx_safetensors_index.
//
// Format and validation rules: see safetensors.cuh.  The JSON reader below
// handles exactly what a header holds (objects, arrays, strings with escapes,
// integers, and for metadata any scalar), with a nesting limit, and rejects
// anything else; it never reads past the header bytes it is given.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>

#include "ctx.cuh"
#include "emx.h"
#include "safetensors.cuh"

namespace emx {

namespace {

// ------------------------------------------------------------ JSON values
struct JVal {
  enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  int64_t i = 0;
  double d = 0.0;
  std::string s;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* key) const {
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JReader {
 public:
  JReader(const char* p, size_t n) : p_(p), e_(p + n) {}
  bool document(JVal* v) {
    if (!value(v, 0)) return false;
    ws();
    if (p_ != e_) return err("trailing bytes after the header object");
    return true;
  }
  const std::string& error() const { return err_; }

 private:
  const char* p_;
  const char* e_;
  std::string err_;
  static constexpr int kMaxDepth = 32;

  bool err(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w, size_t n) {
    if ((size_t)(e_ - p_) < n || std::memcmp(p_, w, n) != 0) return err("invalid literal");
    p_ += n;
    return true;
  }
  static void utf8(uint32_t c, std::string* o) {
    if (c < 0x80) {
      o->push_back((char)c);
    } else if (c < 0x800) {
      o->push_back((char)(0xC0 | (c >> 6)));
      o->push_back((char)(0x80 | (c & 0x3F)));
    } else if (c < 0x10000) {
      o->push_back((char)(0xE0 | (c >> 12)));
      o->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      o->push_back((char)(0x80 | (c & 0x3F)));
    } else {
      o->push_back((char)(0xF0 | (c >> 18)));
      o->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
      o->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      o->push_back((char)(0x80 | (c & 0x3F)));
    }
  }
  bool hex4(uint32_t* c) {
    if (e_ - p_ < 4) return err("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char h = *p_++;
      v <<= 4;
      if (h >= '0' && h <= '9') v |= (uint32_t)(h - '0');
      else if (h >= 'a' && h <= 'f') v |= (uint32_t)(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') v |= (uint32_t)(h - 'A' + 10);
      else return err("bad \\u escape");
    }
    *c = v;
    return true;
  }
  bool str(std::string* o) {
    if (p_ >= e_ || *p_ != '"') return err("expected a string");
    ++p_;
    while (true) {
      if (p_ >= e_) return err("unterminated string");
      const unsigned char ch = (unsigned char)*p_++;
      if (ch == '"') return true;
      if (ch < 0x20) return err("control character in a string");
      if (ch != '\\') {
        o->push_back((char)ch);
        continue;
      }
      if (p_ >= e_) return err("unterminated escape");
      const char x = *p_++;
      switch (x) {
        case '"': o->push_back('"'); break;
        case '\\': o->push_back('\\'); break;
        case '/': o->push_back('/'); break;
        case 'b': o->push_back('\b'); break;
        case 'f': o->push_back('\f'); break;
        case 'n': o->push_back('\n'); break;
        case 'r': o->push_back('\r'); break;
        case 't': o->push_back('\t'); break;
        case 'u': {
          uint32_t c;
          if (!hex4(&c)) return false;
          if (c >= 0xD800 && c < 0xDC00) {  // a surrogate pair
            uint32_t lo;
            if (e_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return err("lone surrogate");
            p_ += 2;
            if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return err("bad surrogate pair");
            c = 0x10000 + ((c - 0xD800) << 10) + (lo - 0xDC00);
          } else if (c >= 0xDC00 && c < 0xE000) {
            return err("lone surrogate");
          }
          utf8(c, o);
          break;
        }
        default: return err("bad escape");
      }
    }
  }
  bool num(JVal* v) {
    const char* s = p_;
    if (p_ < e_ && *p_ == '-') ++p_;
    if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return err("bad number");
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    bool frac = false;
    if (p_ < e_ && *p_ == '.') {
      frac = true;
      ++p_;
      if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return err("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
      frac = true;
      ++p_;
      if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return err("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    const std::string t(s, p_);
    if (!frac) {
      // integers: exact in int64 or rejected (offsets and dimensions)
      const bool neg = t[0] == '-';
      uint64_t acc = 0;
      for (size_t k = neg ? 1 : 0; k < t.size(); ++k) {
        const uint64_t dgt = (uint64_t)(t[k] - '0');
        if (acc > (UINT64_MAX - dgt) / 10) return err("integer out of range");
        acc = acc * 10 + dgt;
      }
      if (acc > (uint64_t)INT64_MAX) return err("integer out of range");
      v->kind = JVal::Int;
      v->i = neg ? -(int64_t)acc : (int64_t)acc;
      return true;
    }
    v->kind = JVal::Num;
    v->d = strtod(t.c_str(), nullptr);
    return true;
  }
  bool value(JVal* v, int depth) {
    if (depth > kMaxDepth) return err("nesting too deep");
    ws();
    if (p_ >= e_) return err("unexpected end of header");
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->kind = JVal::Obj;
      ws();
      if (p_ < e_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        std::string key;
        if (!str(&key)) return false;
        for (const auto& kv : v->obj)
          if (kv.first == key) return err("duplicate key");
        ws();
        if (p_ >= e_ || *p_ != ':') return err("expected ':'");
        ++p_;
        v->obj.emplace_back(std::move(key), JVal());
        if (!value(&v->obj.back().second, depth + 1)) return false;
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return err("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      v->kind = JVal::Arr;
      ws();
      if (p_ < e_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (true) {
        v->arr.emplace_back();
        if (!value(&v->arr.back(), depth + 1)) return false;
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return err("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->kind = JVal::Str;
      return str(&v->s);
    }
    if (c == 't') {
      v->kind = JVal::Bool;
      v->b = true;
      return lit("true", 4);
    }
    if (c == 'f') {
      v->kind = JVal::Bool;
      return lit("false", 5);
    }
    if (c == 'n') {
      v->kind = JVal::Null;
      return lit("null", 4);
    }
    return num(v);
  }
};

// The crate's upper bound on the header (MAX_HEADER_SIZE).
constexpr uint64_t kMaxHeader = 100000000ull;

}  // namespace

int st_dtype_size(const std::string& t) {
  if (t == "BOOL" || t == "U8" || t == "I8" || t == "F8_E5M2" || t == "F8_E4M3") return 1;
  if (t == "I16" || t == "U16" || t == "F16" || t == "BF16") return 2;
  if (t == "I32" || t == "U32" || t == "F32") return 4;
  if (t == "I64" || t == "U64" || t == "F64") return 8;
  return 0;
}

int st_parse_header(const char* json, size_t len, uint64_t data_bytes, uint64_t data_start,
                    std::vector<StTensor>* out, const char* what) {
  JVal root;
  JReader rd(json, len);
  if (!rd.document(&root)) return fail(EMX_ERR_INVALID, "%s: header is not valid JSON (%s)", what, rd.error().c_str());
  if (root.kind != JVal::Obj) return fail(EMX_ERR_INVALID, "%s: header is not a JSON object", what);
  out->clear();
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind != JVal::Obj) return fail(EMX_ERR_INVALID, "%s: __metadata__ is not an object", what);
      for (const auto& m : kv.second.obj)
        if (m.second.kind != JVal::Str)
          return fail(EMX_ERR_INVALID, "%s: __metadata__ value '%s' is not a string", what, m.first.c_str());
      continue;
    }
    const JVal& t = kv.second;
    const JVal* dt = t.kind == JVal::Obj ? t.get("dtype") : nullptr;
    const JVal* sh = t.kind == JVal::Obj ? t.get("shape") : nullptr;
    const JVal* of = t.kind == JVal::Obj ? t.get("data_offsets") : nullptr;
    if (!dt || !sh || !of || dt->kind != JVal::Str || sh->kind != JVal::Arr || of->kind != JVal::Arr ||
        of->arr.size() != 2 || t.obj.size() != 3)
      return fail(EMX_ERR_INVALID, "%s: tensor '%s' is not {dtype, shape, data_offsets}", what, kv.first.c_str());
    StTensor e;
    e.name = kv.first;
    e.dtype = dt->s;
    const int es = st_dtype_size(e.dtype);
    if (es == 0) return fail(EMX_ERR_INVALID, "%s: tensor '%s' has unknown dtype '%s'", what, kv.first.c_str(), e.dtype.c_str());
    uint64_t nel = 1;
    for (const auto& d : sh->arr) {
      if (d.kind != JVal::Int || d.i < 0)
        return fail(EMX_ERR_INVALID, "%s: tensor '%s' has a bad shape", what, kv.first.c_str());
      if (d.i != 0 && nel > UINT64_MAX / (uint64_t)d.i)
        return fail(EMX_ERR_INVALID, "%s: tensor '%s' shape overflows", what, kv.first.c_str());
      nel *= (uint64_t)d.i;
      e.shape.push_back(d.i);
    }
    if (nel > UINT64_MAX / (uint64_t)es) return fail(EMX_ERR_INVALID, "%s: tensor '%s' shape overflows", what, kv.first.c_str());
    const JVal& b = of->arr[0];
    const JVal& en = of->arr[1];
    if (b.kind != JVal::Int || en.kind != JVal::Int || b.i < 0 || en.i < b.i)
      return fail(EMX_ERR_INVALID, "%s: tensor '%s' has bad data_offsets", what, kv.first.c_str());
    e.bytes = (uint64_t)(en.i - b.i);
    if (e.bytes != nel * (uint64_t)es)
      return fail(EMX_ERR_INVALID, "%s: tensor '%s' holds %llu bytes, its shape and dtype need %llu", what,
                  kv.first.c_str(), (unsigned long long)e.bytes, (unsigned long long)(nel * es));
    e.offset = (uint64_t)b.i;  // relative to the data section for now
    out->push_back(std::move(e));
  }
  // the tensors must tile the data section: sorted by start, each begins where
  // the previous one ended, the last ends at the end of the file
  std::vector<const StTensor*> ord;
  for (const auto& e : *out) ord.push_back(&e);
  std::stable_sort(ord.begin(), ord.end(), [](const StTensor* a, const StTensor* b) { return a->offset < b->offset; });
  uint64_t at = 0;
  for (const StTensor* e : ord) {
    if (e->offset != at)
      return fail(EMX_ERR_INVALID, "%s: tensor '%s' starts at data byte %llu, expected %llu (gap or overlap)", what,
                  e->name.c_str(), (unsigned long long)e->offset, (unsigned long long)at);
    at = e->offset + e->bytes;
  }
  if (at != data_bytes)
    return fail(EMX_ERR_INVALID, "%s: tensors cover %llu data bytes, the file holds %llu", what,
                (unsigned long long)at, (unsigned long long)data_bytes);
  for (auto& e : *out) e.offset += data_start;
  return EMX_OK;
}

StFile::~StFile() {
  if (base) munmap(const_cast<unsigned char*>(base), size);
}

int st_open(const char* path, StFile* out) {
  out->path = path;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(EMX_ERR_INVALID, "%s: cannot open (%s)", path, strerror(errno));
  struct stat stt;
  if (fstat(fd, &stt) != 0) {
    close(fd);
    return fail(EMX_ERR_INVALID, "%s: cannot stat", path);
  }
  const size_t size = (size_t)stt.st_size;
  if (size < 8) {
    close(fd);
    return fail(EMX_ERR_INVALID, "%s: %zu bytes, shorter than the 8-byte header length", path, size);
  }
  void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return fail(EMX_ERR_INVALID, "%s: mmap failed (%s)", path, strerror(errno));
  out->base = static_cast<const unsigned char*>(p);
  out->size = size;
  uint64_t n = 0;
  for (int k = 7; k >= 0; --k) n = (n << 8) | out->base[k];  // little endian
  if (n > kMaxHeader || n > size - 8)
    return fail(EMX_ERR_INVALID, "%s: header length %llu does not fit the %zu-byte file", path,
                (unsigned long long)n, size);
  return st_parse_header(reinterpret_cast<const char*>(out->base + 8), (size_t)n, size - 8 - n, 8 + n,
                         &out->tensors, path);
}

namespace {

// A whole JSON file (at most kMaxHeader bytes) that must hold one object.
int read_json_file(const char* path, JVal* root) {
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(EMX_ERR_INVALID, "%s: cannot open (%s)", path, strerror(errno));
  std::string text;
  char buf[65536];
  while (true) {
    const ssize_t r = read(fd, buf, sizeof(buf));
    if (r < 0) {
      close(fd);
      return fail(EMX_ERR_INVALID, "%s: read failed", path);
    }
    if (r == 0) break;
    text.append(buf, (size_t)r);
    if (text.size() > kMaxHeader) {
      close(fd);
      return fail(EMX_ERR_INVALID, "%s: larger than %llu bytes", path, (unsigned long long)kMaxHeader);
    }
  }
  close(fd);
  JReader rd(text.data(), text.size());
  if (!rd.document(root) || root->kind != JVal::Obj)
    return fail(EMX_ERR_INVALID, "%s: not a JSON object (%s)", path, rd.error().c_str());
  return EMX_OK;
}

}  // namespace

int st_index_files(const char* index_path, std::vector<std::string>* files) {
  JVal root;
  const int rc = read_json_file(index_path, &root);
  if (rc) return rc;
  const JVal* wm = root.get("weight_map");
  if (!wm || wm->kind != JVal::Obj) return fail(EMX_ERR_INVALID, "%s: no weight_map object", index_path);
  files->clear();
  for (const auto& kv : wm->obj) {
    if (kv.second.kind != JVal::Str) return fail(EMX_ERR_INVALID, "%s: weight_map value is not a string", index_path);
    const std::string& fn = kv.second.s;
    if (fn.empty() || fn.find('/') != std::string::npos || fn == "." || fn == "..")
      return fail(EMX_ERR_INVALID, "%s: shard name '%s' is not a file name", index_path, fn.c_str());
    if (std::find(files->begin(), files->end(), fn) == files->end()) files->push_back(fn);
  }
  return EMX_OK;
}

namespace {

// config.json fields (Qwen3Config, crates/serve/src/config.rs:8-30, read by
// Qwen3Config::from_dir, config.rs:77-90, with its serde defaults).
struct CfgReader {
  const JVal& root;
  const char* path;
  int rc = EMX_OK;
  int need_int(const char* key) {
    const JVal* v = root.get(key);
    if (!v || v->kind != JVal::Int || v->i <= 0 || v->i > (1 << 30)) {
      if (!rc) rc = fail(EMX_ERR_INVALID, "%s: '%s' missing or not a positive integer", path, key);
      return 0;
    }
    return (int)v->i;
  }
  int opt_int(const char* key, int dflt) {
    const JVal* v = root.get(key);
    if (!v || v->kind == JVal::Null) return dflt;
    if (v->kind != JVal::Int || v->i < 0 || v->i > (1 << 30)) {
      if (!rc) rc = fail(EMX_ERR_INVALID, "%s: '%s' is not a non-negative integer", path, key);
      return dflt;
    }
    return (int)v->i;
  }
  float opt_float(const char* key, float dflt) {
    const JVal* v = root.get(key);
    if (!v || v->kind == JVal::Null) return dflt;
    if (v->kind == JVal::Int) return (float)v->i;
    if (v->kind == JVal::Num) return (float)v->d;
    if (!rc) rc = fail(EMX_ERR_INVALID, "%s: '%s' is not a number", path, key);
    return dflt;
  }
  bool opt_bool(const char* key, bool dflt) {
    const JVal* v = root.get(key);
    if (!v || v->kind == JVal::Null) return dflt;
    if (v->kind != JVal::Bool) {
      if (!rc) rc = fail(EMX_ERR_INVALID, "%s: '%s' is not a boolean", path, key);
      return dflt;
    }
    return v->b;
  }
};

// One quantization setting ({"group_size": g, "bits": b}); false when the
// entry is not such an object.
bool quant_pair(const JVal& v, int* gs, int* bits) {
  if (v.kind != JVal::Obj) return false;
  const JVal* g = v.get("group_size");
  const JVal* b = v.get("bits");
  if (!g || !b || g->kind != JVal::Int || b->kind != JVal::Int) return false;
  *gs = (int)g->i;
  *bits = (int)b->i;
  return true;
}

}  // namespace

}  // namespace emx

using namespace emx;

extern "C" int emx_qwen3_config_from_dir(const char* model_dir, int kv_cap, int max_prefill, emx_qwen3_config* out) {
  if (!model_dir || !out) return fail(EMX_ERR_INVALID, "emx_qwen3_config_from_dir: null argument");
  if (kv_cap < 1 || max_prefill < 1 || max_prefill > kv_cap)
    return fail(EMX_ERR_INVALID, "emx_qwen3_config_from_dir: kv_cap %d / max_prefill %d out of range", kv_cap,
                max_prefill);
  std::string path = model_dir;
  struct stat st;
  if (stat(path.c_str(), &st) == 0 && S_ISDIR(st.st_mode)) path += "/config.json";
  JVal root;
  int rc = read_json_file(path.c_str(), &root);
  if (rc) return rc;
  CfgReader r{root, path.c_str()};
  emx_qwen3_config c;
  std::memset(&c, 0, sizeof(c));
  c.hidden = r.need_int("hidden_size");
  c.layers = r.need_int("num_hidden_layers");
  c.inter = r.need_int("intermediate_size");
  c.n_q = r.need_int("num_attention_heads");
  c.n_kv = r.need_int("num_key_value_heads");
  c.vocab = r.need_int("vocab_size");
  if (r.rc) return r.rc;
  c.eps = r.opt_float("rms_norm_eps", 1e-6f);
  c.rope_theta = r.opt_float("rope_theta", 1000000.0f);
  c.head_dim = r.opt_int("head_dim", c.n_q ? c.hidden / c.n_q : 0);
  c.norm_groups = r.opt_int("layernorm_num_groups", 1);
  c.tied = r.opt_bool("tie_word_embeddings", true) ? 1 : 0;
  // MoE (Qwen3-MoE config keys)
  c.n_experts = r.opt_int("num_experts", 0);
  c.top_k = r.opt_int("num_experts_per_tok", 0);
  c.moe_inter = r.opt_int("moe_intermediate_size", 0);
  c.norm_topk = r.opt_bool("norm_topk_prob", false) ? 1 : 0;
  if (r.rc) return r.rc;
  if (c.n_experts > 0 && (c.top_k < 1 || c.top_k > c.n_experts || c.moe_inter < 1))
    return fail(EMX_ERR_INVALID, "%s: num_experts %d needs num_experts_per_tok in [1, %d] and moe_intermediate_size",
                path.c_str(), c.n_experts, c.n_experts);
  // quantization: the model-wide {group_size, bits}, then MLX's per-module
  // entries keyed by module name (one setting per class of projection)
  const JVal* q = root.get("quantization");
  if (!q) q = root.get("quantization_config");
  int gs = 0, bits = 0;
  if (!q || !quant_pair(*q, &gs, &bits))
    return fail(EMX_ERR_INVALID, "%s: no quantization {group_size, bits}: the engine takes affine-quantized "
                "checkpoints only", path.c_str());
  int cls_gs[6], cls_bits[6], cls_set[6] = {0, 0, 0, 0, 0, 0};  // attn, mlp, embed, lm, router, expert
  for (int k = 0; k < 6; ++k) {
    cls_gs[k] = gs;
    cls_bits[k] = bits;
  }
  for (const auto& kv : q->obj) {
    const std::string& key = kv.first;
    if (key == "group_size" || key == "bits" || key == "mode") continue;
    int cls = -1;
    if (key.find(".switch_mlp.") != std::string::npos) cls = 5;
    else if (key.size() >= 8 && key.compare(key.size() - 8, 8, "mlp.gate") == 0) cls = 4;
    else if (key.find(".self_attn.") != std::string::npos) cls = 0;
    else if (key.find(".mlp.") != std::string::npos) cls = 1;
    else if (key == "model.embed_tokens") cls = 2;
    else if (key == "lm_head") cls = 3;
    else continue;  // a module off this path
    int g2, b2;
    if (!quant_pair(kv.second, &g2, &b2))
      return fail(EMX_ERR_INVALID, "%s: module '%s' is not quantized ({group_size, bits}); the engine takes "
                  "affine-quantized projections only", path.c_str(), key.c_str());
    if (cls_set[cls] && (cls_gs[cls] != g2 || cls_bits[cls] != b2))
      return fail(EMX_ERR_INVALID, "%s: module '%s' (%d bits, group %d) differs from others of its kind (%d, %d); "
                  "the engine takes one setting per kind", path.c_str(), key.c_str(), b2, g2, cls_bits[cls],
                  cls_gs[cls]);
    cls_set[cls] = 1;
    cls_gs[cls] = g2;
    cls_bits[cls] = b2;
  }
  c.attn_bits = cls_bits[0], c.attn_group = cls_gs[0];
  c.mlp_bits = cls_bits[1], c.mlp_group = cls_gs[1];
  c.embed_bits = cls_bits[2], c.embed_group = cls_gs[2];
  c.lm_bits = cls_bits[3], c.lm_group = cls_gs[3];
  c.router_bits = cls_bits[4], c.router_group = cls_gs[4];
  c.expert_bits = cls_bits[5], c.expert_group = cls_gs[5];
  c.kv_cap = kv_cap;
  c.max_prefill = max_prefill;
  *out = c;
  return EMX_OK;
}


extern "C" int emx_safetensors_index(const char* file, emx_st_tensor* out, int cap, int* n) {
  if (!file || !n || (cap > 0 && !out)) return fail(EMX_ERR_INVALID, "emx_safetensors_index: null argument");
  StFile f;
  int rc = st_open(file, &f);
  if (rc) return rc;
  *n = (int)f.tensors.size();
  for (int k = 0; k < cap && k < *n; ++k) {
    const StTensor& t = f.tensors[(size_t)k];
    emx_st_tensor& o = out[k];
    std::memset(&o, 0, sizeof(o));
    if (t.name.size() >= sizeof(o.name) || t.shape.size() > 8)
      return fail(EMX_ERR_INVALID, "emx_safetensors_index: tensor '%s' name or rank exceeds the record", t.name.c_str());
    std::memcpy(o.name, t.name.c_str(), t.name.size());
    std::memcpy(o.dtype, t.dtype.c_str(), std::min(t.dtype.size(), sizeof(o.dtype) - 1));
    o.ndim = (int)t.shape.size();
    for (size_t d = 0; d < t.shape.size(); ++d) o.shape[d] = t.shape[d];
    o.offset = t.offset;
    o.bytes = t.bytes;
  }
  return EMX_OK;
}
