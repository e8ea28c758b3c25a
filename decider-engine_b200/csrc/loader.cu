// Checkpoint loading in the library: the reference's directory layout
// (src/lib.rs:287-367) read on the host and streamed into an Engine.
//   strands_decider_config.json (or hobson_config.json)  read_config, src/lib.rs:188-222
//   base/config.json (text_config)                        Config::validate, src/qwen.rs:133-188
//   lora/adapter_config.json                              src/lib.rs:300-358
//   base/model.safetensors, lora/adapter_model.safetensors, head.safetensors
//                                                         read_tensors, src/weights.rs:298-365
// Host code only (no kernels).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <memory>
#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

#include "engine.h"

namespace dg {

namespace json {

// A small JSON reader: enough for the checkpoint's config files and the
// safetensors headers.
struct Value {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;
  const Value* get(const std::string& k) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  bool truthy() const {
    switch (kind) {
      case Null: return false;
      case Bool: return b;
      case Num: return num != 0.0;
      case Str: return !str.empty();
      case Arr: return !arr.empty();
      case Obj: return !obj.empty();
    }
    return false;
  }
};

class Parser {
 public:
  Parser(const char* p, size_t n, const std::string& what) : p_(p), end_(p + n), what_(what) {}
  Value parse() {
    Value v = value(0);
    ws();
    if (p_ != end_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  const char* end_;
  std::string what_;
  [[noreturn]] void fail(const std::string& m) { throw std::runtime_error("invalid JSON in " + what_ + ": " + m); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = std::strlen(s);
    if (size_t(end_ - p_) >= n && std::memcmp(p_, s, n) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }
  static void utf8(std::string& o, unsigned cp) {
    if (cp < 0x80) {
      o += char(cp);
    } else if (cp < 0x800) {
      o += char(0xC0 | (cp >> 6));
      o += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += char(0xE0 | (cp >> 12));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    } else {
      o += char(0xF0 | (cp >> 18));
      o += char(0x80 | ((cp >> 12) & 0x3F));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    }
  }
  unsigned hex4() {
    if (end_ - p_ < 4) fail("short \\u escape");
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= unsigned(c - '0');
      else if (c >= 'a' && c <= 'f') v |= unsigned(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= unsigned(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    if (p_ >= end_ || *p_ != '"') fail("expected a string");
    ++p_;
    std::string o;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      const char c = *p_++;
      if (c == '"') break;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p_ >= end_) fail("unterminated escape");
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
          unsigned cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && lit("\\u")) {
            const unsigned lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(o, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return o;
  }
  Value value(int depth) {
    if (depth > 64) fail("nesting too deep");
    ws();
    if (p_ >= end_) fail("unexpected end");
    Value v;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.kind = Value::Obj;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return v;
      }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (p_ >= end_ || *p_ != ':') fail("expected ':'");
        ++p_;
        v.obj.emplace_back(std::move(k), value(depth + 1));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      v.kind = Value::Arr;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return v;
      }
      while (true) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Value::Str;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Value::Bool;
      return v;
    }
    if (lit("null")) return v;
    // number
    const char* s = p_;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' ||
                         *p_ == '+'))
      ++p_;
    if (p_ == s) fail("unexpected character");
    v.kind = Value::Num;
    v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
    return v;
  }
};

}  // namespace json

namespace {

std::string read_text(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot read " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

json::Value read_json(const std::string& path) {
  const std::string t = read_text(path);
  return json::Parser(t.data(), t.size(), path).parse();
}

bool exists(const std::string& path) {
  struct stat st;
  return ::stat(path.c_str(), &st) == 0;
}

const json::Value& need(const json::Value& o, const char* k, const std::string& what) {
  const json::Value* v = o.get(k);
  if (!v) throw std::runtime_error(what + ": missing \"" + k + "\"");
  return *v;
}
double num(const json::Value& o, const char* k, const std::string& what) {
  const json::Value& v = need(o, k, what);
  if (v.kind != json::Value::Num) throw std::runtime_error(what + ": \"" + k + "\" must be a number");
  return v.num;
}
int integer(const json::Value& o, const char* k, const std::string& what) {
  const double d = num(o, k, what);
  if (d != std::floor(d) || std::fabs(d) > 2147483647.0) throw std::runtime_error(what + ": \"" + k + "\" must be an integer");
  return int(d);
}
std::string str(const json::Value& o, const char* k) {
  const json::Value* v = o.get(k);
  return v && v->kind == json::Value::Str ? v->str : std::string();
}
bool flag(const json::Value& o, const char* k) {
  const json::Value* v = o.get(k);
  return v && v->truthy();
}

// Memory-mapped safetensors file: header bound and length checks as
// read_tensors (src/weights.rs:305-318).
struct Safetensors {
  struct Entry {
    std::string name;
    int dtype;  // 0 F32, 1 BF16, 2 F16
    std::vector<int64_t> shape;
    const void* data;
  };
  std::vector<Entry> entries;
  void* map = nullptr;
  size_t size = 0;
  explicit Safetensors(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot read " + path);
    struct stat st;
    if (::fstat(fd, &st) != 0) {
      ::close(fd);
      throw std::runtime_error("cannot stat " + path);
    }
    size = size_t(st.st_size);
    if (size < 8) {
      ::close(fd);
      throw std::runtime_error(path + ": invalid or oversized safetensors header");
    }
    map = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map == MAP_FAILED) {
      map = nullptr;
      throw std::runtime_error("cannot map " + path);
    }
    const auto* bytes = static_cast<const unsigned char*>(map);
    uint64_t n = 0;
    for (int i = 0; i < 8; ++i) n |= uint64_t(bytes[i]) << (8 * i);
    if (n > 16u * 1024 * 1024 || n + 8 > size) throw std::runtime_error(path + ": invalid or oversized safetensors header");
    const json::Value h = json::Parser(reinterpret_cast<const char*>(bytes) + 8, size_t(n), path).parse();
    if (h.kind != json::Value::Obj) throw std::runtime_error(path + ": safetensors header is not an object");
    const size_t base = size_t(8 + n);
    size_t data_len = 0;
    for (const auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      const json::Value& info = kv.second;
      const std::string dt = str(info, "dtype");
      int code;
      if (dt == "F32") code = 0;
      else if (dt == "BF16") code = 1;
      else if (dt == "F16") code = 2;
      else throw std::runtime_error(kv.first + ": unsupported weight dtype " + dt);
      const json::Value& shp = need(info, "shape", kv.first);
      const json::Value& off = need(info, "data_offsets", kv.first);
      if (shp.kind != json::Value::Arr || off.kind != json::Value::Arr || off.arr.size() != 2)
        throw std::runtime_error(kv.first + ": malformed safetensors entry");
      Entry e;
      e.name = kv.first;
      e.dtype = code;
      size_t count = 1;
      for (const auto& d : shp.arr) {
        if (d.kind != json::Value::Num || d.num < 0) throw std::runtime_error(kv.first + ": bad shape");
        e.shape.push_back(int64_t(d.num));
        count *= size_t(d.num);
      }
      const size_t lo = size_t(off.arr[0].num), hi = size_t(off.arr[1].num);
      const size_t esz = code == 0 ? 4 : 2;
      if (hi < lo || hi - lo != count * esz || base + hi > size)
        throw std::runtime_error(kv.first + ": tensor bytes do not match its shape");
      data_len = std::max(data_len, hi);
      e.data = bytes + base + lo;
      entries.push_back(std::move(e));
    }
    if (base + data_len != size) throw std::runtime_error(path + ": safetensors file length does not match metadata");
  }
  ~Safetensors() {
    if (map) ::munmap(map, size);
  }
  Safetensors(const Safetensors&) = delete;
  Safetensors& operator=(const Safetensors&) = delete;
};

// ---- allocation budgets at the checkpoint boundary (src/loading.rs:27-80).
// Checked size arithmetic: an overflow is an error, never a wrapped size.
size_t checked_product(const std::string& name, std::initializer_list<size_t> dims) {
  size_t n = 1;
  for (size_t d : dims)
    if (__builtin_mul_overflow(n, d, &n)) throw std::runtime_error(name + ": dimension product overflow");
  return n;
}
size_t checked_sum(const std::string& name, std::initializer_list<size_t> values) {
  size_t n = 0;
  for (size_t v : values)
    if (__builtin_add_overflow(n, v, &n)) throw std::runtime_error(name + ": dimension sum overflow");
  return n;
}
void within(const std::string& name, size_t bytes, uint64_t limit) {
  if (bytes > limit || bytes > size_t(INT64_MAX))
    throw std::runtime_error(name + ": allocation of " + std::to_string(bytes) + " bytes exceeds budget " +
                             std::to_string(limit));
}

// WeightBudget (src/loading.rs:52-80): every tensor is charged as FP32 plus
// its possible group-64 scales, against the per-tensor budget and, with the
// tensor counted twice (the original plus its conversion scratch), against
// the aggregate budget shared by every file of the checkpoint.
struct WeightBudget {
  LoadLimits limits;
  size_t used = 0;
  explicit WeightBudget(const LoadLimits& l) : limits(l) {}
  void charge(const std::string& name, const std::vector<size_t>& shape) {
    size_t elements = 1;
    for (size_t d : shape)
      if (__builtin_mul_overflow(elements, d, &elements)) throw std::runtime_error(name + ": dimension product overflow");
    size_t bytes = checked_product(name, {elements, 4});
    if (shape.size() == 2)
      bytes = checked_sum(name, {bytes, checked_product(name, {shape[0], (shape[1] + 63) / 64, 4})});
    within(name, bytes, limits.max_tensor_bytes);
    used = checked_sum("checkpoint weights", {used, bytes});
    within("checkpoint weights and conversion scratch", checked_sum(name, {used, bytes}), limits.max_weight_bytes);
  }
};

}  // namespace

// Config::validate_layout (src/qwen.rs:37-135): the architecture's weights
// (FP32 estimates, LoRA included) charged against a fresh budget and the
// forward workspace bound, all before any payload is read or any device
// memory is taken.
void validate_layout(const Config& c, int tokens, int rank, int pointer, const LoadLimits& limits) {
  const size_t h = size_t(c.hidden);
  const size_t qw = checked_product("query width", {size_t(c.heads), size_t(c.head_dim)});
  const size_t kw = checked_product("key/value width", {size_t(c.kv_heads), size_t(c.head_dim)});
  const size_t kd = checked_product("delta key width", {size_t(c.key_heads), size_t(c.dk)});
  const size_t vd = checked_product("delta value width", {size_t(c.value_heads), size_t(c.dv)});
  const size_t qkv = checked_sum("delta QKV width", {checked_product("delta keys", {2, kd}), vd});
  const size_t recurrent =
      checked_product("recurrent state", {size_t(c.value_heads), size_t(c.dk), size_t(c.dv)});
  WeightBudget w(limits);
  w.charge("embedding", {size_t(c.vocab), h});
  w.charge("final norm", {h});
  w.charge("pointer head", {2, size_t(pointer), h});
  w.charge("pointer norms/biases", {2, checked_sum("pointer norms", {h, size_t(pointer)})});
  size_t max_width = std::max({h, size_t(c.intermediate), size_t(rank), size_t(pointer)});
  for (int kind : c.layer_types) {
    std::vector<std::pair<size_t, size_t>> projections = {
        {h, size_t(c.intermediate)}, {h, size_t(c.intermediate)}, {size_t(c.intermediate), h}};
    w.charge("layer norms", {2, h});
    if (kind == 1) {
      projections.push_back({h, checked_product("gated query width", {2, qw})});
      projections.push_back({h, kw});
      projections.push_back({h, kw});
      projections.push_back({qw, h});
      w.charge("attention norms", {2, size_t(c.head_dim)});
    } else {
      projections.push_back({h, qkv});
      projections.push_back({h, vd});
      projections.push_back({h, size_t(c.value_heads)});
      projections.push_back({h, size_t(c.value_heads)});
      projections.push_back({vd, h});
      w.charge("convolution", {qkv, size_t(c.conv_kernel)});
      w.charge("delta constants",
               {checked_sum("delta constants",
                            {checked_product("delta heads", {2, size_t(c.value_heads)}), size_t(c.dv)})});
    }
    for (const auto& io : projections) {
      w.charge("projection", {io.second, io.first});
      w.charge("LoRA A", {size_t(rank), io.first});
      w.charge("LoRA B", {io.second, size_t(rank)});
      max_width = std::max({max_width, io.first, io.second});
    }
  }
  const size_t activations = checked_product("activation workspace", {size_t(tokens), max_width, 16});
  const size_t angles = checked_product("rotary workspace", {size_t(tokens), size_t(c.rotary_dim()), 2});
  const size_t elements = checked_sum("forward workspace", {activations, angles, recurrent});
  within("forward workspace", checked_product("forward workspace", {elements, 4}), limits.max_workspace_bytes);
}

// read_config (src/lib.rs:188-222), Config::validate's config checks
// (src/qwen.rs:133-188) and the adapter checks (src/lib.rs:300-358).
void read_checkpoint_config(const std::string& dir, Config& c, int& pointer_dim, int* max_length_out) {
  std::string dpath = dir + "/strands_decider_config.json";
  if (!exists(dpath)) dpath = dir + "/hobson_config.json";
  const json::Value d = read_json(dpath);
  const json::Value* fb = d.get("force_bos");
  if (str(d, "base_model") != "Qwen/Qwen3.5-2B-Base" || str(d, "head_type") != "pointer" || !flag(d, "use_lora") ||
      (fb && fb->truthy()))
    throw std::runtime_error(
        "native engine requires Qwen3.5-2B-Base, pointer head, LoRA, and default BOS behavior");
  const int max_length = integer(d, "max_length", dpath);
  if (max_length_out) *max_length_out = max_length;
  pointer_dim = integer(d, "pointer_dim", dpath);
  const double temp = d.get("temperature") ? num(d, "temperature", dpath) : 0.0;
  const double smooth = d.get("ordinal_smoothing") ? num(d, "ordinal_smoothing", dpath) : 0.0;
  bool kinds_ok = true;
  if (const json::Value* tk = d.get("temperature_by_kind"))
    for (const auto& kv : tk->obj) kinds_ok = kinds_ok && kv.second.kind == json::Value::Num && std::isfinite(kv.second.num) && kv.second.num > 0;
  if (!(max_length > 0 && max_length <= 4096) || !(pointer_dim > 0 && pointer_dim <= 4096) || !std::isfinite(temp) ||
      temp <= 0 || !kinds_ok || !std::isfinite(smooth) || smooth < 0.0 || smooth > 1.0)
    throw std::runtime_error("invalid decision window, pointer dimension, or calibration");

  const std::string bpath = dir + "/base/config.json";
  const json::Value b = read_json(bpath);
  if (str(b, "model_type") != "qwen3_5") throw std::runtime_error("base model must be qwen3_5");
  const json::Value& t = need(b, "text_config", bpath);
  const json::Value& rp = need(t, "rope_parameters", bpath);
  c.hidden = integer(t, "hidden_size", bpath);
  c.intermediate = integer(t, "intermediate_size", bpath);
  c.layers = integer(t, "num_hidden_layers", bpath);
  c.vocab = integer(t, "vocab_size", bpath);
  c.heads = integer(t, "num_attention_heads", bpath);
  c.kv_heads = integer(t, "num_key_value_heads", bpath);
  c.head_dim = integer(t, "head_dim", bpath);
  c.conv_kernel = integer(t, "linear_conv_kernel_dim", bpath);
  c.dk = integer(t, "linear_key_head_dim", bpath);
  c.dv = integer(t, "linear_value_head_dim", bpath);
  c.key_heads = integer(t, "linear_num_key_heads", bpath);
  c.value_heads = integer(t, "linear_num_value_heads", bpath);
  c.eps = float(num(t, "rms_norm_eps", bpath));
  c.rope_theta = float(num(rp, "rope_theta", bpath));
  c.partial_rotary = float(num(rp, "partial_rotary_factor", bpath));
  const int rot = int(float(c.head_dim) * c.partial_rotary);
  if (flag(t, "attention_bias") || !flag(t, "attn_output_gate") || str(t, "hidden_act") != "silu" ||
      str(rp, "rope_type") != "default" || rot == 0 || rot > c.head_dim || rot % 2)
    throw std::runtime_error("unsupported Qwen normalization, activation, attention, or RoPE config");
  const json::Value& lt = need(t, "layer_types", bpath);
  c.layer_types.clear();
  for (const auto& v : lt.arr) {
    if (v.kind != json::Value::Str || (v.str != "full_attention" && v.str != "linear_attention"))
      throw std::runtime_error("unsupported layer type");
    c.layer_types.push_back(v.str == "full_attention" ? 1 : 0);
  }

  const std::string apath = dir + "/lora/adapter_config.json";
  const json::Value a = read_json(apath);
  const json::Value* r = a.get("r");
  if (!r || r->kind != json::Value::Num || r->num != std::floor(r->num) || r->num <= 0 || r->num > 4096)
    throw std::runtime_error("invalid LoRA rank");
  const json::Value* alpha = a.get("lora_alpha");
  if (!alpha || alpha->kind != json::Value::Num || !std::isfinite(alpha->num) || alpha->num <= 0)
    throw std::runtime_error("invalid LoRA alpha");
  if (str(a, "peft_type") != "LORA" || str(a, "bias") != "none" || flag(a, "use_dora") || flag(a, "use_rslora") ||
      flag(a, "fan_in_fan_out") || flag(a, "rank_pattern") || flag(a, "alpha_pattern") || flag(a, "modules_to_save"))
    throw std::runtime_error("unsupported LoRA adapter configuration");
  c.rank = int(r->num);
  c.lora_scale = float(alpha->num) / float(c.rank);
  c.pointer_dim = pointer_dim;
}

// The base checkpoint's files: model.safetensors, or the distinct files of
// model.safetensors.index.json's weight_map in name order (Weights::base,
// src/weights.rs:218-259).
static std::vector<std::string> base_files(const std::string& dir) {
  const std::string single = dir + "/base/model.safetensors";
  if (exists(single)) return {single};
  const std::string ipath = dir + "/base/model.safetensors.index.json";
  const json::Value idx = read_json(ipath);
  const json::Value* map = idx.get("weight_map");
  if (!map || map->kind != json::Value::Obj) throw std::runtime_error("missing weight_map in base index");
  std::vector<std::string> files;
  for (const auto& kv : map->obj) {
    if (kv.second.kind != json::Value::Str || kv.second.str.empty() || kv.second.str.find('/') != std::string::npos ||
        kv.second.str.find("..") != std::string::npos)
      throw std::runtime_error("invalid base shard name");
    files.push_back(dir + "/base/" + kv.second.str);
  }
  std::sort(files.begin(), files.end());
  files.erase(std::unique(files.begin(), files.end()), files.end());
  return files;
}

// Model::load + Head::load (src/lib.rs:287-367): the base tensors without
// their "model.language_model." prefix, the adapter tensors as stored, the
// head tensors prefixed "head.". Every file's selected tensors are charged
// to one WeightBudget from their header shapes before any payload of that
// file is read (read_tensors, src/weights.rs:316-325), in the reference's
// order: adapter, head, base.
// The checkpoint files' budget check alone (no engine, no payload read): run
// before the engine takes device memory, so an over-budget checkpoint is
// refused without any allocation.
void ensure_checkpoint_budget(const std::string& dir, const LoadLimits& limits) {
  const std::string prefix = "model.language_model.";
  WeightBudget budget(limits);
  auto charge_all = [&](const Safetensors& f, const std::string* pfx) {
    for (const auto& t : f.entries) {
      if (pfx && t.name.compare(0, pfx->size(), *pfx) != 0) continue;
      budget.charge(t.name, std::vector<size_t>(t.shape.begin(), t.shape.end()));
    }
  };
  {
    Safetensors adapter(dir + "/lora/adapter_model.safetensors");
    charge_all(adapter, nullptr);
    if (adapter.entries.empty()) throw std::runtime_error("empty LoRA adapter");
  }
  {
    Safetensors head(dir + "/head.safetensors");
    charge_all(head, nullptr);
  }
  for (const std::string& f : base_files(dir)) {
    Safetensors b(f);
    charge_all(b, &prefix);
  }
}

void load_checkpoint_tensors(Engine& e, const std::string& dir, const LoadLimits& limits) {
  const std::string prefix = "model.language_model.";
  WeightBudget budget(limits);
  auto charge_all = [&](const Safetensors& f, const std::string* pfx) {
    for (const auto& t : f.entries) {
      if (pfx && t.name.compare(0, pfx->size(), *pfx) != 0) continue;
      std::vector<size_t> shape(t.shape.begin(), t.shape.end());
      budget.charge(t.name, shape);
    }
  };
  Safetensors adapter(dir + "/lora/adapter_model.safetensors");
  charge_all(adapter, nullptr);
  if (adapter.entries.empty()) throw std::runtime_error("empty LoRA adapter");
  Safetensors head(dir + "/head.safetensors");
  charge_all(head, nullptr);
  std::vector<std::unique_ptr<Safetensors>> base;
  for (const std::string& f : base_files(dir)) {
    base.emplace_back(new Safetensors(f));
    charge_all(*base.back(), &prefix);
  }
  for (const auto& b : base)
    for (const auto& t : b->entries)
      if (t.name.compare(0, prefix.size(), prefix) == 0) e.set_tensor(t.name.substr(prefix.size()), t.dtype, t.shape, t.data);
  for (const auto& t : adapter.entries) e.set_tensor(t.name, t.dtype, t.shape, t.data);
  for (const auto& t : head.entries) e.set_tensor("head." + t.name, t.dtype, t.shape, t.data);
}

}  // namespace dg
