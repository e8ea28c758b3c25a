// TEST INFRASTRUCTURE ONLY: C entry points of the CPU oracle for tests/ and
// bench.py's cpu_baseline leg (loaded with ctypes). Nothing in the product
// links or loads this library.
#include <map>
#include <mutex>

#include "oracle_model.cpp"  // one translation unit keeps the statics private

using namespace oracle;

namespace {
thread_local std::string g_error;

struct Tensor {
  Data data;
  std::vector<int64_t> shape;
};
struct OracleModel {
  Model m;
  std::map<std::string, Tensor> tensors;  // consumed by or_model_build
};

Data make_data(int dtype, const void* p, size_t n) {
  Data d;
  if (dtype == 0) {
    d.kind = Data::F32;
    d.f32.assign(static_cast<const float*>(p), static_cast<const float*>(p) + n);
  } else {
    d.kind = dtype == 1 ? Data::BF16 : Data::F16;
    d.h16.assign(static_cast<const uint16_t*>(p), static_cast<const uint16_t*>(p) + n);
  }
  return d;
}

Data take(OracleModel* om, const std::string& name, std::vector<int64_t> shape) {
  auto it = om->tensors.find(name);
  if (it == om->tensors.end()) throw std::runtime_error("missing tensor " + name);
  if (it->second.shape != shape) throw std::runtime_error(name + ": unexpected shape");
  Data d = std::move(it->second.data);
  om->tensors.erase(it);
  return d;
}
std::vector<float> take_f32(OracleModel* om, const std::string& name, std::vector<int64_t> shape) {
  return take(om, name, shape).to_f32();
}

// read_tensors' quantization selection, src/weights.rs:346-355, then
// Linear::load + Linear::adapter, src/weights.rs:392-432.
Linear load_linear(OracleModel* om, const std::string& key, size_t input, size_t output,
                   Precision p, size_t rank, float scale, bool lora) {
  Linear l;
  l.input = input;
  l.output = output;
  Data w = take(om, key + ".weight", {int64_t(output), int64_t(input)});
  bool quantizable = key.rfind("layers.", 0) == 0 && key.find("_proj") != std::string::npos;
  l.w = quantizable ? w.quantize(input, p) : w;
  if (lora) {
    l.has_lora = true;
    l.lora_a = take(om, "base_model.model." + key + ".lora_A.weight", {int64_t(rank), int64_t(input)});
    l.lora_b = take(om, "base_model.model." + key + ".lora_B.weight", {int64_t(output), int64_t(rank)});
    l.rank = rank;
    l.scale = scale;
  }
  return l;
}
}  // namespace

extern "C" {

const char* or_last_error() { return g_error.c_str(); }
void or_set_threads(int n) { set_threads(n); }

int32_t or_scalar_dot(const int8_t* a, const uint8_t* b, size_t n) {
  try {
    return scalar_dot(a, b, n);
  } catch (const std::exception& e) {
    g_error = e.what();
    return INT32_MIN;
  }
}
float or_scaled_dot(const int8_t* x, const float* xs, const uint8_t* w, const float* ws, size_t width) {
  return scaled_dot(x, xs, w, ws, width);
}
float or_dot_scores(const float* a, const float* b, size_t n) { return dot_scores(a, b, n); }
void or_softmax(float* v, size_t n) { softmax(v, n); }

// 1 if quantized, 0 if an input is non-finite (QuantizedInputs::new returned None).
int or_quantize_inputs(const float* x, size_t rows, size_t width, int8_t* values, float* scales) {
  std::vector<int8_t> v;
  std::vector<float> s;
  if (!quantize_inputs(x, rows * width, width, v, s)) return 0;
  std::copy(v.begin(), v.end(), values);
  std::copy(s.begin(), s.end(), scales);
  return 1;
}

// Data::quantize of an F32 [rows, width] tensor. bits 8 or 4; values hold
// rows*width bytes (bits 8) or ceil(rows*width/2) bytes (bits 4).
void or_quantize_weights(const float* w, size_t rows, size_t width, int bits, uint8_t* values,
                         float* scales) {
  Data d = make_data(0, w, rows * width);
  Data q = d.quantize(width, bits == 4 ? Int4 : Int8Compute);
  std::copy(q.values.begin(), q.values.end(), values);
  std::copy(q.scales.begin(), q.scales.end(), scales);
}

// One projection through Linear::apply_into: F32 weights [output, input]
// quantized per `precision`, optional bias and LoRA (A [rank,input], B
// [output,rank]), epilogue 0 Write / 1 Add / 2 SwiGlu into `out` [rows, output].
int or_linear(const float* x, size_t rows, size_t input, const float* w, size_t output, int precision,
              const float* bias, const float* lora_a, const float* lora_b, size_t rank, float scale,
              int epilogue, float* out) {
  try {
    Linear l;
    l.input = input;
    l.output = output;
    l.w = make_data(0, w, input * output).quantize(input, Precision(precision));
    if (bias) l.bias.assign(bias, bias + output);
    if (lora_a && lora_b && rank) {
      l.has_lora = true;
      l.lora_a = make_data(0, lora_a, rank * input);
      l.lora_b = make_data(0, lora_b, output * rank);
      l.rank = rank;
      l.scale = scale;
    }
    l.apply_into(x, rows, out, Epilogue(epilogue), nullptr, nullptr);
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// linear_int8 over already-quantized weights (values [output,input] as i8,
// scales [output, ceil(input/64)]), no bias, no LoRA: column sums only.
void or_linear_int8_prequant(const float* x, size_t rows, size_t input, const uint8_t* wq,
                             const float* ws, size_t output, float* out) {
  Data w;
  w.kind = Data::Quantized;
  w.values.assign(wq, wq + input * output);
  w.scales.assign(ws, ws + output * ((input + 63) / 64));
  w.width = input;
  w.elements = input * output;
  w.bits = 8;
  w.compute_int8 = true;
  Projection p{input, output, &w, nullptr, nullptr};
  p.apply_quantized(x, rows, nullptr, out, Epilogue::Write);
}

// dims: hidden, intermediate, layers, vocab, heads, kv_heads, head_dim,
//       conv_kernel, dk, dv, key_heads, value_heads
// fl:   rms_norm_eps, rope_theta, partial_rotary_factor
void* or_model_new(const int64_t* dims, const float* fl, const int32_t* layer_types) {
  auto* om = new OracleModel();
  Config& c = om->m.c;
  c.hidden = dims[0];
  c.intermediate = dims[1];
  c.layers = dims[2];
  c.vocab = dims[3];
  c.heads = dims[4];
  c.kv_heads = dims[5];
  c.head_dim = dims[6];
  c.conv_kernel = dims[7];
  c.dk = dims[8];
  c.dv = dims[9];
  c.key_heads = dims[10];
  c.value_heads = dims[11];
  c.eps = fl[0];
  c.rope_theta = fl[1];
  c.partial_rotary = fl[2];
  c.layer_types.assign(layer_types, layer_types + c.layers);
  return om;
}

// dtype 0 F32, 1 BF16, 2 F16. Base tensors use names without the
// "model.language_model." prefix; adapter tensors keep "base_model.model.";
// pointer-head tensors are named "head.<name>".
void or_model_set(void* h, const char* name, int dtype, const int64_t* shape, int ndim, const void* data) {
  auto* om = static_cast<OracleModel*>(h);
  size_t n = 1;
  std::vector<int64_t> s(shape, shape + ndim);
  for (auto v : s) n *= size_t(v);
  om->tensors[name] = Tensor{make_data(dtype, data, n), s};
}

// Model::load, src/qwen.rs:291-406, and Head::load, src/lib.rs:94-105.
int or_model_build(void* h, int precision, size_t rank, float scale) {
  auto* om = static_cast<OracleModel*>(h);
  Model& m = om->m;
  const Config& c = m.c;
  Precision p = Precision(precision);
  m.precision = precision;
  try {
    int64_t H = c.hidden;
    for (size_t i = 0; i < c.layers; ++i) {
      std::string pre = "layers." + std::to_string(i) + ".";
      Layer L;
      L.full = c.layer_types[i] == 1;
      auto lin = [&](const std::string& n, size_t in, size_t out) {
        return load_linear(om, pre + n, in, out, p, rank, scale, true);
      };
      if (L.full) {
        L.q = lin("self_attn.q_proj", c.hidden, c.heads * c.head_dim * 2);
        L.k = lin("self_attn.k_proj", c.hidden, c.kv_heads * c.head_dim);
        L.v = lin("self_attn.v_proj", c.hidden, c.kv_heads * c.head_dim);
        L.o = lin("self_attn.o_proj", c.heads * c.head_dim, c.hidden);
        L.q_norm = take_f32(om, pre + "self_attn.q_norm.weight", {int64_t(c.head_dim)});
        L.k_norm = take_f32(om, pre + "self_attn.k_norm.weight", {int64_t(c.head_dim)});
      } else {
        size_t kd = c.dk * c.key_heads, vd = c.dv * c.value_heads, w = 2 * kd + vd;
        L.qkv = lin("linear_attn.in_proj_qkv", c.hidden, w);
        L.z = lin("linear_attn.in_proj_z", c.hidden, vd);
        L.a = lin("linear_attn.in_proj_a", c.hidden, c.value_heads);
        L.b = lin("linear_attn.in_proj_b", c.hidden, c.value_heads);
        L.out = lin("linear_attn.out_proj", vd, c.hidden);
        std::vector<float> conv =
            take_f32(om, pre + "linear_attn.conv1d.weight", {int64_t(w), 1, int64_t(c.conv_kernel)});
        // tap_major, src/qwen.rs:698-703
        L.conv.resize(conv.size());
        for (size_t j = 0; j < conv.size(); ++j) L.conv[j] = conv[(j % w) * c.conv_kernel + j / w];
        L.dt = take_f32(om, pre + "linear_attn.dt_bias", {int64_t(c.value_heads)});
        L.decay_rate = take_f32(om, pre + "linear_attn.A_log", {int64_t(c.value_heads)});
        for (auto& v : L.decay_rate) v = -std::exp(v);
        L.norm = take_f32(om, pre + "linear_attn.norm.weight", {int64_t(c.dv)});
      }
      L.gate = lin("mlp.gate_proj", c.hidden, c.intermediate);
      L.up = lin("mlp.up_proj", c.hidden, c.intermediate);
      L.down = lin("mlp.down_proj", c.intermediate, c.hidden);
      L.input_norm = take_f32(om, pre + "input_layernorm.weight", {H});
      L.post_norm = take_f32(om, pre + "post_attention_layernorm.weight", {H});
      m.layers.push_back(std::move(L));
    }
    m.embedding = take(om, "embed_tokens.weight", {int64_t(c.vocab), H});
    m.norm = take_f32(om, "norm.weight", {H});
    if (om->tensors.count("head.norm.weight")) {
      m.has_head = true;
      m.head_norm = take_f32(om, "head.norm.weight", {H});
      m.head_bias = take_f32(om, "head.norm.bias", {H});
      int64_t dim = om->tensors.at("head.q.weight").shape[0];
      m.head_q = load_linear(om, "head.q", c.hidden, dim, Checkpoint, 0, 0, false);
      m.head_q.bias = take_f32(om, "head.q.bias", {dim});
      m.head_k = load_linear(om, "head.k", c.hidden, dim, Checkpoint, 0, 0, false);
      m.head_k.bias = take_f32(om, "head.k.bias", {dim});
    }
    if (!om->tensors.empty())
      throw std::runtime_error(std::to_string(om->tensors.size()) + " unconsumed tensors, e.g. " +
                               om->tensors.begin()->first);
    bool any_full = false;
    for (int t : c.layer_types) any_full |= t == 1;
    size_t r = c.rotary_dim();
    if (any_full)
      for (size_t i = 0; i < r / 2; ++i)
        m.rotary_divisors.push_back(std::pow(c.rope_theta, float(2 * i) / float(r)));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

void or_model_free(void* h) { delete static_cast<OracleModel*>(h); }
void or_prefix_free(void* p) { delete static_cast<Prefix*>(p); }
size_t or_prefix_len(const void* p) { return static_cast<const Prefix*>(p)->len; }

// Model::forward / prefill / forward_after. `hidden_out` (nullable) receives
// [n, hidden]; with capture, *prefix_out receives a new prefix.
int or_forward(void* h, const uint32_t* ids, size_t n, const void* past, int capture, float* hidden_out,
               void** prefix_out) {
  auto* om = static_cast<OracleModel*>(h);
  std::vector<float> x;
  Prefix* cap = capture ? new Prefix() : nullptr;
  std::string err;
  int rc;
  try {
    rc = run(om->m, ids, n, static_cast<const Prefix*>(past), capture != 0, x, cap, err);
  } catch (const std::exception& e) {
    err = e.what();
    rc = 1;
  }
  if (rc) {
    g_error = err;
    delete cap;
    return 1;
  }
  if (hidden_out) std::copy(x.begin(), x.end(), hidden_out);
  if (capture) *prefix_out = cap;
  return 0;
}

// Model::run with every layer's residual rows recorded: trace_out receives
// [layers + 1][n][hidden] (the embedded input, then each layer's output,
// before the final norm).
int or_forward_trace(void* h, const uint32_t* ids, size_t n, float* trace_out) {
  auto* om = static_cast<OracleModel*>(h);
  std::vector<float> x, trace;
  std::string err;
  int rc;
  try {
    rc = run(om->m, ids, n, nullptr, false, x, nullptr, err, &trace);
  } catch (const std::exception& e) {
    err = e.what();
    rc = 1;
  }
  if (rc) {
    g_error = err;
    return 1;
  }
  std::copy(trace.begin(), trace.end(), trace_out);
  return 0;
}

// One layer of the loop teacher-forced on the residual rows x [n][hidden]
// (positions 0..n-1, no prefix); out receives the layer's output rows.
int or_layer(void* h, int layer, const float* x, size_t n, float* out) {
  auto* om = static_cast<OracleModel*>(h);
  const Model& m = om->m;
  if (layer < 0 || size_t(layer) >= m.layers.size() || n == 0 || n > 4096) {
    g_error = "bad layer or row count";
    return 1;
  }
  try {
    std::vector<float> v(x, x + n * m.c.hidden);
    LayerCache cache;
    run_layer(m, size_t(layer), v, n, 0, rotary_angles(m, 0, n), nullptr, &cache);
    std::copy(v.begin(), v.end(), out);
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
  return 0;
}

// or_layer, also returning the FP32 inputs of the layer's four projection
// groups (LayerProbe): in_norm [n][hidden], mix [n][mix_width] (attention
// heads x head_dim, or DeltaNet value heads x dv), post [n][hidden], mlp
// [n][intermediate]. Test infrastructure: the quantised codes of these rows
// are compared with the device's.
int or_layer_probe(void* h, int layer, const float* x, size_t n, float* out, float* in_norm, float* mix,
                   float* post, float* mlp) {
  auto* om = static_cast<OracleModel*>(h);
  const Model& m = om->m;
  if (layer < 0 || size_t(layer) >= m.layers.size() || n == 0 || n > 4096) {
    g_error = "bad layer or row count";
    return 1;
  }
  try {
    std::vector<float> v(x, x + n * m.c.hidden);
    LayerCache cache;
    LayerProbe probe;
    run_layer(m, size_t(layer), v, n, 0, rotary_angles(m, 0, n), nullptr, &cache, &probe);
    std::copy(v.begin(), v.end(), out);
    std::copy(probe.input.begin(), probe.input.end(), in_norm);
    std::copy(probe.mix.begin(), probe.mix.end(), mix);
    std::copy(probe.post.begin(), probe.post.end(), post);
    std::copy(probe.mlp.begin(), probe.mlp.end(), mlp);
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
  return 0;
}

// Head::logits over `rows` hidden rows; the answer row is the last.
int or_head_logits(void* h, const float* hidden, size_t rows, const size_t* positions, size_t n_pos,
                   float* out) {
  auto* om = static_cast<OracleModel*>(h);
  if (!om->m.has_head) {
    g_error = "no pointer head loaded";
    return 1;
  }
  std::vector<float> l = head_logits(om->m, hidden, rows, positions, n_pos);
  std::copy(l.begin(), l.end(), out);
  return 0;
}

// One Recurrence::head pass (src/qwen.rs:813-875) on pre-normalised inputs is
// not a reference entry point; the isolated DeltaNet check instead drives the
// gated delta rule of the recurrence directly: q, k already L2-normalised and
// q pre-scaled by 1/sqrt(dk), per-token decay g (as exp argument) and beta.
// state [dk, dv] is updated in place; o [n, dv] receives q^T S after each token.
void or_gated_delta_rule(const float* q, const float* k, const float* v, const float* g,
                         const float* beta, size_t n, size_t dk, size_t dv, float* state, float* o) {
  std::vector<float> delta(dv);
  for (size_t t = 0; t < n; ++t) {
    float decay = std::exp(g[t]);
    for (size_t i = 0; i < dk * dv; ++i) state[i] = state[i] * decay;
    std::fill(delta.begin(), delta.end(), 0.0f);
    for (size_t i = 0; i < dk; ++i)
      for (size_t j = 0; j < dv; ++j) delta[j] = delta[j] + k[t * dk + i] * state[i * dv + j];
    for (size_t j = 0; j < dv; ++j) delta[j] = (v[t * dv + j] - delta[j]) * beta[t];
    float* ot = o + t * dv;
    for (size_t j = 0; j < dv; ++j) ot[j] = 0.0f;
    for (size_t i = 0; i < dk; ++i)
      for (size_t j = 0; j < dv; ++j) {
        state[i * dv + j] = state[i * dv + j] + k[t * dk + i] * delta[j];
        ot[j] = ot[j] + q[t * dk + i] * state[i * dv + j];
      }
  }
}

}  // extern "C"
