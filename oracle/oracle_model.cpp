// TEST INFRASTRUCTURE ONLY: CPU restatement of decider-engine's Qwen3.5 torso
// (src/qwen.rs), pointer head (src/lib.rs:87-131) and readout
// (src/lib.rs:525-548). See oracle_core.hpp for the parity pin and build rules.
#include <algorithm>
#include <cstdio>

#include "oracle_core.hpp"

namespace oracle {

// Config, src/qwen.rs:8-34 (text_config fields the forward pass reads).
struct Config {
  size_t hidden, intermediate, layers, vocab, heads, kv_heads, head_dim;
  float eps;
  size_t conv_kernel, dk, dv, key_heads, value_heads;
  float rope_theta, partial_rotary;
  std::vector<int> layer_types;  // 1 = full_attention, 0 = linear_attention
  size_t rotary_dim() const { return size_t(float(head_dim) * partial_rotary); }
};

// src/qwen.rs:208-217
static void rms(float* x, size_t len, const float* w, size_t n, float eps, bool centered) {
  for (size_t r = 0; r < len / n; ++r) {
    float* row = x + r * n;
    float s = -0.0f;
    for (size_t i = 0; i < n; ++i) s = s + row[i] * row[i];
    float inv = 1.0f / std::sqrt(s / float(n) + eps);
    for (size_t i = 0; i < n; ++i) row[i] = row[i] * (inv * (centered ? 1.0f + w[i] : w[i]));
  }
}

// src/qwen.rs:218-237
static void residual_norm(float* x, const float* residual, float* normalized, const float* w,
                          size_t n, size_t len, float eps) {
  for (size_t r = 0; r < len / n; ++r) {
    float s = -0.0f;
    for (size_t i = 0; i < n; ++i) {
      size_t k = r * n + i;
      x[k] = x[k] + residual[k];
      normalized[k] = x[k];
      s = s + x[k] * x[k];
    }
    float inv = 1.0f / std::sqrt(s / float(n) + eps);
    for (size_t i = 0; i < n; ++i) {
      size_t k = r * n + i;
      normalized[k] = normalized[k] * (inv * (1.0f + w[i]));
    }
  }
}

// src/qwen.rs:238-246
static void rotary(float* x, const float* sin_cos, size_t half) {
  for (size_t i = 0; i < half; ++i) {
    float s = sin_cos[2 * i], c = sin_cos[2 * i + 1];
    float a = x[i], b = x[i + half];
    x[i] = a * c - b * s;
    x[i + half] = b * c + a * s;
  }
}

struct LayerCache {
  bool full = false;
  std::vector<float> k, v;        // full attention: normalized, rotated keys and values
  std::vector<float> tail, state; // DeltaNet: conv inputs and recurrent state
};
struct Prefix {
  size_t len = 0;
  std::vector<LayerCache> layers;
};

struct Layer {
  bool full = false;
  std::vector<float> input_norm, post_norm;
  Linear q, k, v, o;                     // full attention
  std::vector<float> q_norm, k_norm;
  Linear qkv, z, a, b, out;              // DeltaNet
  std::vector<float> conv, dt, decay_rate, norm;  // conv tap-major
  Linear gate, up, down;
};

struct Model {
  Config c;
  Data embedding;
  std::vector<Layer> layers;
  std::vector<float> norm, rotary_divisors;
  int precision = 0;
  // Pointer head, src/lib.rs:87-131.
  bool has_head = false;
  std::vector<float> head_norm, head_bias;
  Linear head_q, head_k;
};

// causal_attention, src/qwen.rs:590-643
static std::vector<float> causal_attention(const float* q, const float* k, const float* v, size_t n,
                                           size_t heads, size_t key_heads, size_t d, size_t offset) {
  size_t qw = heads * d, kw = key_heads * d;
  std::vector<float> out(n * qw, 0.0f);
  float scale = 1.0f / std::sqrt(float(d));
  parallel_for(n, [&](size_t t0, size_t t1) {
    std::vector<float> scores;
    for (size_t t = t0; t < t1; ++t)
      for (size_t h = 0; h < heads; ++h) {
        size_t kh = h / (heads / key_heads);
        const float* query = q + t * qw + h * d;
        scores.resize(offset + t + 1);
        for (size_t s = 0; s <= offset + t; ++s)
          scores[s] = dot_scores(query, k + s * kw + kh * d, d) * scale;
        softmax(scores.data(), scores.size());
        float* dst = out.data() + t * qw + h * d;
        for (size_t s = 0; s < scores.size(); ++s) {
          const float* vs = v + s * kw + kh * d;
          for (size_t i = 0; i < d; ++i) dst[i] = dst[i] + scores[s] * vs[i];
        }
      }
  });
  return out;
}

// Full::forward, src/qwen.rs:530-585
static std::vector<float> full_forward(const Layer& L, const Config& c, const float* x, size_t n,
                                       const std::vector<float>& angles, const LayerCache* past,
                                       LayerCache* next, std::vector<float>* mix_probe = nullptr) {
  size_t d = c.head_dim, qw = c.heads * d, kw = c.kv_heads * d;
  std::shared_ptr<QuantizedInputs> shared;
  bool done = false;
  std::vector<float> raw_q(n * 2 * qw), k(n * kw), v(n * kw);
  L.q.apply_into(x, n, raw_q.data(), Epilogue::Write, &shared, &done);
  std::vector<float> q(n * qw), gate(n * qw);
  for (size_t t = 0; t < n; ++t)
    for (size_t h = 0; h < c.heads; ++h) {
      size_t src = t * qw * 2 + h * d * 2, dst = t * qw + h * d;
      std::copy(raw_q.begin() + src, raw_q.begin() + src + d, q.begin() + dst);
      std::copy(raw_q.begin() + src + d, raw_q.begin() + src + 2 * d, gate.begin() + dst);
    }
  L.k.apply_into(x, n, k.data(), Epilogue::Write, &shared, &done);
  L.v.apply_into(x, n, v.data(), Epilogue::Write, &shared, &done);
  rms(q.data(), q.size(), L.q_norm.data(), d, c.eps, true);
  rms(k.data(), k.size(), L.k_norm.data(), d, c.eps, true);
  size_t half = c.rotary_dim() / 2;
  for (size_t t = 0; t < n; ++t) {
    const float* a = angles.data() + t * half * 2;
    for (size_t h = 0; h < c.heads; ++h) rotary(q.data() + t * qw + h * d, a, half);
    for (size_t h = 0; h < c.kv_heads; ++h) rotary(k.data() + t * kw + h * d, a, half);
  }
  std::vector<float> keys, values;
  size_t offset = 0;
  if (past) {
    offset = past->k.size() / kw;
    keys = past->k;
    keys.insert(keys.end(), k.begin(), k.end());
    values = past->v;
    values.insert(values.end(), v.begin(), v.end());
  } else {
    keys = k;
    values = v;
  }
  std::vector<float> out =
      causal_attention(q.data(), keys.data(), values.data(), n, c.heads, c.kv_heads, d, offset);
  for (size_t i = 0; i < out.size(); ++i) out[i] = out[i] * sigmoid(gate[i]);
  if (mix_probe) *mix_probe = out;
  next->full = true;
  next->k = std::move(keys);
  next->v = std::move(values);
  // The reference returns only this call's keys; a continuation concatenates
  // them onto the prefix, so storing the joined arrays is equivalent.
  return L.o.apply(out.data(), n);
}

// convolve, src/qwen.rs:712-756
static std::vector<float> convolve(const float* raw, size_t n, const float* tail, size_t tail_rows,
                                   size_t start, size_t width, size_t kernel, const float* taps) {
  std::vector<float> conv(n * width, 0.0f);
  parallel_for(n, [&](size_t t0, size_t t1) {
    for (size_t t = t0; t < t1; ++t) {
      float* out = conv.data() + t * width;
      size_t position = start + t;
      for (size_t j = 0; j < kernel; ++j) {
        if (position + j + 1 < kernel) continue;
        size_t source = position + j + 1 - kernel;
        const float* input = source >= start ? raw + (source - start) * width
                                             : tail + (source + tail_rows - start) * width;
        const float* w = taps + j * width;
        for (size_t ch = 0; ch < width; ++ch) out[ch] = out[ch] + input[ch] * w[ch];
      }
      for (size_t ch = 0; ch < width; ++ch) out[ch] = silu(out[ch]);
    }
  });
  return conv;
}

// Recurrence::head, src/qwen.rs:813-875
static void recurrence_head(const Layer& L, const Config& c, size_t head, const float* conv, size_t n,
                            const float* a, const float* b, const float* z, float* dst, float* state) {
  size_t dk = c.dk, dv = c.dv, heads = c.value_heads, kd = c.key_heads * dk, vd = heads * dv;
  size_t width = 2 * kd + vd, kh = head / (heads / c.key_heads);
  std::vector<float> q(dk), k(dk), delta(dv);
  for (size_t t = 0; t < n; ++t) {
    float* o = dst + t * dv;
    std::copy(conv + t * width + kh * dk, conv + t * width + (kh + 1) * dk, q.begin());
    std::copy(conv + t * width + kd + kh * dk, conv + t * width + kd + (kh + 1) * dk, k.begin());
    float sq = -0.0f, sk = -0.0f;
    for (size_t i = 0; i < dk; ++i) sq = sq + q[i] * q[i];
    for (size_t i = 0; i < dk; ++i) sk = sk + k[i] * k[i];
    float qnorm = (1.0f / std::sqrt(sq + 1e-6f)) / std::sqrt(float(dk));
    float knorm = 1.0f / std::sqrt(sk + 1e-6f);
    for (auto& v : q) v = v * qnorm;
    for (auto& v : k) v = v * knorm;
    float decay = std::exp(L.decay_rate[head] * softplus(a[t * heads + head] + L.dt[head]));
    float beta = sigmoid(b[t * heads + head]);
    for (size_t i = 0; i < dk * dv; ++i) state[i] = state[i] * decay;
    std::fill(delta.begin(), delta.end(), 0.0f);
    for (size_t i = 0; i < dk; ++i)
      for (size_t j = 0; j < dv; ++j) delta[j] = delta[j] + k[i] * state[i * dv + j];
    const float* v = conv + t * width + 2 * kd + head * dv;
    for (size_t j = 0; j < dv; ++j) delta[j] = (v[j] - delta[j]) * beta;
    for (size_t i = 0; i < dk; ++i)
      for (size_t j = 0; j < dv; ++j) {
        state[i * dv + j] = state[i * dv + j] + k[i] * delta[j];
        o[j] = o[j] + q[i] * state[i * dv + j];
      }
    rms(o, dv, L.norm.data(), dv, c.eps, false);
    const float* g = z + t * vd + head * dv;
    for (size_t j = 0; j < dv; ++j) o[j] = o[j] * silu(g[j]);
  }
}

// Delta::forward, src/qwen.rs:649-694 (+ Recurrence::run 775-809)
static std::vector<float> delta_forward(const Layer& L, const Config& c, const float* x, size_t n,
                                        size_t start, const LayerCache* past, LayerCache* next,
                                        std::vector<float>* mix_probe = nullptr) {
  size_t dk = c.dk, dv = c.dv, kd = c.key_heads * dk, vd = c.value_heads * dv;
  size_t width = 2 * kd + vd, heads = c.value_heads;
  std::shared_ptr<QuantizedInputs> shared;
  bool done = false;
  std::vector<float> raw(n * width), z(n * vd), a(n * heads), b(n * heads);
  L.qkv.apply_into(x, n, raw.data(), Epilogue::Write, &shared, &done);
  L.z.apply_into(x, n, z.data(), Epilogue::Write, &shared, &done);
  L.a.apply_into(x, n, a.data(), Epilogue::Write, &shared, &done);
  L.b.apply_into(x, n, b.data(), Epilogue::Write, &shared, &done);
  size_t kernel = c.conv_kernel;
  static const std::vector<float> empty;
  const std::vector<float>& tail = past ? past->tail : empty;
  size_t tail_rows = tail.size() / width;
  if (tail_rows != std::min(start, kernel - 1)) throw std::runtime_error("tail rows mismatch");
  std::vector<float> conv = convolve(raw.data(), n, tail.data(), tail_rows, start, width, kernel,
                                     L.conv.data());
  std::vector<float> state = past ? past->state : std::vector<float>(heads * dk * dv, 0.0f);
  std::vector<float> by_head(heads * n * dv, 0.0f);
  parallel_for(heads, [&](size_t h0, size_t h1) {
    for (size_t h = h0; h < h1; ++h)
      recurrence_head(L, c, h, conv.data(), n, a.data(), b.data(), z.data(),
                      by_head.data() + h * n * dv, state.data() + h * dk * dv);
  });
  std::vector<float> out(n * vd);
  for (size_t h = 0; h < heads; ++h)
    for (size_t t = 0; t < n; ++t)
      std::copy(by_head.begin() + (h * n + t) * dv, by_head.begin() + (h * n + t + 1) * dv,
                out.begin() + t * vd + h * dv);
  size_t keep = std::min(start + n, kernel - 1);
  size_t from_tail = keep > n ? keep - n : 0;
  next->full = false;
  next->tail.assign(tail.begin() + (tail_rows - from_tail) * width, tail.end());
  next->tail.insert(next->tail.end(), raw.begin() + (n - (keep - from_tail)) * width, raw.end());
  next->state = std::move(state);
  if (mix_probe) *mix_probe = out;
  return L.out.apply(out.data(), n);
}

// Rotary angles of positions start..start+n-1 (src/qwen.rs:452-458).
static std::vector<float> rotary_angles(const Model& m, size_t start, size_t n) {
  size_t half = m.rotary_divisors.size();
  std::vector<float> angles(n * half * 2);
  for (size_t t = 0; t < n; ++t)
    for (size_t i = 0; i < half; ++i) {
      float a = float(start + t) / m.rotary_divisors[i];
      angles[(t * half + i) * 2] = std::sin(a);
      angles[(t * half + i) * 2 + 1] = std::cos(a);
    }
  return angles;
}

// FP32 inputs of a layer's four projection groups, recorded for parity
// checks of the quantised activations (not part of the reference): the
// normalised input rows (q/k/v or qkv/z/a/b), the mixer output (o_proj or
// out_proj), the normalised post-mixer rows (gate/up) and the SwiGLU rows
// (down_proj).
struct LayerProbe {
  std::vector<float> input, mix, post, mlp;
};

// One pass of the layer loop of Model::run (src/qwen.rs:470-494) on the
// residual rows x [n, hidden]: input norm, Full/Delta forward, residual_norm,
// SwiGLU MLP with the residual add.
static void run_layer(const Model& m, size_t i, std::vector<float>& x, size_t n, size_t start,
                      const std::vector<float>& angles, const LayerCache* lp, LayerCache* cache,
                      LayerProbe* probe = nullptr) {
  const Config& c = m.c;
  size_t h = c.hidden;
  const Layer& L = m.layers[i];
  std::vector<float> nrm = x;
  rms(nrm.data(), nrm.size(), L.input_norm.data(), h, c.eps, true);
  if (probe) probe->input = nrm;
  std::vector<float>* mp = probe ? &probe->mix : nullptr;
  std::vector<float> mixed = L.full ? full_forward(L, c, nrm.data(), n, angles, lp, cache, mp)
                                    : delta_forward(L, c, nrm.data(), n, start, lp, cache, mp);
  residual_norm(x.data(), mixed.data(), nrm.data(), L.post_norm.data(), h, x.size(), c.eps);
  if (probe) probe->post = nrm;
  std::shared_ptr<QuantizedInputs> shared;
  bool done = false;
  std::vector<float> gate(n * c.intermediate);
  L.gate.apply_into(nrm.data(), n, gate.data(), Epilogue::Write, &shared, &done);
  L.up.apply_into(nrm.data(), n, gate.data(), Epilogue::SwiGlu, &shared, &done);
  if (probe) probe->mlp = gate;
  L.down.apply_into(gate.data(), n, x.data(), Epilogue::Add, nullptr, nullptr);
}

// Model::run, src/qwen.rs:426-504. Returns 0, or an error message in `err`.
static int run(const Model& m, const uint32_t* ids, size_t n, const Prefix* past, bool capture,
               std::vector<float>& x, Prefix* captured, std::string& err,
               std::vector<float>* layer_trace = nullptr) {
  const Config& c = m.c;
  size_t start = past ? past->len : 0;
  if (n == 0 || start + n > 4096) {
    err = "token sequence must contain 1\xe2\x80\x93" "4096 tokens";
    return 1;
  }
  size_t h = c.hidden;
  x.assign(n * h, 0.0f);
  std::vector<float> scratch;
  for (size_t t = 0; t < n; ++t) {
    if (ids[t] >= c.vocab) {
      err = "token " + std::to_string(ids[t]) + " outside vocabulary";
      return 1;
    }
    const float* row = m.embedding.row(size_t(ids[t]) * h, h, scratch);
    std::copy(row, row + h, x.begin() + t * h);
  }
  std::vector<float> angles = rotary_angles(m, start, n);
  if (layer_trace) layer_trace->assign(x.begin(), x.end());
  if (captured) captured->layers.clear();
  for (size_t i = 0; i < m.layers.size(); ++i) {
    const LayerCache* lp = past ? &past->layers[i] : nullptr;
    if (lp && lp->full != m.layers[i].full) {
      err = "prefix cache does not match the layer types";
      return 1;
    }
    LayerCache cache;
    run_layer(m, i, x, n, start, angles, lp, &cache);
    if (layer_trace) layer_trace->insert(layer_trace->end(), x.begin(), x.end());
    if (capture) captured->layers.push_back(std::move(cache));
  }
  rms(x.data(), x.size(), m.norm.data(), h, c.eps, true);
  for (float v : x)
    if (!std::isfinite(v)) {
      err = "non-finite Qwen hidden states";
      return 1;
    }
  if (capture) captured->len = start + n;
  return 0;
}

// Head::normalize, src/lib.rs:106-115
static std::vector<float> head_normalize(const Model& m, const float* x, size_t n) {
  float mean = sum_from_neg_zero(x, n) / float(n);
  float var = -0.0f;
  for (size_t i = 0; i < n; ++i) var = var + (x[i] - mean) * (x[i] - mean);
  var = var / float(n);
  float inv = 1.0f / std::sqrt(var + 1e-5f);
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = (x[i] - mean) * inv * m.head_norm[i] + m.head_bias[i];
  return out;
}

// Head::logits, src/lib.rs:116-131. `hidden` holds `rows` rows; the answer is the last.
static std::vector<float> head_logits(const Model& m, const float* hidden, size_t rows,
                                      const size_t* positions, size_t n_pos) {
  size_t size = m.head_norm.size();
  std::vector<float> nq = head_normalize(m, hidden + (rows - 1) * size, size);
  std::vector<float> query = m.head_q.apply(nq.data(), 1);
  float scale = 1.0f / std::sqrt(float(m.head_q.output));
  std::vector<float> out(n_pos);
  for (size_t p = 0; p < n_pos; ++p) {
    std::vector<float> nk = head_normalize(m, hidden + positions[p] * size, size);
    std::vector<float> key = m.head_k.apply(nk.data(), 1);
    out[p] = dot_scores(query.data(), key.data(), query.size()) * scale;
  }
  return out;
}

}  // namespace oracle
