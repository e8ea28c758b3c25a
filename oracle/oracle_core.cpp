// TEST INFRASTRUCTURE ONLY: CPU restatement of decider-engine's INT8 and FP32
// projection arithmetic. See oracle_core.hpp for the parity pin and build rules.
#include "oracle_core.hpp"

#include <algorithm>
#include <cfloat>
#include <thread>

namespace oracle {

static int g_threads = 1;
void set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int threads() { return g_threads; }

void parallel_for(size_t n, const std::function<void(size_t, size_t)>& body) {
  size_t t = std::min<size_t>(static_cast<size_t>(g_threads), n);
  if (t <= 1) {
    if (n) body(0, n);
    return;
  }
  std::vector<std::thread> pool;
  size_t chunk = (n + t - 1) / t;
  for (size_t i = 0; i < t; ++i) {
    size_t lo = i * chunk, hi = std::min(n, lo + chunk);
    if (lo >= hi) break;
    pool.emplace_back([&, lo, hi] { body(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

// src/int8.rs:149-154
int32_t scalar_dot(const int8_t* a, const uint8_t* b, size_t n) {
  if (n > 64) throw std::runtime_error("dot of more than 64 products");
  int32_t s = 0;
  for (size_t i = 0; i < n; ++i) s += int32_t(a[i]) * int32_t(int8_t(b[i]));
  return s;
}

// src/int8.rs:55-61
float scaled_dot(const int8_t* x, const float* xs, const uint8_t* w, const float* ws,
                 size_t width) {
  float sum = 0.0f;
  size_t groups = (width + 63) / 64;
  for (size_t g = 0; g < groups; ++g) {
    size_t lo = g * 64, n = std::min<size_t>(64, width - lo);
    float s = xs[g] * ws[g];
    sum = sum + float(scalar_dot(x + lo, w + lo, n)) * s;
  }
  return sum;
}

// src/tensor.rs:6-25, x86 branch
float dot_scores(const float* a, const float* b, size_t n) {
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t chunks = n / 8;
  for (size_t c = 0; c < chunks; ++c)
    for (int i = 0; i < 8; ++i) {
      float p = a[c * 8 + i] * b[c * 8 + i];
      lanes[i] = lanes[i] + p;
    }
  float sum = sum_from_neg_zero(lanes, 8);
  for (size_t t = chunks * 8; t < n; ++t) {
    float p = a[t] * b[t];
    sum = sum + p;
  }
  return sum;
}

// src/tensor.rs:534-546
void softmax(float* v, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, v[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    v[i] = std::exp(v[i] - mx);
    sum = sum + v[i];
  }
  if (sum > 0.0f)
    for (size_t i = 0; i < n; ++i) v[i] = v[i] / sum;
}

// src/weights.rs:367-382
float half_to_f32(uint16_t v) {
  float sign = (v & 0x8000) ? -1.0f : 1.0f;
  int e = (v >> 10) & 31;
  int m = v & 1023;
  if (e == 0) return sign * float(m) * std::ldexp(1.0f, -24);
  if (e == 31) return m == 0 ? sign * INFINITY : NAN;
  return sign * (1.0f + float(m) / 1024.0f) * std::ldexp(1.0f, e - 15);
}

static inline float bf16_to_f32(uint16_t v) {
  uint32_t bits = uint32_t(v) << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

size_t Data::len() const {
  switch (kind) {
    case F32: return f32.size();
    case BF16:
    case F16: return h16.size();
    default: return elements;
  }
}

// src/weights.rs:33-82
const float* Data::row(size_t start, size_t n, std::vector<float>& scratch) const {
  switch (kind) {
    case F32: return f32.data() + start;
    case BF16:
      scratch.resize(n);
      for (size_t i = 0; i < n; ++i) scratch[i] = bf16_to_f32(h16[start + i]);
      return scratch.data();
    case F16:
      scratch.resize(n);
      for (size_t i = 0; i < n; ++i) scratch[i] = half_to_f32(h16[start + i]);
      return scratch.data();
    default: {
      size_t groups = (width + 63) / 64;
      scratch.resize(n);
      for (size_t i = start; i < start + n; ++i) {
        size_t r = i / width, off = i % width;
        float scale = scales[r * groups + off / 64];
        float q;
        if (bits == 8) {
          q = float(int8_t(values[i]));
        } else {
          int nib = (values[i / 2] >> (4 * (i % 2))) & 15;
          q = float(nib) - 8.0f;
        }
        scratch[i - start] = q * scale;
      }
      return scratch.data();
    }
  }
}

std::vector<float> Data::to_f32() const {
  std::vector<float> out, scratch;
  const float* p = row(0, len(), scratch);
  out.assign(p, p + len());
  return out;
}

// src/weights.rs:98-146
Data Data::quantize(size_t w, Precision p) const {
  if (p == Checkpoint) return *this;
  int b = (p == Int4) ? 4 : 8;
  size_t el = len();
  if (w == 0 || el % w) throw std::runtime_error("quantize: bad width");
  Data out;
  out.kind = Quantized;
  out.width = w;
  out.elements = el;
  out.bits = b;
  out.compute_int8 = (p == Int8Compute);
  out.values.assign(b == 8 ? el : (el + 1) / 2, 0);
  size_t groups = (w + 63) / 64;
  out.scales.resize((el / w) * groups);
  float bound = b == 8 ? 127.0f : 7.0f;
  std::vector<float> scratch;
  for (size_t r = 0; r < el / w; ++r) {
    const float* weights = row(r * w, w, scratch);
    for (size_t g = 0; g < groups; ++g) {
      size_t lo = g * 64, n = std::min<size_t>(64, w - lo);
      float mx = 0.0f;
      for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs(weights[lo + i]));
      float scale = mx == 0.0f ? 1.0f : std::fmax(mx / bound, FLT_MIN);
      out.scales[r * groups + g] = scale;
      for (size_t i = 0; i < n; ++i) {
        size_t index = r * w + lo + i;
        float q = std::round(weights[lo + i] / scale);
        q = std::fmin(std::fmax(q, -bound), bound);
        int8_t qi = int8_t(q);
        if (b == 8)
          out.values[index] = uint8_t(qi);
        else
          out.values[index / 2] |= uint8_t(uint8_t(qi + 8) << (4 * (index % 2)));
      }
    }
  }
  return out;
}

// src/tensor.rs:315-353
bool quantize_inputs(const float* x, size_t len, size_t width, std::vector<int8_t>& values,
                     std::vector<float>& scales) {
  for (size_t i = 0; i < len; ++i)
    if (!std::isfinite(x[i])) return false;
  size_t groups = (width + 63) / 64;
  size_t rows = len / width;
  values.assign(len, 0);
  scales.assign(rows * groups, 0.0f);
  parallel_for(rows, [&](size_t r0, size_t r1) {
    for (size_t r = r0; r < r1; ++r)
      for (size_t g = 0; g < groups; ++g) {
        size_t lo = g * 64, n = std::min<size_t>(64, width - lo);
        const float* v = x + r * width + lo;
        float mx = 0.0f;
        for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs(v[i]));
        float scale = mx == 0.0f ? 1.0f : std::fmax(mx / 127.0f, FLT_MIN);
        scales[r * groups + g] = scale;
        for (size_t i = 0; i < n; ++i) {
          float q = std::round(v[i] / scale);
          q = std::fmin(std::fmax(q, -127.0f), 127.0f);
          values[r * width + lo + i] = int8_t(q);
        }
      }
  });
  return true;
}

// linear_int8, src/tensor.rs:379-456 (x86: per-output scaled_dot).
bool Projection::linear_int8(const float* x, size_t rows, const QuantizedInputs* shared,
                             std::vector<float>& columns) const {
  QuantizedInputs owned;
  const QuantizedInputs* q = shared;
  if (!q) {
    if (!quantize_inputs(x, rows * input, input, owned.values, owned.scales)) return false;
    q = &owned;
  }
  size_t groups = (input + 63) / 64;
  columns.assign(rows * output, 0.0f);
  const Data& w = *weights;
  parallel_for(output, [&](size_t c0, size_t c1) {
    std::vector<float> scratch;
    for (size_t column = c0; column < c1; ++column) {
      const uint8_t* wv = w.values.data() + column * input;
      const float* wsc = w.scales.data() + column * groups;
      const float* aw = adapter ? adapter->weights->row(column * adapter->rank, adapter->rank, scratch)
                                : nullptr;
      for (size_t r = 0; r < rows; ++r) {
        float sum = scaled_dot(q->values.data() + r * input, q->scales.data() + r * groups, wv,
                               wsc, input);
        float base = sum + (bias ? bias[column] : 0.0f);
        columns[column * rows + r] = adapter ? adapter->combine(base, r, aw) : base;
      }
    }
  });
  return true;
}

// columns_tiled::<1>, src/tensor.rs:206-269
std::vector<float> Projection::columns_f32(const float* x, size_t rows) const {
  std::vector<float> columns(rows * output, 0.0f);
  parallel_for(output, [&](size_t c0, size_t c1) {
    std::vector<float> ws, as;
    for (size_t column = c0; column < c1; ++column) {
      const float* w = weights->row(column * input, input, ws);
      for (size_t r = 0; r < rows; ++r) columns[column * rows + r] = dot_scores(x + r * input, w, input);
      const float* aw = adapter ? adapter->weights->row(column * adapter->rank, adapter->rank, as)
                                : nullptr;
      float b = bias ? bias[column] : 0.0f;
      for (size_t r = 0; r < rows; ++r) {
        float base = columns[column * rows + r] + b;
        columns[column * rows + r] = adapter ? adapter->combine(base, r, aw) : base;
      }
    }
  });
  return columns;
}

// src/tensor.rs:190-202
std::vector<float> Projection::columns_quantized(const float* x, size_t rows,
                                                 const QuantizedInputs* q) const {
  if (weights->kind == Data::Quantized && weights->bits == 8 && weights->compute_int8) {
    std::vector<float> columns;
    if (linear_int8(x, rows, q, columns)) return columns;
  }
  return columns_f32(x, rows);
}

// write_columns, src/tensor.rs:272-288
static void write_columns(const std::vector<float>& columns, const std::vector<float>* delta,
                          float scale, size_t rows, size_t output, float* result, Epilogue e) {
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < output; ++c) {
      size_t index = c * rows + r;
      float base = columns[index];
      float projected = delta ? base + scale * (*delta)[index] : base;
      store(e, result[r * output + c], projected);
    }
}

// src/tensor.rs:135-184
void Projection::apply_quantized(const float* x, size_t rows, const QuantizedInputs* q,
                                 float* result, Epilogue e) const {
  if (rows == 0) return;
  if (adapter && rows >= 64) {
    Projection base{input, output, weights, bias, nullptr};
    std::vector<float> b = base.columns_quantized(x, rows, q);
    Projection d{adapter->rank, output, adapter->weights, nullptr, nullptr};
    std::vector<float> delta = d.columns_f32(adapter->inputs, rows);
    write_columns(b, &delta, adapter->scale, rows, output, result, e);
  } else {
    std::vector<float> columns = columns_quantized(x, rows, q);
    write_columns(columns, nullptr, 0.0f, rows, output, result, e);
  }
}

// src/tensor.rs:290-308
void linear(const float* x, size_t rows, size_t input, const Data& w, size_t output,
            const float* bias, float* result) {
  Projection p{input, output, &w, bias, nullptr};
  p.apply_quantized(x, rows, nullptr, result, Epilogue::Write);
}

// src/weights.rs:446-521
void Linear::apply_into(const float* x, size_t rows, float* out, Epilogue e,
                        std::shared_ptr<QuantizedInputs>* shared, bool* shared_done) const {
  const float* b = bias.empty() ? nullptr : bias.data();
  bool int8_compute = w.kind == Data::Quantized && w.compute_int8;
  if (int8_compute) {
    // Separate plan of the non-accelerated (x86) INT8 kernel, src/weights.rs:450-491.
    bool direct = e == Epilogue::Write;
    std::vector<float> temporary;
    float* values = out;
    if (!direct) {
      temporary.assign(rows * output, 0.0f);
      values = temporary.data();
    }
    // `linear` quantizes its input afresh; the result equals the shared copy.
    const QuantizedInputs* q = nullptr;
    if (shared) {
      if (!*shared_done) {
        auto qi = std::make_shared<QuantizedInputs>();
        if (quantize_inputs(x, rows * input, input, qi->values, qi->scales)) *shared = qi;
        *shared_done = true;
      }
      q = shared->get();
    }
    Projection p{input, output, &w, b, nullptr};
    p.apply_quantized(x, rows, q, values, Epilogue::Write);
    if (has_lora) {
      std::vector<float> mid(rows * rank), delta(rows * output);
      linear(x, rows, input, lora_a, rank, nullptr, mid.data());
      linear(mid.data(), rows, rank, lora_b, output, nullptr, delta.data());
      for (size_t i = 0; i < rows * output; ++i) values[i] = values[i] + scale * delta[i];
    }
    if (!direct)
      for (size_t i = 0; i < rows * output; ++i) store(e, out[i], temporary[i]);
    return;
  }
  std::vector<float> mid;
  Adapter ad{};
  if (has_lora) {
    mid.assign(rows * rank, 0.0f);
    linear(x, rows, input, lora_a, rank, nullptr, mid.data());
    ad = Adapter{mid.data(), &lora_b, rank, scale};
  }
  Projection p{input, output, &w, b, has_lora ? &ad : nullptr};
  p.apply_quantized(x, rows, nullptr, out, e);
}

std::vector<float> Linear::apply(const float* x, size_t rows) const {
  std::vector<float> out(rows * output, 0.0f);
  apply_into(x, rows, out.data(), Epilogue::Write, nullptr, nullptr);
  return out;
}

}  // namespace oracle
