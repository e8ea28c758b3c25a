// TEST INFRASTRUCTURE ONLY. A CPU restatement of decider-engine's prefill path
// (reference crate `decider-engine` v0.2.2), used by tests/ and by bench.py's
// cpu_baseline leg as the checker and the timed CPU baseline. The product path
// never links, loads or calls anything in oracle/.
//
// Parity pin: the restatement is checked against the reference's own golden
// vectors (tests/fixtures/tiny raw-reference.json and reference.json, copied
// into tests/golden/ by tests/golden/make_golden.py) and its known-answer tests
// (src/int8.rs:191-192,263; src/tensor.rs:606-662,769-803).
//
// Arithmetic follows the reference's x86_64 code path: scalar INT8 dots
// (src/int8.rs:149-154), single-dot FP32 columns (TILE = 1, src/tensor.rs:30),
// and the separate LoRA plan for non-accelerated int8-compute
// (src/weights.rs:450-491). Build with -ffp-contract=off and no fast-math so
// every a*b+c rounds twice, as Rust does; transcendental functions are glibc's.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace oracle {

enum Precision { Checkpoint = 0, Int8 = 1, Int8Compute = 2, Int4 = 3 };
enum class Epilogue { Write, Add, SwiGlu };

// ---------------------------------------------------------------- threading
// Work splits mirror rayon's disjoint output slices; arithmetic order per
// output element never depends on the thread count.
void set_threads(int n);
int threads();
void parallel_for(size_t n, const std::function<void(size_t, size_t)>& body);

// ---------------------------------------------------------------- src/int8.rs
// Kernel::dot / scalar_dot, src/int8.rs:34-44,149-154. At most 64 products.
int32_t scalar_dot(const int8_t* a, const uint8_t* b, size_t n);
// Kernel::scaled_dot, src/int8.rs:55-61: group-ordered FP32 sum of
// dot * (xs * ws), no fused multiply-add.
float scaled_dot(const int8_t* x, const float* xs, const uint8_t* w, const float* ws,
                 size_t width);

// ---------------------------------------------------------------- FP32 helpers
// dot_scores, src/tensor.rs:6-25 (x86: eight lanes of `+= a*b`, lanes summed
// from -0.0 in order, then the tail).
float dot_scores(const float* a, const float* b, size_t n);
// softmax, src/tensor.rs:534-546.
void softmax(float* v, size_t n);
// src/qwen.rs:194-206
inline float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float silu(float x) { return x * sigmoid(x); }
inline float softplus(float x) { return x > 20.0f ? x : std::log1p(std::exp(x)); }
// Rust's `f32::sum` on an iterator starts from -0.0 and adds in order.
inline float sum_from_neg_zero(const float* v, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; ++i) s = s + v[i];
  return s;
}
// half(), src/weights.rs:367-382
float half_to_f32(uint16_t v);

// ---------------------------------------------------------------- src/weights.rs Data
struct Data {
  enum Kind { F32, BF16, F16, Quantized } kind = F32;
  std::vector<float> f32;
  std::vector<uint16_t> h16;
  std::vector<uint8_t> values;
  std::vector<float> scales;
  size_t width = 0, elements = 0;
  int bits = 0;
  bool compute_int8 = false;

  size_t len() const;
  // Data::row, src/weights.rs:33-82.
  const float* row(size_t start, size_t n, std::vector<float>& scratch) const;
  std::vector<float> to_f32() const;
  // Data::quantize, src/weights.rs:98-146.
  Data quantize(size_t w, Precision p) const;
};

// ---------------------------------------------------------------- src/tensor.rs
// QuantizedInputs::new, src/tensor.rs:315-353. Returns false (None) if any input
// is non-finite.
bool quantize_inputs(const float* x, size_t len, size_t width, std::vector<int8_t>& values,
                     std::vector<float>& scales);

struct QuantizedInputs {
  std::vector<int8_t> values;
  std::vector<float> scales;
};

struct Adapter {
  const float* inputs;  // rows * rank
  const Data* weights;  // output * rank
  size_t rank;
  float scale;
  // Adapter::combine, src/tensor.rs:109-117.
  float combine(float base, size_t row, const float* w) const {
    float delta = dot_scores(inputs + row * rank, w, rank) + 0.0f;
    return base + scale * delta;
  }
};

struct Projection {
  size_t input, output;
  const Data* weights;
  const float* bias;       // nullable
  const Adapter* adapter;  // nullable
  // Projection::apply_quantized, src/tensor.rs:135-184.
  void apply_quantized(const float* x, size_t rows, const QuantizedInputs* q, float* result,
                       Epilogue e) const;
  // columns_quantized / columns_tiled::<1> / linear_int8, src/tensor.rs:190-269,379-456.
  // Column-major [output][rows]. Returns false if int8 quantization was refused.
  std::vector<float> columns_quantized(const float* x, size_t rows, const QuantizedInputs* q) const;
  std::vector<float> columns_f32(const float* x, size_t rows) const;
  bool linear_int8(const float* x, size_t rows, const QuantizedInputs* q,
                   std::vector<float>& columns) const;
};

inline void store(Epilogue e, float& dst, float value) {
  switch (e) {
    case Epilogue::Write: dst = value; break;
    case Epilogue::Add: dst = dst + value; break;
    case Epilogue::SwiGlu: dst = silu(dst) * value; break;
  }
}

// linear, src/tensor.rs:290-308
void linear(const float* x, size_t rows, size_t input, const Data& w, size_t output,
            const float* bias, float* result);

// ---------------------------------------------------------------- Linear + LoRA
struct Linear {
  Data w;
  std::vector<float> bias;  // empty: none
  size_t input = 0, output = 0;
  bool has_lora = false;
  Data lora_a, lora_b;
  size_t rank = 0;
  float scale = 0.0f;
  // Linear::apply_into_shared, src/weights.rs:446-521. `shared` caches the
  // input's quantization across projections (SharedInput, src/tensor.rs:358-377).
  void apply_into(const float* x, size_t rows, float* out, Epilogue e,
                  std::shared_ptr<QuantizedInputs>* shared, bool* shared_done) const;
  std::vector<float> apply(const float* x, size_t rows) const;
};

}  // namespace oracle
