// Engine construction: tensor staging, load-time weight quantisation (bit-exact
// with Data::quantize, src/weights.rs:98-146), device layouts and workspaces.
#include <cstdlib>
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>

#include "engine.h"

namespace dg {

// ---------------------------------------------------------------- DevBuf
DevBuf::DevBuf(size_t n) : bytes(n) {
  if (n) DG_CUDA(cudaMalloc(&ptr, n));
}
DevBuf DevBuf::pooled_on(size_t n, cudaStream_t s) {
  DevBuf b;
  b.bytes = n;
  b.pooled = true;
  DG_CUDA(cudaGetDevice(&b.device));
  if (n) DG_CUDA(cudaMallocAsync(&b.ptr, n, s));
  return b;
}

// The device's default stream-ordered pool keeps up to 4 GiB of released
// prefix blocks while any engine lives on the device (instead of returning
// them to the driver at every synchronisation). The first engine on a device
// saves the pool's release threshold and raises it; the last one trims the
// pool and restores the threshold, so the retained memory does not outlive
// the engines. (The prefixes use the default pool rather than a pool of
// their own: profilers track allocations from the default pool.)
namespace {
std::mutex g_pool_mu;
int g_pool_users[64] = {};
uint64_t g_pool_saved[64] = {};
}  // namespace

void prefix_pool_acquire(int device) {
  if (device < 0 || device >= 64) return;
  std::lock_guard<std::mutex> lk(g_pool_mu);
  if (g_pool_users[device]++ == 0) {
    cudaMemPool_t pool = nullptr;
    DG_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    DG_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &g_pool_saved[device]));
    uint64_t keep = uint64_t(4) << 30;
    DG_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
  }
}

void prefix_pool_release(int device) {
  if (device < 0 || device >= 64) return;
  std::lock_guard<std::mutex> lk(g_pool_mu);
  if (g_pool_users[device] > 0 && --g_pool_users[device] == 0) {
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &g_pool_saved[device]);
      cudaMemPoolTrimTo(pool, 0);
    }
  }
}
// A pooled buffer goes back on the legacy stream: every use of a prefix
// buffer is a forward on the engine stream that the host has synchronised
// before returning, so nothing is in flight when it is released.
static void release(void* p, bool pooled, int device) {
  if (!p) return;
  if (!pooled) {
    cudaFree(p);
    return;
  }
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != device) cudaSetDevice(device);
  cudaFreeAsync(p, 0);  // the legacy stream of the pool's device
  if (cur != device && cur >= 0) cudaSetDevice(cur);
}
DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
  if (this != &o) {
    if (!borrowed) release(ptr, pooled, device);
    ptr = o.ptr;
    bytes = o.bytes;
    pooled = o.pooled;
    device = o.device;
    borrowed = o.borrowed;
    o.ptr = nullptr;
    o.bytes = 0;
    o.pooled = false;
    o.borrowed = false;
  }
  return *this;
}
DevBuf::~DevBuf() {
  if (!borrowed) release(ptr, pooled, device);
}

static void host_parallel(size_t n, const std::function<void(size_t, size_t)>& f) {
  size_t t = std::min<size_t>(std::max(1u, std::thread::hardware_concurrency()), 32);
  t = std::min(t, std::max<size_t>(1, n / 64));
  if (t <= 1) {
    if (n) f(0, n);
    return;
  }
  std::vector<std::thread> pool;
  size_t chunk = (n + t - 1) / t;
  for (size_t i = 0; i < t; ++i) {
    size_t lo = i * chunk, hi = std::min(n, lo + chunk);
    if (lo < hi) pool.emplace_back([&, lo, hi] { f(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

// Config::validate, src/qwen.rs:133-188 (the checks the forward pass relies on).
void Config::validate() const {
  const int dims[] = {hidden, intermediate, layers, vocab, heads, kv_heads, head_dim,
                      conv_kernel, dk, dv, key_heads, value_heads};
  for (int d : dims)
    if (d <= 0 || d > 1000000) throw std::runtime_error("invalid Qwen dimensions");
  if (int(layer_types.size()) != layers) throw std::runtime_error("invalid Qwen layer_types");
  if (heads % kv_heads || value_heads % key_heads)
    throw std::runtime_error("key head counts must divide query/value head counts");
  const int r = rotary_dim();
  if (!std::isfinite(eps) || eps <= 0 || !std::isfinite(rope_theta) || rope_theta <= 0 || r == 0 ||
      r > head_dim || r % 2)
    throw std::runtime_error("unsupported Qwen normalization, activation, attention, or RoPE config");
  if (rank < 0 || (rank > 0 && !(lora_scale > 0.0f))) throw std::runtime_error("invalid LoRA rank or scale");
}

// ---------------------------------------------------------------- Engine
Engine::Engine(const Config& c, int precision, int device, int max_tokens)
    : c_(c), precision_(precision), device_(device), max_tokens_(max_tokens) {
  c_.validate();
  if (precision < 0 || precision > 3) throw std::runtime_error("unknown precision");
  if (max_tokens <= 0 || max_tokens > 4096) throw std::runtime_error("max_tokens must be in 1..4096");
  DG_CUDA(cudaSetDevice(device));
  int major = 0;
  DG_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  if (major != 10) throw std::runtime_error("decider GPU kernels need an sm_100 (B200) device");
  DG_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  DG_CUDA(cudaEventCreate(&ev0_));
  DG_CUDA(cudaEventCreate(&ev1_));
  // DG_CUDA_GRAPHS=0 launches every forward kernel by kernel (A/B timing).
  if (const char* g = std::getenv("DG_CUDA_GRAPHS")) graphs_on_ = std::atoi(g) != 0;
  if (const char* o = std::getenv("DG_LORA_OVERLAP")) lora_overlap_ = std::atoi(o) != 0;
  if (const char* b = std::getenv("DG_BATCH_QUESTIONS")) batch_questions = std::atoi(b) != 0;
  if (const char* a = std::getenv("DG_ATTN_TC")) attn_tc_ = std::atoi(a) != 0;
  prefix_pool_acquire(device_);  // last: nothing after it can throw
  pool_held_ = true;
}

Engine::~Engine() {
  if (stream_) {
    cudaSetDevice(device_);
    cudaStreamSynchronize(stream_);
    drop_graphs();
    cudaStreamDestroy(stream_);
  }
  if (ev0_) cudaEventDestroy(ev0_);
  if (ev1_) cudaEventDestroy(ev1_);
  for (cudaEvent_t ev : gemm_ev_) cudaEventDestroy(ev);
  if (pool_held_) {
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
    prefix_pool_release(device_);
  }
}

// Timing covers up to 128 projection launches per forward (24 layers use 96).
void Engine::set_gemm_timing(bool on, int first_layer, int layers) {
  DG_CUDA(cudaSetDevice(device_));
  DG_CUDA(cudaStreamSynchronize(stream_));
  gemm_timing = GemmTiming{};
  gemm_ops_pending_.clear();
  gemm_lo_ = std::max(0, first_layer);
  gemm_hi_ = layers >= (1 << 30) - gemm_lo_ ? (1 << 30) : gemm_lo_ + std::max(0, layers);
  drop_graphs();  // captured graphs record into the event pool
  if (on && gemm_ev_.empty()) {
    gemm_ev_.resize(256, nullptr);
    for (auto& ev : gemm_ev_) DG_CUDA(cudaEventCreate(&ev));
  } else if (!on) {
    for (cudaEvent_t ev : gemm_ev_) cudaEventDestroy(ev);
    gemm_ev_.clear();
  }
}

void Engine::collect_gemm_timing() {
  if (!gemm_ev_.empty()) {
    gemm_timing.ops_all += fwd_ops_all_;
    gemm_timing.launches_all += fwd_proj_;
  }
  for (size_t k = 0; k < gemm_ops_pending_.size(); ++k) {
    float ms = 0.0f;
    DG_CUDA(cudaEventElapsedTime(&ms, gemm_ev_[2 * k], gemm_ev_[2 * k + 1]));
    gemm_timing.ms += ms;
    gemm_timing.ops += gemm_ops_pending_[k];
    gemm_timing.launches += 1;
  }
  gemm_ops_pending_.clear();
}

std::map<std::string, Engine::Expected> Engine::expected_names() const {
  std::map<std::string, Expected> e;
  const int64_t H = c_.hidden, I = c_.intermediate, R = c_.rank;
  auto proj = [&](const std::string& key, int64_t in, int64_t out) {
    e[key + ".weight"] = {{out, in}, true};
    if (R > 0) {
      e["base_model.model." + key + ".lora_A.weight"] = {{R, in}, false};
      e["base_model.model." + key + ".lora_B.weight"] = {{out, R}, false};
    }
  };
  for (int i = 0; i < c_.layers; ++i) {
    const std::string p = "layers." + std::to_string(i) + ".";
    if (c_.layer_types[i] == 1) {
      proj(p + "self_attn.q_proj", H, 2LL * c_.qw());
      proj(p + "self_attn.k_proj", H, c_.kw());
      proj(p + "self_attn.v_proj", H, c_.kw());
      proj(p + "self_attn.o_proj", c_.qw(), H);
      e[p + "self_attn.q_norm.weight"] = {{c_.head_dim}, false};
      e[p + "self_attn.k_norm.weight"] = {{c_.head_dim}, false};
    } else {
      const int64_t W = c_.conv_width(), vd = c_.vd(), VH = c_.value_heads;
      proj(p + "linear_attn.in_proj_qkv", H, W);
      proj(p + "linear_attn.in_proj_z", H, vd);
      proj(p + "linear_attn.in_proj_a", H, VH);
      proj(p + "linear_attn.in_proj_b", H, VH);
      proj(p + "linear_attn.out_proj", vd, H);
      e[p + "linear_attn.conv1d.weight"] = {{W, 1, c_.conv_kernel}, false};
      e[p + "linear_attn.dt_bias"] = {{VH}, false};
      e[p + "linear_attn.A_log"] = {{VH}, false};
      e[p + "linear_attn.norm.weight"] = {{c_.dv}, false};
    }
    proj(p + "mlp.gate_proj", H, I);
    proj(p + "mlp.up_proj", H, I);
    proj(p + "mlp.down_proj", I, H);
    e[p + "input_layernorm.weight"] = {{H}, false};
    e[p + "post_attention_layernorm.weight"] = {{H}, false};
  }
  e["embed_tokens.weight"] = {{c_.vocab, H}, false};
  e["norm.weight"] = {{H}, false};
  if (c_.pointer_dim > 0) {
    const int64_t P = c_.pointer_dim;
    e["head.norm.weight"] = {{H}, false};
    e["head.norm.bias"] = {{H}, false};
    e["head.q.weight"] = {{P, H}, false};
    e["head.q.bias"] = {{P}, false};
    e["head.k.weight"] = {{P, H}, false};
    e["head.k.bias"] = {{P}, false};
  }
  return e;
}

static float bf16_to_f32(uint16_t v) {
  uint32_t b = uint32_t(v) << 16;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}
// half(), src/weights.rs:367-382
static float f16_to_f32(uint16_t v) {
  const float sign = (v & 0x8000) ? -1.0f : 1.0f;
  const int e = (v >> 10) & 31, m = v & 1023;
  if (e == 0) return sign * float(m) * std::ldexp(1.0f, -24);
  if (e == 31) return m == 0 ? sign * INFINITY : NAN;
  return sign * (1.0f + float(m) / 1024.0f) * std::ldexp(1.0f, e - 15);
}

void Engine::set_tensor(const std::string& name, int dtype, const std::vector<int64_t>& shape, const void* data) {
  if (finalized_) throw std::runtime_error("engine already finalized");
  size_t n = 1;
  for (auto d : shape) {
    if (d < 0) throw std::runtime_error(name + ": negative dimension");
    n *= size_t(d);
  }
  std::vector<float> f(n);
  if (dtype == 0) {
    std::memcpy(f.data(), data, n * 4);
  } else if (dtype == 1 || dtype == 2) {
    const uint16_t* h = static_cast<const uint16_t*>(data);
    for (size_t i = 0; i < n; ++i) f[i] = dtype == 1 ? bf16_to_f32(h[i]) : f16_to_f32(h[i]);
  } else {
    throw std::runtime_error(name + ": unsupported weight dtype");
  }
  // Data::read rejects non-finite weights (src/weights.rs:170-187).
  for (float v : f)
    if (!std::isfinite(v)) throw std::runtime_error(name + ": non-finite weights");
  stage(name, shape, std::move(f));
}

void Engine::stage(const std::string& name, std::vector<int64_t> shape, std::vector<float>&& f32) {
  auto exp = expected_names();
  auto it = exp.find(name);
  if (it == exp.end()) throw std::runtime_error("unexpected tensor " + name);
  if (it->second.shape != shape) throw std::runtime_error(name + ": unexpected shape");
  if (staged_.count(name)) throw std::runtime_error("duplicate tensor " + name);
  HostTensor t;
  t.shape = shape;
  // read_tensors' quantisation selection, src/weights.rs:346-355; the
  // quantisation itself runs on the device when the projection is built.
  if (it->second.projection && precision_ != kCheckpoint) {
    t.quantized = true;
    t.bits = precision_ == kInt4 ? 4 : 8;
  }
  t.f32 = std::move(f32);
  staged_[name] = std::move(t);
}

// Counter-based N(0, stddev^2) values: splitmix64 hashes, Box-Muller in double.
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void Engine::fill_synthetic(uint64_t seed, float stddev) {
  for (auto& kv : expected_names()) {
    const std::string& name = kv.first;
    if (staged_.count(name)) continue;
    size_t n = 1;
    for (auto d : kv.second.shape) n *= size_t(d);
    std::vector<float> f(n);
    const bool is_norm = name.find("norm.weight") != std::string::npos || name.find("layernorm") != std::string::npos;
    const bool is_bias = name.size() > 5 && name.compare(name.size() - 5, 5, ".bias") == 0;
    if (is_norm || is_bias) {
      std::fill(f.begin(), f.end(), is_norm ? 1.0f : 0.0f);
    } else {
      uint64_t key = seed;
      for (char ch : name) key = mix64(key ^ uint64_t(uint8_t(ch)));
      host_parallel(n, [&](size_t lo, size_t hi) {
        for (size_t i = lo; i < hi; ++i) {
          const uint64_t a = mix64(key ^ (2 * i)), b = mix64(key ^ (2 * i + 1));
          const double u1 = (double((a >> 11) + 1)) * (1.0 / 9007199254740992.0);
          const double u2 = double(b >> 11) * (1.0 / 9007199254740992.0);
          f[i] = float(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2) * stddev);
        }
      });
    }
    stage(name, kv.second.shape, std::move(f));
  }
}

HostTensor Engine::take(const std::string& name) {
  auto it = staged_.find(name);
  if (it == staged_.end()) throw std::runtime_error("missing tensor " + name);
  HostTensor t = std::move(it->second);
  staged_.erase(it);
  return t;
}

DevBuf Engine::upload_f32(const std::vector<float>& v) {
  DevBuf b(v.size() * 4);
  if (!v.empty()) DG_CUDA(cudaMemcpy(b.ptr, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return b;
}

}  // namespace dg
