// extern "C" boundary of libdecider_gpu (declared in include/decider_gpu.h).
#include <cstdlib>
#include <atomic>
#include <cmath>
#include <cstring>
#include <algorithm>
#include <thread>

#include "../../include/decider_gpu.h"
#include "engine.h"

namespace dg {
static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(); }
void note_launch() { g_launches.fetch_add(1); }
bool pdl_enabled() {  // opt-in: measured no faster than plain stream order inside the forward's graph
  static const bool on = [] {
    const char* v = std::getenv("DG_PDL");
    return v && std::atoi(v) != 0;
  }();
  return on;
}
void note_launches(uint64_t n) { g_launches.fetch_add(n); }
}  // namespace dg

struct dg_engine {
  // The engine whose weights this one reads (dg_engine_create_sibling),
  // held so that the weights outlive every engine sharing them; declared
  // first, so it is released after `e`.
  std::shared_ptr<dg::Engine> weights_owner;
  std::shared_ptr<dg::Engine> e;
  // dg_engine_set_lanes: engines sharing e's weights that serve a batch's
  // requests alongside e, each from its own host thread.
  std::vector<std::unique_ptr<dg::Engine>> lanes;
  float last_batch_ms = 0.0f;
};
struct dg_prefix {
  std::unique_ptr<dg::Prefix> p;
  const dg_engine* owner;
};

// The isolated INT8 projection of BASELINE config 1.
struct dg_linear {
  int device = 0, n = 0, k = 0, n_pad = 0, rank = 0;
  float scale = 0.0f;
  bool exact = true;
  cudaStream_t stream = nullptr;
  dg::DevBuf wq, ws_t, lora_a, lora_b, chunk_pid, status;
  dg::WeightMaps maps{};
  int cap_m = 0, ldxs = 0;
  dg::DevBuf x, xq, xs, mid, y, yh;
  // Device time of the last forward (events on `stream`): before the
  // quantiser, before the projection kernel, after it.
  cudaEvent_t ev[3] = {};
  float last_total_ms = 0.0f, last_gemm_ms = 0.0f;
  // dg_linear_test_wait_fault: 0, or the group whose completion the next
  // projections leave out, plus one; and their wait budget (0: 2 s).
  int test_skip_commit = 0;
  unsigned long long test_wait_ns = 0;
};

namespace {
thread_local std::string g_error;

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& ex) {
    g_error = ex.what();
    return 1;
  } catch (...) {
    g_error = "unknown error";
    return 1;
  }
}

dg::Config to_config(const dg_model_config* c) {
  dg::Config k;
  k.hidden = c->hidden_size;
  k.intermediate = c->intermediate_size;
  k.layers = c->num_hidden_layers;
  k.vocab = c->vocab_size;
  k.heads = c->num_attention_heads;
  k.kv_heads = c->num_key_value_heads;
  k.head_dim = c->head_dim;
  k.conv_kernel = c->linear_conv_kernel_dim;
  k.dk = c->linear_key_head_dim;
  k.dv = c->linear_value_head_dim;
  k.key_heads = c->linear_num_key_heads;
  k.value_heads = c->linear_num_value_heads;
  k.eps = c->rms_norm_eps;
  k.rope_theta = c->rope_theta;
  k.partial_rotary = c->partial_rotary_factor;
  if (c->num_hidden_layers > 0 && !c->layer_types) throw std::runtime_error("layer_types is required");
  k.layer_types.assign(c->layer_types, c->layer_types + std::max(0, c->num_hidden_layers));
  k.rank = c->lora_rank;
  k.lora_scale = c->lora_scale;
  k.pointer_dim = c->pointer_dim;
  return k;
}

void check_engine(const dg_engine* e) {
  if (!e || !e->e) throw std::runtime_error("null engine");
}

void linear_reserve(dg_linear* l, int m) {
  if (m <= l->cap_m) return;
  const int cap = (m + 127) / 128 * 128;
  l->ldxs = cap;
  l->x = dg::DevBuf(size_t(cap) * l->k * 4);
  l->xq = dg::DevBuf(size_t(cap) * l->k);
  l->xs = dg::DevBuf(size_t(l->k / 64) * cap * 4);
  DG_CUDA(cudaMemset(l->xs.ptr, 0, l->xs.bytes));
  l->mid = dg::DevBuf(size_t(cap) * 32 * 4);
  l->y = dg::DevBuf(size_t(cap) * l->n_pad * 4);
  l->yh = dg::DevBuf(size_t(cap) * l->n * 4);
  l->cap_m = cap;
}

void linear_run(dg_linear* l, const float* x_dev, int m, float* y_dev, int32_t* dots) {
  using namespace dg;
  if (m <= 0) throw std::runtime_error("dg_linear: need at least one row");
  DG_CUDA(cudaSetDevice(l->device));
  linear_reserve(l, m);
  DG_CUDA(cudaMemsetAsync(l->status.ptr, 0, sizeof(DeviceStatus), l->stream));
  DeviceStatus* st = l->status.as<DeviceStatus>();
  DG_CUDA(cudaEventRecord(l->ev[0], l->stream));
  launch_norm_quant(x_dev, l->k, m, l->k, nullptr, 0.0f, nullptr, 0, l->xq.as<int8_t>(), l->xs.as<float>(), l->ldxs, st,
                    l->stream);
  if (l->rank) {
    launch_lora_a(x_dev, l->k, m, l->k, l->lora_a.as<float>(), l->rank, l->mid.as<float>(), 32, l->exact, l->stream);
  }
  CUtensorMap map_a;
  make_tmap_i8_2d(&map_a, l->xq.ptr, uint64_t(l->k), uint64_t(m), 128, 128);
  GemmArgs a{};
  a.M = m;
  a.N = l->n_pad;
  a.K = l->k;
  a.xs = l->xs.as<float>();
  a.ldxs = l->ldxs;
  a.ws = l->ws_t.as<float>();
  a.lora_mid = l->mid.as<float>();
  a.ld_mid = 32;
  a.lora_b = l->lora_b.as<float>();
  a.chunk_pid = l->chunk_pid.as<int>();
  a.lora_scale = l->scale;
  const bool direct = l->n_pad == l->n && dots == nullptr;
  a.out = direct ? y_dev : l->y.as<float>();
  a.ldo = direct ? l->n : l->n_pad;
  a.status = st;
  int32_t* dump = nullptr;
  if (dots) {
    if (l->n_pad != l->n) throw std::runtime_error("dg_linear: group-dot dump needs n % 256 == 0");
    dump = dots;
  }
  a.dots = dump;
  a.test_skip_commit = l->test_skip_commit;
  a.wait_ns = l->test_wait_ns;
  DG_CUDA(cudaEventRecord(l->ev[1], l->stream));
  launch_gemm_i8(map_a, l->maps, a, l->rank, kEpiWrite, l->exact, l->stream);
  DG_CUDA(cudaEventRecord(l->ev[2], l->stream));
  if (!direct)
    DG_CUDA(cudaMemcpy2DAsync(y_dev, size_t(l->n) * 4, l->y.ptr, size_t(l->n_pad) * 4, size_t(l->n) * 4, m,
                              cudaMemcpyDeviceToDevice, l->stream));
  DeviceStatus h{};
  DG_CUDA(cudaMemcpyAsync(&h, l->status.ptr, sizeof(h), cudaMemcpyDeviceToHost, l->stream));
  DG_CUDA(cudaStreamSynchronize(l->stream));
  DG_CUDA(cudaEventElapsedTime(&l->last_total_ms, l->ev[0], l->ev[2]));
  DG_CUDA(cudaEventElapsedTime(&l->last_gemm_ms, l->ev[1], l->ev[2]));
  if (h.code == kNonFinite) throw std::runtime_error("non-finite projection input");
  if (h.code == kWaitTimeout)
    throw std::runtime_error("device pipeline wait timed out (device error code " + std::to_string(h.code) +
                             " at location " + std::to_string(h.where) + ")");
  if (h.code) throw std::runtime_error("device error code " + std::to_string(h.code) + " at " + std::to_string(h.where));
}
}  // namespace

extern "C" {

const char* dg_last_error(void) { return g_error.c_str(); }
uint64_t dg_launch_count(void) { return dg::launch_count(); }

int dg_engine_create(const dg_model_config* cfg, int precision, int device, int max_tokens, dg_engine** out) {
  return guarded([&] {
    if (!cfg || !out) throw std::runtime_error("null argument");
    auto* e = new dg_engine();
    try {
      e->e.reset(new dg::Engine(to_config(cfg), precision, device, max_tokens));
    } catch (...) {
      delete e;
      throw;
    }
    *out = e;
  });
}

int dg_engine_create_sibling(dg_engine* base, dg_engine** out) {
  return guarded([&] {
    check_engine(base);
    if (!out) throw std::runtime_error("null argument");
    std::unique_ptr<dg_engine> e(new dg_engine());
    {
      std::lock_guard<std::mutex> lk(base->e->mu);
      const dg::Engine& b = *base->e;
      e->e = std::make_shared<dg::Engine>(b.config(), b.precision(), b.device(), b.max_tokens());
      e->e->share_weights(b);
      e->e->exact = b.exact;  // the base's arithmetic mode
      e->e->batch_questions = b.batch_questions;
    }
    e->weights_owner = base->weights_owner ? base->weights_owner : base->e;
    *out = e.release();
  });
}

int dg_engine_set_tensor(dg_engine* e, const char* name, int dtype, const int64_t* shape, int ndim, const void* data) {
  return guarded([&] {
    check_engine(e);
    if (!name || (ndim > 0 && !shape) || ndim < 0 || ndim > 8) throw std::runtime_error("bad tensor arguments");
    std::vector<int64_t> s(shape, shape + ndim);
    size_t n = 1;
    for (auto d : s) n *= size_t(d < 0 ? 0 : d);
    if (n && !data) throw std::runtime_error("null tensor data");
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->set_tensor(name, dtype, s, data);
  });
}

int dg_engine_fill_synthetic(dg_engine* e, uint64_t seed, float stddev) {
  return guarded([&] {
    check_engine(e);
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->fill_synthetic(seed, stddev);
  });
}

int dg_engine_finalize(dg_engine* e) {
  return guarded([&] {
    check_engine(e);
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->finalize();
  });
}

int dg_read_checkpoint_config(const char* dir, dg_model_config* cfg, int32_t* layer_types, int max_layers) {
  return guarded([&] {
    if (!dir || !cfg || (max_layers > 0 && !layer_types)) throw std::runtime_error("null argument");
    dg::Config c;
    int pointer_dim = 0;
    dg::read_checkpoint_config(dir, c, pointer_dim);
    if (int(c.layer_types.size()) > max_layers) throw std::runtime_error("layer_types buffer too small");
    std::copy(c.layer_types.begin(), c.layer_types.end(), layer_types);
    cfg->hidden_size = c.hidden;
    cfg->intermediate_size = c.intermediate;
    cfg->num_hidden_layers = c.layers;
    cfg->vocab_size = c.vocab;
    cfg->num_attention_heads = c.heads;
    cfg->num_key_value_heads = c.kv_heads;
    cfg->head_dim = c.head_dim;
    cfg->linear_conv_kernel_dim = c.conv_kernel;
    cfg->linear_key_head_dim = c.dk;
    cfg->linear_value_head_dim = c.dv;
    cfg->linear_num_key_heads = c.key_heads;
    cfg->linear_num_value_heads = c.value_heads;
    cfg->rms_norm_eps = c.eps;
    cfg->rope_theta = c.rope_theta;
    cfg->partial_rotary_factor = c.partial_rotary;
    cfg->layer_types = layer_types;
    cfg->lora_rank = c.rank;
    cfg->lora_scale = c.lora_scale;
    cfg->pointer_dim = pointer_dim;
  });
}

void dg_load_limits_default(dg_load_limits* out) {
  if (!out) return;
  const dg::LoadLimits d;
  out->max_tensor_bytes = d.max_tensor_bytes;
  out->max_weight_bytes = d.max_weight_bytes;
  out->max_workspace_bytes = d.max_workspace_bytes;
}

int dg_engine_load_with_limits(const char* dir, int precision, const dg_load_limits* limits, int device,
                               int max_tokens, dg_engine** out) {
  return guarded([&] {
    if (!dir || !out) throw std::runtime_error("null argument");
    dg::LoadLimits lim;
    if (limits) {
      lim.max_tensor_bytes = limits->max_tensor_bytes;
      lim.max_weight_bytes = limits->max_weight_bytes;
      lim.max_workspace_bytes = limits->max_workspace_bytes;
    }
    dg::Config c;
    int pointer_dim = 0, max_length = 0;
    dg::read_checkpoint_config(dir, c, pointer_dim, &max_length);
    // Every budget is checked before the engine takes any device memory.
    dg::validate_layout(c, max_length, c.rank, pointer_dim, lim);
    dg::ensure_checkpoint_budget(dir, lim);
    std::unique_ptr<dg_engine> e(new dg_engine());
    e->e.reset(new dg::Engine(c, precision, device, max_tokens));
    dg::load_checkpoint_tensors(*e->e, dir, lim);
    e->e->finalize();
    *out = e.release();
  });
}

int dg_engine_load(const char* dir, int precision, int device, int max_tokens, dg_engine** out) {
  return dg_engine_load_with_limits(dir, precision, nullptr, device, max_tokens, out);
}

int dg_engine_fast_path(const dg_engine* e) { return e && e->e && e->e->fast_path() ? 1 : 0; }

int dg_engine_set_exact(dg_engine* e, int exact) {
  return guarded([&] {
    check_engine(e);
    e->e->exact = exact != 0;
    for (auto& l : e->lanes) l->exact = exact != 0;
  });
}

int dg_engine_set_lanes(dg_engine* e, int lanes) {
  return guarded([&] {
    check_engine(e);
    if (lanes < 1 || lanes > 8) throw std::runtime_error("lanes must be 1 to 8");
    std::lock_guard<std::mutex> lk(e->e->mu);
    const dg::Engine& b = *e->e;
    while (int(e->lanes.size()) > lanes - 1) e->lanes.pop_back();
    while (int(e->lanes.size()) < lanes - 1) {
      std::unique_ptr<dg::Engine> l(new dg::Engine(b.config(), b.precision(), b.device(), b.max_tokens()));
      l->share_weights(b);
      l->exact = b.exact;
      l->batch_questions = b.batch_questions;
      e->lanes.push_back(std::move(l));
    }
    e->e->wide_scan = lanes > 1;
    for (auto& l : e->lanes) l->wide_scan = lanes > 1;
  });
}

int dg_engine_lanes(const dg_engine* e) { return e && e->e ? 1 + int(e->lanes.size()) : 0; }

float dg_engine_last_batch_ms(const dg_engine* e) { return e && e->e ? e->last_batch_ms : -1.0f; }

void dg_engine_free(dg_engine* e) { delete e; }

void* dg_engine_stream(const dg_engine* e) { return e && e->e ? static_cast<void*>(e->e->stream()) : nullptr; }

float dg_engine_last_forward_ms(const dg_engine* e) { return e && e->e ? e->e->last_forward_ms : -1.0f; }

int dg_engine_last_launches(const dg_engine* e) { return e && e->e ? e->e->last_launches : -1; }

int dg_engine_gemm_timing(dg_engine* e, int enable) {
  return guarded([&] {
    check_engine(e);
    e->e->set_gemm_timing(enable != 0);
  });
}

int dg_engine_gemm_timing_layers(dg_engine* e, int first_layer, int layers) {
  return guarded([&] {
    check_engine(e);
    if (first_layer < 0 || layers < 0) throw std::runtime_error("layer range must be non-negative");
    e->e->set_gemm_timing(true, first_layer, layers);
  });
}

int dg_engine_gemm_time_all(const dg_engine* e, double* ops_all, uint64_t* launches_all) {
  return guarded([&] {
    check_engine(e);
    if (!ops_all || !launches_all) throw std::runtime_error("null argument");
    *ops_all = e->e->gemm_timing.ops_all;
    *launches_all = e->e->gemm_timing.launches_all;
  });
}

int dg_engine_gemm_time(const dg_engine* e, double* ms, double* ops, uint64_t* launches) {
  return guarded([&] {
    check_engine(e);
    if (!ms || !ops || !launches) throw std::runtime_error("null argument");
    *ms = e->e->gemm_timing.ms;
    *ops = e->e->gemm_timing.ops;
    *launches = e->e->gemm_timing.launches;
  });
}

int dg_forward_hidden(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t n, float* hidden_out) {
  return guarded([&] {
    check_engine(e);
    if (past && past->owner != e) throw std::runtime_error("prefix belongs to another engine");
    if (n && !ids) throw std::runtime_error("null ids");
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->forward(ids, int(std::min<size_t>(n, 1u << 30)), past ? past->p.get() : nullptr, false, hidden_out, nullptr);
  });
}

int dg_prefill(dg_engine* e, const uint32_t* ids, size_t n, dg_prefix** out) {
  return guarded([&] {
    check_engine(e);
    if (!out || (n && !ids)) throw std::runtime_error("null argument");
    std::lock_guard<std::mutex> lk(e->e->mu);
    std::unique_ptr<dg::Prefix> p;
    e->e->forward(ids, int(std::min<size_t>(n, 1u << 30)), nullptr, true, nullptr, &p);
    auto* h = new dg_prefix();
    h->p = std::move(p);
    h->owner = e;
    *out = h;
  });
}

size_t dg_prefix_len(const dg_prefix* p) { return p && p->p ? size_t(p->p->len) : 0; }
void dg_prefix_free(dg_prefix* p) { delete p; }

int dg_logits(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t n, const size_t* opt_pos, size_t n_opt,
              float* logits_out) {
  return guarded([&] {
    check_engine(e);
    if (past && past->owner != e) throw std::runtime_error("prefix belongs to another engine");
    if (!ids || !opt_pos || !logits_out || n == 0 || n_opt == 0)
      throw std::runtime_error("invalid encoding positions or window");
    for (size_t i = 0; i < n_opt; ++i)
      if (opt_pos[i] + 1 >= n) throw std::runtime_error("invalid encoding positions or window");
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->forward(ids, int(std::min<size_t>(n, 1u << 30)), past ? past->p.get() : nullptr, false, nullptr, nullptr);
    e->e->head_logits(int(n), opt_pos, int(n_opt), logits_out);
  });
}

int dg_debug_layer(dg_engine* e, int layer, const float* x_in, size_t n, float* x_out) {
  return guarded([&] {
    check_engine(e);
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->debug_layer(layer, x_in, int(std::min<size_t>(n, 1u << 30)), x_out);
  });
}

int dg_measure_i8_peak(int device, int iters, double* tops_out, float* ms_out) {
  return guarded([&] {
    if (!tops_out) throw std::runtime_error("null argument");
    *tops_out = dg::measure_i8_peak(device, iters, ms_out);
  });
}

int dg_debug_layer_codes(dg_engine* e, int layer, const float* x_in, size_t n, float* x_out, int8_t* codes_out) {
  return guarded([&] {
    check_engine(e);
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->debug_layer_codes(layer, x_in, int(std::min<size_t>(n, 1u << 30)), x_out, codes_out);
  });
}

size_t dg_attention_workspace_bytes(int heads, int kv_heads, int d, int n) {
  if (!dg::attention_tc_supported(d, heads, kv_heads) || n <= 0) return 0;
  return dg::attention_tc_workspace_floats(heads, kv_heads, d, n) * 4;
}

int dg_attention_device(const float* q, const float* kc, const float* vc, const float* gate, int ld_gate, int n,
                        int offset, int heads, int kv_heads, int d, float* out, int tensor_cores, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return guarded([&] {
    if (!q || !kc || !vc || !gate || !out) throw std::runtime_error("null argument");
    if (n <= 0 || offset < 0 || offset + n > 4096 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || d <= 0)
      throw std::runtime_error("attention: bad shape");
    auto s = static_cast<cudaStream_t>(stream);
    static thread_local dg::DevBuf status;
    if (!status.ptr) {
      status = dg::DevBuf(sizeof(dg::DeviceStatus));
    }
    DG_CUDA(cudaMemsetAsync(status.ptr, 0, sizeof(dg::DeviceStatus), s));
    if (tensor_cores) {
      if (!workspace || workspace_bytes < dg_attention_workspace_bytes(heads, kv_heads, d, n))
        throw std::runtime_error("attention: workspace too small");
      dg::launch_attention_tc(q, kc, vc, gate, ld_gate, n, offset, heads, kv_heads, d, out,
                              static_cast<float*>(workspace), workspace_bytes / 4, status.as<dg::DeviceStatus>(), s);
    } else {
      dg::launch_attention(q, kc, vc, gate, ld_gate, n, offset, heads, kv_heads, d, out, true, s);
    }
    dg::DeviceStatus h{};
    DG_CUDA(cudaMemcpyAsync(&h, status.ptr, sizeof(h), cudaMemcpyDeviceToHost, s));
    DG_CUDA(cudaStreamSynchronize(s));
    if (h.code) throw std::runtime_error("attention: device error code " + std::to_string(h.code));
  });
}

int dg_quantize_weights_device(const float* w, size_t rows, size_t width, int bits, uint8_t* values, float* scales,
                               void* stream) {
  return guarded([&] {
    if (!w || !values || !scales) throw std::runtime_error("null argument");
    auto s = static_cast<cudaStream_t>(stream);
    dg::quantize_weights_device(w, rows, width, bits, values, scales, nullptr, s);
    DG_CUDA(cudaStreamSynchronize(s));
  });
}

int dg_forward_segments_hidden(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t seg_len, size_t segs,
                               float* hidden_out) {
  return guarded([&] {
    check_engine(e);
    if (past && past->owner != e) throw std::runtime_error("prefix belongs to another engine");
    if (!ids || seg_len == 0 || segs == 0 || seg_len * segs > (1u << 30))
      throw std::runtime_error("token sequence must contain 1\xe2\x80\x93" "4096 tokens");
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->forward_segments(ids, int(seg_len), int(segs), past ? past->p.get() : nullptr, hidden_out);
  });
}

}  // extern "C"

namespace {

// One request of dg_logits_batch on engine g (NativeEngine::evaluate,
// src/lib.rs:477-559): the state prefilled once, then its questions, the
// logits written from `logits_out` on. Returns the status; the device time
// of its forwards goes to ms.
int run_request(const dg_engine* e, dg::Engine& g, const dg_request& q, float* logits_out, float& ms) {
  return guarded([&] {
    if (!q.questions || q.n_questions == 0) throw std::runtime_error("request has no questions");
    if (q.past && q.past->owner != e) throw std::runtime_error("prefix belongs to another engine");
    if (q.past && q.n_state) throw std::runtime_error("a request continues either a prefix or its own state ids");
    if (q.n_state && !q.state_ids) throw std::runtime_error("null state ids");
    for (size_t i = 0; i < q.n_questions; ++i) {
      const dg_question& u = q.questions[i];
      if (!u.ids || !u.opt_pos || u.n == 0 || u.n_opt == 0)
        throw std::runtime_error("invalid encoding positions or window");
      for (size_t j = 0; j < u.n_opt; ++j)
        if (u.opt_pos[j] + 1 >= u.n) throw std::runtime_error("invalid encoding positions or window");
    }
    std::lock_guard<std::mutex> lk(g.mu);
    std::unique_ptr<dg::Prefix> state;
    const dg::Prefix* past = q.past ? q.past->p.get() : nullptr;
    if (q.n_state) {
      g.forward(q.state_ids, int(std::min<size_t>(q.n_state, 1u << 30)), nullptr, true, nullptr, &state);
      ms += g.last_forward_ms;
      past = state.get();
    }
    size_t o = 0;
    // Questions of one length continue the state together: one segmented
    // forward per group of as many as the workspace holds, each question's
    // rows the same as its own forward's (bit for bit in reference order).
    const size_t nq = q.n_questions, len0 = q.questions[0].n;
    bool together = nq >= 2 && g.batch_questions && g.segments_supported() && len0 <= size_t(g.max_tokens());
    for (size_t i = 1; together && i < nq; ++i) together = q.questions[i].n == len0;
    if (together) {
      const size_t per = std::min(nq, std::max<size_t>(1, size_t(g.max_tokens()) / len0));
      std::vector<uint32_t> ids;
      for (size_t i0 = 0; i0 < nq; i0 += per) {
        const size_t cnt = std::min(per, nq - i0);
        ids.clear();
        for (size_t i = i0; i < i0 + cnt; ++i) ids.insert(ids.end(), q.questions[i].ids, q.questions[i].ids + len0);
        g.forward_segments(ids.data(), int(len0), int(cnt), past, nullptr);
        ms += g.last_forward_ms;
        for (size_t j = 0; j < cnt; ++j) {
          const dg_question& u = q.questions[i0 + j];
          g.head_logits(int(len0), u.opt_pos, int(u.n_opt), logits_out + o, int(j * len0));
          o += u.n_opt;
        }
      }
    } else {
      for (size_t i = 0; i < nq; ++i) {
        const dg_question& u = q.questions[i];
        g.forward(u.ids, int(std::min<size_t>(u.n, 1u << 30)), past, false, nullptr, nullptr);
        ms += g.last_forward_ms;
        g.head_logits(int(u.n), u.opt_pos, int(u.n_opt), logits_out + o);
        o += u.n_opt;
      }
    }
  });
}

// Cost of a request in token-equivalents, as the request sharding across
// GPUs weighs it: computed tokens, the attention term of the longest
// window, and a fixed cost per forward pass.
double request_cost(const dg_request& q) {
  double tokens = double(q.n_state), window = 0.0, forwards = q.n_state ? 1.0 : 0.0;
  for (size_t i = 0; q.questions && i < q.n_questions; ++i) {
    tokens += double(q.questions[i].n);
    window = std::max(window, double(q.n_state + q.questions[i].n));
    forwards += 1.0;
  }
  return tokens + window * window / 4096.0 + 300.0 * forwards;
}

}  // namespace

extern "C" {

int dg_logits_batch(dg_engine* e, const dg_request* requests, size_t n_requests, float* logits_out, int* status_out,
                    float* request_ms) {
  const int rc = guarded([&] {
    check_engine(e);
    if (n_requests && (!requests || !logits_out)) throw std::runtime_error("null argument");
  });
  if (rc) return rc;
  // Where each request's logits start (request order).
  std::vector<size_t> off(n_requests + 1, 0);
  for (size_t r = 0; r < n_requests; ++r) {
    size_t n_logits = 0;
    const dg_request& q = requests[r];
    for (size_t i = 0; q.questions && i < q.n_questions; ++i) n_logits += q.questions[i].n_opt;
    off[r + 1] = off[r] + n_logits;
  }
  // Requests over the lanes, longest processing time first (a request that
  // continues a prefix stays on the engine that made it); each lane runs
  // its share in request order.
  const size_t lanes = 1 + e->lanes.size();
  std::vector<std::vector<size_t>> plan(lanes);
  {
    std::vector<size_t> order(n_requests);
    for (size_t r = 0; r < n_requests; ++r) order[r] = r;
    std::vector<double> cost(n_requests);
    for (size_t r = 0; r < n_requests; ++r) cost[r] = request_cost(requests[r]);
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return cost[a] > cost[b]; });
    std::vector<double> load(lanes, 0.0);
    for (size_t r : order) {
      size_t best = 0;
      if (!requests[r].past)
        for (size_t k = 1; k < lanes; ++k)
          if (load[k] < load[best]) best = k;
      plan[best].push_back(r);
      load[best] += cost[r];
    }
    for (auto& p : plan) std::sort(p.begin(), p.end());
  }
  std::vector<int> status(n_requests, 0);
  std::vector<float> ms(n_requests, 0.0f);
  std::vector<std::string> errors(n_requests);
  // The batch's device span: every lane's stream waits for an event of the
  // engine's stream recorded before the first request; each lane records
  // its end after its last request.
  dg::Engine& g0 = *e->e;
  std::vector<cudaEvent_t> ev(lanes + 1, nullptr);
  // The events belong to the engine's device (the calling thread may have
  // another one current).
  bool timed = cudaSetDevice(g0.device()) == cudaSuccess;
  for (auto& x : ev) timed = timed && cudaEventCreate(&x) == cudaSuccess;
  if (timed) timed = cudaEventRecord(ev[0], g0.stream()) == cudaSuccess;
  if (!timed) cudaGetLastError();  // a failed timing call must not fail the first launch
  auto run_lane = [&](size_t k) {
    dg::Engine& g = k == 0 ? g0 : *e->lanes[k - 1];
    cudaSetDevice(g.device());
    if (timed && cudaStreamWaitEvent(g.stream(), ev[0], 0) != cudaSuccess) cudaGetLastError();
    for (size_t r : plan[k]) {
      float t = 0.0f;
      status[r] = run_request(e, g, requests[r], logits_out + off[r], t);
      ms[r] = t;
      if (status[r]) errors[r] = dg_last_error();
    }
    if (timed && cudaEventRecord(ev[k + 1], g.stream()) != cudaSuccess) cudaGetLastError();
  };
  std::vector<std::thread> threads;
  std::vector<size_t> inline_lanes;  // lanes whose thread could not be started run here
  for (size_t k = 1; k < lanes; ++k) {
    if (plan[k].empty()) continue;
    try {
      threads.emplace_back(run_lane, k);
    } catch (...) {
      inline_lanes.push_back(k);
    }
  }
  run_lane(0);
  for (size_t k : inline_lanes) run_lane(k);
  for (auto& t : threads) t.join();
  float span = 0.0f;
  for (size_t k = 0; timed && k < lanes; ++k) {
    if (k > 0 && plan[k].empty()) continue;
    float t = 0.0f;
    if (cudaEventSynchronize(ev[k + 1]) == cudaSuccess && cudaEventElapsedTime(&t, ev[0], ev[k + 1]) == cudaSuccess)
      span = std::max(span, t);
  }
  for (auto& x : ev)
    if (x) cudaEventDestroy(x);
  cudaGetLastError();  // the timing calls' own failures are not the batch's
  e->last_batch_ms = span;
  std::string first_error;
  for (size_t r = 0; r < n_requests; ++r) {
    if (status_out) status_out[r] = status[r];
    if (request_ms) request_ms[r] = ms[r];
    if (status[r] && first_error.empty()) first_error = errors[r];
  }
  if (first_error.empty()) return 0;
  g_error = first_error;
  return 1;
}

int dg_linear_create(const float* w, int n, int k, const float* lora_a, const float* lora_b, int rank, float lora_scale,
                     int device, dg_linear** out) {
  return guarded([&] {
    using namespace dg;
    if (!w || !out || n <= 0 || k <= 0) throw std::runtime_error("bad dg_linear arguments");
    if (k % 128) throw std::runtime_error("dg_linear: k must be a multiple of 128");
    if (rank != 0 && rank != 32) throw std::runtime_error("dg_linear: LoRA rank must be 0 or 32");
    if (rank && (!lora_a || !lora_b)) throw std::runtime_error("dg_linear: LoRA weights missing");
    DG_CUDA(cudaSetDevice(device));
    std::unique_ptr<dg_linear> l(new dg_linear());
    l->device = device;
    l->n = n;
    l->k = k;
    l->rank = rank;
    l->scale = lora_scale;
    l->n_pad = (n + 255) / 256 * 256;
    const int G = k / 64, N = l->n_pad;
    auto up = [](const void* src, size_t bytes) {
      DevBuf b(bytes);
      DG_CUDA(cudaMemcpy(b.ptr, src, bytes, cudaMemcpyHostToDevice));
      return b;
    };
    // Data::quantize on the device into the kernel's layout: rows padded
    // to N with zero weights and unit scales, scales transposed to [G][N].
    l->wq = DevBuf(size_t(N) * k);
    DG_CUDA(cudaMemset(l->wq.ptr, 0, l->wq.bytes));
    std::vector<float> ones(size_t(G) * N, 1.0f);
    l->ws_t = up(ones.data(), ones.size() * 4);
    {
      DevBuf wf = up(w, size_t(n) * k * 4);
      QuantLayout L = quant_plain_layout(size_t(n), size_t(k));
      L.s_row = 1;
      L.s_group = size_t(N);
      quantize_weights_device(wf.as<float>(), size_t(n), size_t(k), 8, l->wq.as<uint8_t>(), l->ws_t.as<float>(), &L,
                              0);
      DG_CUDA(cudaStreamSynchronize(0));
    }
    std::vector<int> pid(N / 16, 0);
    l->chunk_pid = up(pid.data(), pid.size() * 4);
    if (rank) {
      std::vector<float> lb(size_t(N) * rank, 0.0f);
      std::memcpy(lb.data(), lora_b, size_t(n) * rank * 4);
      l->lora_b = up(lb.data(), lb.size() * 4);
      l->lora_a = up(lora_a, size_t(rank) * k * 4);
    }
    l->status = DevBuf(sizeof(DeviceStatus));
    make_weight_maps(&l->maps, l->wq.ptr, k, N, rank ? l->lora_b.as<float>() : nullptr, rank);
    DG_CUDA(cudaStreamCreateWithFlags(&l->stream, cudaStreamNonBlocking));
    for (auto& ev : l->ev) DG_CUDA(cudaEventCreate(&ev));
    *out = l.release();
  });
}

int dg_linear_forward(dg_linear* l, const float* x, int m, float* y) {
  return guarded([&] {
    if (!l || !x || !y) throw std::runtime_error("null argument");
    DG_CUDA(cudaSetDevice(l->device));
    linear_reserve(l, m);
    DG_CUDA(cudaMemcpyAsync(l->x.ptr, x, size_t(m) * l->k * 4, cudaMemcpyHostToDevice, l->stream));
    linear_run(l, l->x.as<float>(), m, l->yh.as<float>(), nullptr);
    DG_CUDA(cudaMemcpyAsync(y, l->yh.ptr, size_t(m) * l->n * 4, cudaMemcpyDeviceToHost, l->stream));
    DG_CUDA(cudaStreamSynchronize(l->stream));
  });
}

int dg_linear_forward_device(dg_linear* l, const float* x_device, int m, float* y_device, int32_t* group_dots_device) {
  return guarded([&] {
    if (!l || !x_device || !y_device) throw std::runtime_error("null argument");
    linear_run(l, x_device, m, y_device, group_dots_device);
  });
}

int dg_linear_last_quantized(dg_linear* l, int m, int8_t* xq, float* xs) {
  return guarded([&] {
    if (!l || m <= 0 || m > l->cap_m) throw std::runtime_error("no quantized rows of that size");
    DG_CUDA(cudaSetDevice(l->device));
    DG_CUDA(cudaMemcpy(xq, l->xq.ptr, size_t(m) * l->k, cudaMemcpyDeviceToHost));
    for (int g = 0; g < l->k / 64; ++g)
      DG_CUDA(cudaMemcpy(xs + size_t(g) * m, l->xs.as<float>() + size_t(g) * l->ldxs, size_t(m) * 4,
                         cudaMemcpyDeviceToHost));
  });
}

void* dg_linear_stream(const dg_linear* l) { return l ? static_cast<void*>(l->stream) : nullptr; }

int dg_linear_last_times(const dg_linear* l, float* total_ms, float* gemm_ms) {
  return guarded([&] {
    if (!l) throw std::runtime_error("null argument");
    if (total_ms) *total_ms = l->last_total_ms;
    if (gemm_ms) *gemm_ms = l->last_gemm_ms;
  });
}

int dg_linear_test_wait_fault(dg_linear* l, int skip_group, uint64_t wait_ns) {
  return guarded([&] {
    if (!l) throw std::runtime_error("null argument");
    if (skip_group >= 0 && (l->k / 64 <= skip_group || wait_ns == 0 || wait_ns > 1000000000ull))
      throw std::runtime_error("dg_linear_test_wait_fault: group out of range or wait budget not in (0, 1 s]");
    l->test_skip_commit = skip_group >= 0 ? skip_group + 1 : 0;
    l->test_wait_ns = skip_group >= 0 ? wait_ns : 0;
  });
}

int dg_linear_set_exact(dg_linear* l, int exact) {
  return guarded([&] {
    if (!l) throw std::runtime_error("null argument");
    l->exact = exact != 0;
  });
}

void dg_linear_free(dg_linear* l) {
  if (!l) return;
  cudaSetDevice(l->device);
  if (l->stream) {
    cudaStreamSynchronize(l->stream);
    cudaStreamDestroy(l->stream);
  }
  for (auto& ev : l->ev)
    if (ev) cudaEventDestroy(ev);
  delete l;
}

static dg::DeltaArgs delta_args(const float* q, const float* k, const float* v, const float* g, const float* beta,
                                int batch, int t, int heads, float* state, float* o) {
  if (!q || !k || !v || !g || !beta || !state || !o) throw std::runtime_error("null argument");
  if (batch <= 0 || t <= 0 || heads <= 0) throw std::runtime_error("bad gated delta rule shape");
  dg::DeltaArgs a{};
  const size_t row = size_t(heads) * 128;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ld_qk = a.ld_v = int(row);
  a.bs_qkv = size_t(t) * row;
  a.decay = g;
  a.beta = beta;
  a.log_decay = 1;
  a.ld_gb = heads;
  a.bs_gb = size_t(t) * heads;
  a.n = t;
  a.key_heads = a.value_heads = heads;
  a.dv = 128;
  a.state = state;
  a.bs_state = size_t(heads) * 128 * 128;
  a.o = o;
  a.ldo = int(row);
  a.bs_o = size_t(t) * row;
  return a;
}

int dg_gated_delta_rule_device(const float* q, const float* k, const float* v, const float* g, const float* beta,
                               int batch, int t, int heads, float* state, float* o, void* stream) {
  return guarded([&] {
    dg::DeltaArgs a = delta_args(q, k, v, g, beta, batch, t, heads, state, o);
    dg::launch_delta_rec128(a, batch, static_cast<cudaStream_t>(stream));
  });
}

size_t dg_gated_delta_chunk_workspace_bytes(int batch, int t, int heads) {
  if (batch <= 0 || t <= 0 || heads <= 0) return 0;
  return dg::delta_chunk_workspace_bytes(batch, heads, t);
}

int dg_gated_delta_rule_chunked_device(const float* q, const float* k, const float* v, const float* g,
                                       const float* beta, int batch, int t, int heads, float* state, float* o,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  return guarded([&] {
    dg::DeltaArgs a = delta_args(q, k, v, g, beta, batch, t, heads, state, o);
    if (!workspace) throw std::runtime_error("null workspace");
    dg::launch_delta_chunked(a, batch, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"

// ---- Allocation-free projection call (no counterpart in the reference).
// Some hosts cannot allocate device memory while serving a request: services
// that reserve their whole device-memory budget at start-up (an allocation in
// mid-request can fail under memory pressure), and latency-bound callers for
// which cudaMalloc/cudaFree are too costly (cudaFree waits for the device).
// dg_linear_forward_device_noalloc runs the same kernels as
// dg_linear_forward_device, but its per-call scratch (quantised rows, their
// group scales, the LoRA-A rows, a padded output and the status word) lives
// in one fixed area of static device memory per device instead of buffers the
// handle grows with cudaMalloc. Calls on one device share that area, so they
// must not overlap in time (from several threads, or several handles).
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_base[kNoAllocMaxDevices] = {};

// Address of this device's scratch area; resolved once per device, with that
// device current, on the first call that needs it.
unsigned char* noalloc_scratch(int device) {
  if (device < 0 || device >= kNoAllocMaxDevices) throw std::runtime_error("dg_linear: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_base[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      throw std::runtime_error(std::string("dg_linear_forward_device_noalloc: cannot resolve its scratch area: ") +
                               cudaGetErrorString(e));
    g_noalloc_base[device] = p;
  }
  return static_cast<unsigned char*>(g_noalloc_base[device]);
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

extern "C" {

int dg_linear_forward_device_noalloc(dg_linear* l, const float* x_device, int m, float* y_device) {
  return guarded([&] {
    using namespace dg;
    if (!l || !x_device || !y_device) throw std::runtime_error("null argument");
    if (m <= 0) throw std::runtime_error("dg_linear: need at least one row");
    // Scratch layout: status | xs [k/64][ldxs] | xq [m][k] | mid [m][32] | y [m][n_pad]
    const int ldxs = (m + 127) / 128 * 128;
    const bool direct = l->n_pad == l->n;
    const size_t st_off = 0;
    const size_t xs_off = st_off + align256(sizeof(DeviceStatus));
    const size_t xs_bytes = size_t(l->k / 64) * ldxs * 4;
    const size_t xq_off = xs_off + align256(xs_bytes);
    const size_t mid_off = xq_off + align256(size_t(m) * l->k);
    const size_t y_off = mid_off + align256(l->rank ? size_t(m) * 32 * 4 : 0);
    const size_t total = y_off + (direct ? 0 : size_t(m) * l->n_pad * 4);
    if (total > kNoAllocScratchBytes)
      throw std::runtime_error("dg_linear_forward_device_noalloc: " + std::to_string(m) + " rows of k=" +
                               std::to_string(l->k) + " need " + std::to_string(total) +
                               " bytes of scratch, more than its fixed " + std::to_string(kNoAllocScratchBytes) +
                               "-byte area; split the rows over several calls");
    DG_CUDA(cudaSetDevice(l->device));
    unsigned char* base = noalloc_scratch(l->device);
    DeviceStatus* st = reinterpret_cast<DeviceStatus*>(base + st_off);
    float* xs = reinterpret_cast<float*>(base + xs_off);
    int8_t* xq = reinterpret_cast<int8_t*>(base + xq_off);
    float* mid = reinterpret_cast<float*>(base + mid_off);
    float* ypad = reinterpret_cast<float*>(base + y_off);
    // The status word must start at zero; the scale rows past m (read as part
    // of the last 128-row tile) are cleared too so no stale value remains.
    DG_CUDA(cudaMemsetAsync(st, 0, sizeof(DeviceStatus), l->stream));
    DG_CUDA(cudaMemsetAsync(xs, 0, xs_bytes, l->stream));
    launch_norm_quant(x_device, l->k, m, l->k, nullptr, 0.0f, nullptr, 0, xq, xs, ldxs, st, l->stream);
    if (l->rank) {
      launch_lora_a(x_device, l->k, m, l->k, l->lora_a.as<float>(), l->rank, mid, 32, l->exact, l->stream);
    }
    CUtensorMap map_a;
    make_tmap_i8_2d(&map_a, xq, uint64_t(l->k), uint64_t(m), 128, 128);
    GemmArgs a{};
    a.M = m;
    a.N = l->n_pad;
    a.K = l->k;
    a.xs = xs;
    a.ldxs = ldxs;
    a.ws = l->ws_t.as<float>();
    a.lora_mid = mid;
    a.ld_mid = 32;
    a.lora_b = l->lora_b.as<float>();
    a.chunk_pid = l->chunk_pid.as<int>();
    a.lora_scale = l->scale;
    a.out = direct ? y_device : ypad;
    a.ldo = direct ? l->n : l->n_pad;
    a.status = st;
    a.dots = nullptr;
    launch_gemm_i8(map_a, l->maps, a, l->rank, kEpiWrite, l->exact, l->stream);
    if (!direct)
      DG_CUDA(cudaMemcpy2DAsync(y_device, size_t(l->n) * 4, ypad, size_t(l->n_pad) * 4, size_t(l->n) * 4, m,
                                cudaMemcpyDeviceToDevice, l->stream));
    DeviceStatus h{};
    DG_CUDA(cudaMemcpyAsync(&h, st, sizeof(h), cudaMemcpyDeviceToHost, l->stream));
    DG_CUDA(cudaStreamSynchronize(l->stream));
    if (h.code == kNonFinite) throw std::runtime_error("non-finite projection input");
    if (h.code)
      throw std::runtime_error("device error code " + std::to_string(h.code) + " at " + std::to_string(h.where));
  });
}

}  // extern "C"
