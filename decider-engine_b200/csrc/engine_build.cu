// Engine::finalize: device layouts of every projection, norms, RoPE table and
// the workspaces sized for `max_tokens` rows.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "engine.h"

namespace dg {

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

template <class T>
static DevBuf upload(const std::vector<T>& v) {
  DevBuf b(v.size() * sizeof(T));
  if (!v.empty()) DG_CUDA(cudaMemcpy(b.ptr, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return b;
}

// Projections that read the same input, concatenated along the output for one
// tcgen05 launch. Each part starts on a 32-column boundary (the LoRA block is
// chosen per 16-column chunk); the total is padded to the 256-column tile with
// zero weights. `interleave_mlp` alternates 16 gate columns with the 16
// matching up columns (SwiGLU epilogue).
DevProj Engine::build_fused(const std::vector<std::string>& keys, const std::vector<int>& outs, int in,
                            bool interleave_mlp) {
  const int P = int(keys.size()), R = c_.rank, G = in / 64;
  DevProj d;
  d.in = in;
  std::vector<int> off(P);
  int total = 0;
  if (interleave_mlp) {
    total = outs[0] + outs[1];
    off = {0, 0};
  } else {
    for (int p = 0; p < P; ++p) {
      off[p] = total;
      total = round_up(total + outs[p], 32);
    }
  }
  const int N = round_up(total, 256);
  d.out = total;
  d.out_pad = N;
  d.part_off = off;
  d.lora_rows = P * R;
  // Padding columns: zero weights, unit scales.
  d.wq = DevBuf(size_t(N) * in);
  DG_CUDA(cudaMemset(d.wq.ptr, 0, d.wq.bytes));
  d.ws_t = upload(std::vector<float>(size_t(G) * N, 1.0f));
  std::vector<float> lb(size_t(N) * R, 0.0f), la(size_t(P) * R * in);
  std::vector<int> pid(N / 16, 0);
  for (int p = 0; p < P; ++p) {
    HostTensor w = take(keys[p] + ".weight");
    if (!w.quantized || w.bits != 8) throw std::runtime_error("fused projection needs INT8 weights");
    HostTensor A = take("base_model.model." + keys[p] + ".lora_A.weight");
    HostTensor B = take("base_model.model." + keys[p] + ".lora_B.weight");
    std::copy(A.f32.begin(), A.f32.end(), la.begin() + size_t(p) * R * in);
    // Every 32 fused columns of the MLP hold 16 gate columns then the 16
    // matching up columns, so any tile of 128 or 256 columns splits into
    // whole pairs; other parts are contiguous from their offset.
    auto fused_row = [&](int j) { return interleave_mlp ? (j / 16) * 32 + p * 16 + (j % 16) : off[p] + j; };
    // Data::quantize on the device, straight into the fused layout (rows
    // of the weights at their fused rows, scales transposed to [G][N]).
    QuantLayout L;
    L.q_row = size_t(in);
    L.s_row = 1;
    L.s_group = size_t(N);
    L.rb = interleave_mlp ? 16 : std::max(outs[p], 1);
    L.rs = interleave_mlp ? 32 : 0;
    L.ro = interleave_mlp ? p * 16 : off[p];
    {
      DevBuf wf = upload(w.f32);
      quantize_weights_device(wf.as<float>(), size_t(outs[p]), size_t(in), 8, d.wq.as<uint8_t>(), d.ws_t.as<float>(),
                              &L, 0);
      DG_CUDA(cudaStreamSynchronize(0));
    }
    for (int j = 0; j < outs[p]; ++j) {
      const int r = fused_row(j);
      std::copy(B.f32.begin() + size_t(j) * R, B.f32.begin() + size_t(j + 1) * R, lb.begin() + size_t(r) * R);
      pid[r / 16] = p;
    }
  }
  d.lora_a = upload(la);
  d.lora_b = upload(lb);
  d.chunk_pid = upload(pid);
  make_weight_maps(&d.maps, d.wq.ptr, in, N, d.lora_b.as<float>(), R);
  return d;
}

// One projection for the generic SIMT kernel, in the reference's own layout.
DevProj Engine::build_generic_proj(const std::string& key, int in, int out, bool lora, bool bias) {
  DevProj d;
  d.in = in;
  d.out = d.out_pad = out;
  HostTensor w = take(key + ".weight");
  GenericProj& g = d.g;
  g.in = in;
  g.out = out;
  if (w.quantized) {
    // Data::quantize on the device, in the reference's own layout.
    g.precision = precision_;
    const size_t rows = size_t(w.shape[0]), width = size_t(w.shape[1]);
    d.wq = DevBuf(w.bits == 8 ? rows * width : (rows * width + 1) / 2);
    d.scale_rows = DevBuf(rows * ((width + 63) / 64) * 4);
    {
      DevBuf wf = upload(w.f32);
      quantize_weights_device(wf.as<float>(), rows, width, w.bits, d.wq.as<uint8_t>(), d.scale_rows.as<float>(),
                              nullptr, 0);
      if (precision_ != kInt8Compute) {
        // Weight-only precisions: the dequantised FP32 weights too, for the
        // tensor-core projections of the fast mode.
        d.w_f32 = DevBuf(rows * width * 4);
        dequantize_weights_device(d.wq.as<uint8_t>(), d.scale_rows.as<float>(), rows, width, w.bits,
                                  d.w_f32.as<float>(), 0);
      }
      DG_CUDA(cudaStreamSynchronize(0));
    }
    g.wq = d.wq.as<uint8_t>();
    g.wscale = d.scale_rows.as<float>();
  } else {
    g.precision = 0;
    d.w_f32 = upload(w.f32);
    g.w = d.w_f32.as<float>();
  }
  if (bias) {
    d.bias = upload(take(key + ".bias").f32);
    g.bias = d.bias.as<float>();
  }
  if (lora && c_.rank > 0) {
    d.lora_a = upload(take("base_model.model." + key + ".lora_A.weight").f32);
    d.lora_b = upload(take("base_model.model." + key + ".lora_B.weight").f32);
    d.lora_rows = c_.rank;
    g.lora_b = d.lora_b.as<float>();
    g.rank = c_.rank;
    g.lora_scale = c_.lora_scale;
  }
  return d;
}

void Engine::finalize() {
  if (finalized_) return;
  DG_CUDA(cudaSetDevice(device_));
  for (auto& kv : expected_names())
    if (!staged_.count(kv.first)) throw std::runtime_error("missing tensor " + kv.first);
  const Config& c = c_;
  const int H = c.hidden, I = c.intermediate;
  // The tcgen05 path needs INT8-compute, rank-32 LoRA and 128-aligned widths.
  fast_ = precision_ == kInt8Compute && c.rank == 32 && H % 256 == 0 && I % 128 == 0 && c.qw() % 128 == 0 &&
          c.vd() % 128 == 0 && c.conv_width() % 32 == 0 && c.kw() % 32 == 0 && c.value_heads <= 32;
  int ld_proj = 0;
  layers_.resize(c.layers);
  for (int i = 0; i < c.layers; ++i) {
    Layer& L = layers_[i];
    const std::string p = "layers." + std::to_string(i) + ".";
    L.full = c.layer_types[i] == 1;
    if (fast_) {
      if (L.full) {
        L.in_proj = build_fused({p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"},
                                {2 * c.qw(), c.kw(), c.kw()}, H, false);
        L.out_proj = build_fused({p + "self_attn.o_proj"}, {H}, c.qw(), false);
      } else {
        L.in_proj = build_fused({p + "linear_attn.in_proj_qkv", p + "linear_attn.in_proj_z",
                                 p + "linear_attn.in_proj_a", p + "linear_attn.in_proj_b"},
                                {c.conv_width(), c.vd(), c.value_heads, c.value_heads}, H, false);
        L.out_proj = build_fused({p + "linear_attn.out_proj"}, {H}, c.vd(), false);
      }
      L.mlp_in = build_fused({p + "mlp.gate_proj", p + "mlp.up_proj"}, {I, I}, H, true);
      L.down = build_fused({p + "mlp.down_proj"}, {H}, I, false);
      ld_proj = std::max(ld_proj, L.in_proj.out_pad);
    } else {
      if (L.full) {
        L.parts.push_back(build_generic_proj(p + "self_attn.q_proj", H, 2 * c.qw(), true, false));
        L.parts.push_back(build_generic_proj(p + "self_attn.k_proj", H, c.kw(), true, false));
        L.parts.push_back(build_generic_proj(p + "self_attn.v_proj", H, c.kw(), true, false));
        L.parts.push_back(build_generic_proj(p + "self_attn.o_proj", c.qw(), H, true, false));
        L.in_proj.part_off = {0, 2 * c.qw(), 2 * c.qw() + c.kw()};
        ld_proj = std::max(ld_proj, 2 * c.qw() + 2 * c.kw());
      } else {
        L.parts.push_back(build_generic_proj(p + "linear_attn.in_proj_qkv", H, c.conv_width(), true, false));
        L.parts.push_back(build_generic_proj(p + "linear_attn.in_proj_z", H, c.vd(), true, false));
        L.parts.push_back(build_generic_proj(p + "linear_attn.in_proj_a", H, c.value_heads, true, false));
        L.parts.push_back(build_generic_proj(p + "linear_attn.in_proj_b", H, c.value_heads, true, false));
        L.parts.push_back(build_generic_proj(p + "linear_attn.out_proj", c.vd(), H, true, false));
        const int W = c.conv_width();
        L.in_proj.part_off = {0, W, W + c.vd(), W + c.vd() + c.value_heads};
        ld_proj = std::max(ld_proj, W + c.vd() + 2 * c.value_heads);
      }
      L.parts.push_back(build_generic_proj(p + "mlp.gate_proj", H, I, true, false));
      L.parts.push_back(build_generic_proj(p + "mlp.up_proj", H, I, true, false));
      L.parts.push_back(build_generic_proj(p + "mlp.down_proj", I, H, true, false));
    }
    L.input_norm = upload(take(p + "input_layernorm.weight").f32);
    L.post_norm = upload(take(p + "post_attention_layernorm.weight").f32);
    if (L.full) {
      L.q_norm = upload(take(p + "self_attn.q_norm.weight").f32);
      L.k_norm = upload(take(p + "self_attn.k_norm.weight").f32);
    } else {
      const int W = c.conv_width(), k = c.conv_kernel;
      std::vector<float> raw = take(p + "linear_attn.conv1d.weight").f32, tap(raw.size());
      // tap_major, src/qwen.rs:698-703: [channel][1][tap] -> [tap][channel]
      for (size_t j = 0; j < raw.size(); ++j) tap[j] = raw[(j % W) * k + j / W];
      L.conv = upload(tap);
      L.dt = upload(take(p + "linear_attn.dt_bias").f32);
      std::vector<float> rate = take(p + "linear_attn.A_log").f32;
      for (auto& v : rate) v = -std::exp(v);  // src/qwen.rs:342-349
      L.decay_rate = upload(rate);
      L.norm = upload(take(p + "linear_attn.norm.weight").f32);
    }
  }
  embedding_ = upload(take("embed_tokens.weight").f32);
  final_norm_ = upload(take("norm.weight").f32);
  if (c.pointer_dim > 0) {
    head_norm_w_ = upload(take("head.norm.weight").f32);
    head_norm_b_ = upload(take("head.norm.bias").f32);
    head_q_ = build_generic_proj("head.q", H, c.pointer_dim, false, true);
    head_k_ = build_generic_proj("head.k", H, c.pointer_dim, false, true);
  }
  staged_.clear();
  // RoPE table for every position of the window, with the reference's own
  // float formulas (src/qwen.rs:389-396,452-458): divisor_i = theta^(2i/r),
  // angle = pos / divisor_i, (sin, cos).
  const int r = c.rotary_dim();
  rope_half_ = r / 2;
  {
    std::vector<float> div(rope_half_), tab(size_t(4096) * rope_half_ * 2);
    for (int i = 0; i < rope_half_; ++i) div[i] = std::pow(c.rope_theta, float(2 * i) / float(r));
    for (int pos = 0; pos < 4096; ++pos)
      for (int i = 0; i < rope_half_; ++i) {
        const float a = float(pos) / div[i];
        tab[(size_t(pos) * rope_half_ + i) * 2] = std::sin(a);
        tab[(size_t(pos) * rope_half_ + i) * 2 + 1] = std::cos(a);
      }
    rope_ = upload(tab);
  }
  alloc_workspaces(ld_proj);
  finalized_ = true;
}

// Read-only views of a projection / layer of another engine's weights.
static DevProj proj_view(const DevProj& p) {
  DevProj d;
  d.in = p.in;
  d.out = p.out;
  d.out_pad = p.out_pad;
  d.wq = DevBuf::view_of(p.wq);
  d.ws_t = DevBuf::view_of(p.ws_t);
  d.lora_a = DevBuf::view_of(p.lora_a);
  d.lora_b = DevBuf::view_of(p.lora_b);
  d.chunk_pid = DevBuf::view_of(p.chunk_pid);
  d.maps = p.maps;
  d.lora_rows = p.lora_rows;
  d.part_off = p.part_off;
  d.g = p.g;
  d.w_f32 = DevBuf::view_of(p.w_f32);
  d.scale_rows = DevBuf::view_of(p.scale_rows);
  d.bias = DevBuf::view_of(p.bias);
  return d;
}

static Layer layer_view(const Layer& L) {
  Layer v;
  v.full = L.full;
  v.input_norm = DevBuf::view_of(L.input_norm);
  v.post_norm = DevBuf::view_of(L.post_norm);
  v.in_proj = proj_view(L.in_proj);
  v.out_proj = proj_view(L.out_proj);
  v.mlp_in = proj_view(L.mlp_in);
  v.down = proj_view(L.down);
  for (const DevProj& p : L.parts) v.parts.push_back(proj_view(p));
  v.q_norm = DevBuf::view_of(L.q_norm);
  v.k_norm = DevBuf::view_of(L.k_norm);
  v.conv = DevBuf::view_of(L.conv);
  v.dt = DevBuf::view_of(L.dt);
  v.decay_rate = DevBuf::view_of(L.decay_rate);
  v.norm = DevBuf::view_of(L.norm);
  return v;
}

void Engine::share_weights(const Engine& base) {
  if (finalized_ || !staged_.empty()) throw std::runtime_error("share_weights: this engine already has weights");
  if (!base.finalized_) throw std::runtime_error("share_weights: the base engine is not finalized");
  if (base.device_ != device_ || base.precision_ != precision_ || base.max_tokens_ != max_tokens_ ||
      base.c_.layers != c_.layers || base.c_.hidden != c_.hidden || base.c_.vocab != c_.vocab ||
      base.c_.pointer_dim != c_.pointer_dim || base.c_.rank != c_.rank)
    throw std::runtime_error("share_weights: the engines differ in device, precision, model or token budget");
  DG_CUDA(cudaSetDevice(device_));
  fast_ = base.fast_;
  layers_.clear();
  for (const Layer& L : base.layers_) layers_.push_back(layer_view(L));
  embedding_ = DevBuf::view_of(base.embedding_);
  final_norm_ = DevBuf::view_of(base.final_norm_);
  rope_ = DevBuf::view_of(base.rope_);
  rope_half_ = base.rope_half_;
  head_norm_w_ = DevBuf::view_of(base.head_norm_w_);
  head_norm_b_ = DevBuf::view_of(base.head_norm_b_);
  head_q_ = proj_view(base.head_q_);
  head_k_ = proj_view(base.head_k_);
  alloc_workspaces(base.ld_proj_);
  finalized_ = true;
}

void Engine::alloc_workspaces(int ld_proj) {
  const Config& c = c_;
  const int H = c.hidden, I = c.intermediate;
  const int M = max_tokens_;
  const int kmax = std::max(std::max(H, I), std::max(c.qw(), c.vd()));
  ldxs_ = round_up(M, 128);
  ld_proj_ = round_up(ld_proj, 4);
  ids_ = DevBuf(size_t(M) * 4);
  x_ = DevBuf(size_t(M) * H * 4);
  n_ = DevBuf(size_t(M) * H * 4);
  xq_ = DevBuf(size_t(M) * kmax);
  xs_ = DevBuf(size_t((kmax + 63) / 64) * ldxs_ * 4);
  DG_CUDA(cudaMemset(xs_.ptr, 0, xs_.bytes));
  mid_ = DevBuf(size_t(M) * 128 * 4);
  proj_ = DevBuf(size_t(M) * ld_proj_ * 4);
  conv_ = DevBuf(size_t(M) * c.conv_width() * 4);
  decay_ = DevBuf(size_t(M) * c.value_heads * 4);
  beta_ = DevBuf(size_t(M) * c.value_heads * 4);
  o_ = DevBuf(size_t(M) * c.vd() * 4);
  ofin_ = DevBuf(size_t(M) * c.vd() * 4);
  h_ = DevBuf(size_t(M) * I * 4);
  qbuf_ = DevBuf(size_t(M) * c.qw() * 4);
  att_ = DevBuf(size_t(M) * c.qw() * 4);
  kcache_.resize(c.layers);
  vcache_.resize(c.layers);
  state_.resize(c.layers);
  for (int i = 0; i < c.layers; ++i) {
    if (layers_[i].full) {
      kcache_[i] = DevBuf(size_t(4096) * c.kw() * 4);
      vcache_[i] = DevBuf(size_t(4096) * c.kw() * 4);
    } else {
      state_[i] = DevBuf(size_t(c.value_heads) * c.dk * c.dv * 4);
    }
  }
  if (c.dk == 128 && c.dv == 128)
    delta_ws_ = DevBuf(delta_chunk_workspace_bytes(1, c.value_heads, M));
  if (fast_ && attention_tc_supported(c.head_dim, c.heads, c.kv_heads))
    attn_ws_ = DevBuf(attention_tc_workspace_floats(c.heads, c.kv_heads, c.head_dim, M) * 4);
  if (segments_supported()) {
    // Segmented forwards: the sequences' own K/V rows (the shared prefix stays in the Prefix).
    kseg_ = DevBuf(size_t(M) * c.kw() * 4);
    vseg_ = DevBuf(size_t(M) * c.kw() * 4);
  }
  if (fast_) lora_part_ = DevBuf(lora_a_partial_floats(M) * 4);
  if (!fast_ && precision_ != kInt8Compute) tc_prod_ = DevBuf(size_t(M) * I * 4);
  if (fast_) {
    gemm_split_ws_ = DevBuf(kGemmSplitFloats * 4);
    gemm_split_cnt_ = DevBuf(kGemmSplitTiles * sizeof(int));
    DG_CUDA(cudaMemset(gemm_split_cnt_.ptr, 0, gemm_split_cnt_.bytes));
  }
  constexpr int kMaxHeadRows = 512;
  hrow_idx_ = DevBuf(kMaxHeadRows * 4);
  hnorm_ = DevBuf(size_t(kMaxHeadRows) * H * 4);
  const int P = std::max(1, c.pointer_dim);
  hq_ = DevBuf(size_t(P) * 4);
  hk_ = DevBuf(size_t(kMaxHeadRows) * P * 4);
  hlogits_ = DevBuf(kMaxHeadRows * 4);
  status_ = DevBuf(sizeof(DeviceStatus));
  DG_CUDA(cudaMemset(status_.ptr, 0, sizeof(DeviceStatus)));
  DG_CUDA(cudaDeviceSynchronize());
}

}  // namespace dg
