// Engine::forward: Model::run (src/qwen.rs:426-504) on the device, plus the
// pointer head (src/lib.rs:116-131).
#include <algorithm>
#include <cmath>
#include <map>
#include <utility>

#include "engine.h"

namespace dg {

struct DgError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Activation tensor maps, cached per (buffer, K, rows): the rows extent makes
// TMA fill rows past the sequence with zeros.
static const CUtensorMap& act_map(const void* base, int K, int rows) {
  static thread_local std::map<std::tuple<const void*, int, int>, CUtensorMap> cache;
  auto key = std::make_tuple(base, K, rows);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  CUtensorMap m;
  make_tmap_i8_2d(&m, base, uint64_t(K), uint64_t(rows), 128, 128);
  return cache.emplace(key, m).first->second;
}

void Engine::run_proj_fast(const DevProj& p, int M, const float* mid, float* out, int ldo, int epi) {
  GemmArgs a{};
  a.M = M;
  a.N = p.out_pad;
  a.K = p.in;
  a.xs = xs_.as<float>();
  a.ldxs = ldxs_;
  a.ws = p.ws_t.as<float>();
  a.lora_mid = mid;
  a.ld_mid = 128;
  a.lora_b = p.lora_b.as<float>();
  a.chunk_pid = p.chunk_pid.as<int>();
  a.lora_scale = c_.lora_scale;
  a.out = out;
  a.ldo = ldo;
  a.status = status();
  // Every fast projection directly follows its own LoRA-A launch.
  a.late_dep = lora_overlap_ ? 1 : 0;
  a.split_ws = gemm_split_ws_.as<float>();
  a.split_cnt = gemm_split_cnt_.as<int>();
  a.split_ws_floats = gemm_split_ws_.bytes / 4;
  const size_t k = gemm_ops_pending_.size();
  fwd_ops_all_ += 2.0 * M * p.out * p.in;
  ++fwd_proj_;
  const bool timed = cur_layer_ >= gemm_lo_ && cur_layer_ < gemm_hi_ && 2 * k + 2 <= gemm_ev_.size();
  // While a graph is captured, external records become event nodes of it.
  unsigned rec = cudaEventRecordDefault;
  if (timed) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    DG_CUDA(cudaStreamIsCapturing(stream_, &cs));
    if (cs == cudaStreamCaptureStatusActive) rec = cudaEventRecordExternal;
    DG_CUDA(cudaEventRecordWithFlags(gemm_ev_[2 * k], stream_, rec));
  }
  launch_gemm_i8(act_map(xq_.ptr, p.in, M), p.maps, a, 32, epi, exact, stream_);
  if (timed) {
    DG_CUDA(cudaEventRecordWithFlags(gemm_ev_[2 * k + 1], stream_, rec));
    gemm_ops_pending_.push_back(2.0 * M * p.out * p.in);
  }
}

void Engine::run_proj_generic(const DevProj& p, const float* x, int ldx, int M, float* out, int ldo, int epi) {
  // Fast mode with FP32 weights (checkpoint precision, or the dequantised
  // weights of the int8 and int4 weight-only precisions): the product on the
  // tensor cores (3 x TF32, FP32 sums per 32-wide K chunk), then LoRA-B as a
  // second product added into the output, then the bias and the SwiGLU.
  // int8-compute quantises its activations and keeps its own kernel.
  const bool lora_tc = p.lora_rows == 0 || (p.lora_rows % 32 == 0 && p.lora_rows <= 128 && p.g.rank == p.lora_rows);
  if (!exact && p.g.precision != kInt8Compute && p.w_f32.ptr && p.in % 32 == 0 && ldx % 4 == 0 &&
      reinterpret_cast<uintptr_t>(x) % 16 == 0 && lora_tc &&
      (epi != kEpiSwiGlu || (tc_prod_.ptr && size_t(M) * p.out * 4 <= tc_prod_.bytes))) {
    float* dst = epi == kEpiSwiGlu ? tc_prod_.as<float>() : out;
    const int ldd = epi == kEpiSwiGlu ? p.out : ldo;
    TcGemmArgs g;
    g.A = x;
    g.lda = ldx;
    g.B = p.w_f32.as<float>();
    g.ldb = p.in;
    g.C = dst;
    g.ldc = ldd;
    g.M = M;
    g.N = p.out;
    g.K = p.in;
    g.accumulate = epi == kEpiAdd ? 1 : 0;
    g.status = status();
    launch_tc_gemm(g, 1, stream_);
    if (p.lora_rows) {
      launch_lora_a(x, ldx, M, p.in, p.lora_a.as<float>(), p.lora_rows, mid_.as<float>(), 128, false, stream_);
      TcGemmArgs l;
      l.A = mid_.as<float>();
      l.lda = 128;
      l.B = p.lora_b.as<float>();
      l.ldb = p.lora_rows;
      l.C = dst;
      l.ldc = ldd;
      l.M = M;
      l.N = p.out;
      l.K = p.lora_rows;
      l.alpha = p.g.lora_scale;
      l.accumulate = 1;
      l.status = status();
      launch_tc_gemm(l, 1, stream_);
    }
    if (epi == kEpiSwiGlu || p.g.bias)
      launch_proj_finish(dst, ldd, p.g.bias, out, ldo, M, p.out, epi == kEpiSwiGlu ? kEpiSwiGlu : kEpiWrite,
                         stream_);
    return;
  }
  if (p.lora_rows) {
    launch_lora_a(x, ldx, M, p.in, p.lora_a.as<float>(), p.lora_rows, mid_.as<float>(), 128, true, stream_);
  }
  launch_proj_generic(p.g, x, ldx, xq_.as<int8_t>(), xs_.as<float>(), ldxs_, mid_.as<float>(), 128, M, out, ldo, epi,
                      stream_);
}

// DeltaNet mixer after the input projections (src/qwen.rs:667-693): conv with
// the prefix tail, recurrence from the prefix state, gated norm; captures the
// next tail and state when prefilling.
void Engine::mixer_tail(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap,
                        const float* raw, int ldr) {
  const Config& c = c_;
  const Layer& L = layers_[i];
  const int W = c.conv_width(), k = c.conv_kernel, H = c.value_heads;
  const float* tail = past ? past->tail.as<float>() : nullptr;
  const int tail_rows = past ? past->tail_rows : 0;
  if (tail_rows != std::min(start, k - 1)) throw DgError("prefix cache does not match the layer types");
  const int* off = L.in_proj.part_off.data();
  float* base = proj_.as<float>();
  const size_t sbytes = size_t(H) * c.dk * c.dv * 4;
  if (seg_len_) {
    // segs_ sequences of seg_len_ rows, each from the prefix's tail and state.
    const int sl = seg_len_, ns = segs_;
    launch_conv_silu(raw, ldr, sl, tail, tail_rows, start, W, k, L.conv.as<float>(), conv_.as<float>(), stream_, ns);
    launch_delta_prep(conv_.as<float>(), W, n, c.key_heads, c.dk, H, base + off[2], base + off[3], ldr,
                      L.decay_rate.as<float>(), L.dt.as<float>(), decay_.as<float>(), beta_.as<float>(), stream_);
    if (past)
      launch_broadcast_copy(seg_state_.ptr, past->state.ptr, sbytes, ns, stream_);
    else
      DG_CUDA(cudaMemsetAsync(seg_state_.ptr, 0, sbytes * ns, stream_));
    DeltaArgs da{};
    da.q = conv_.as<float>();
    da.k = conv_.as<float>() + c.kd();
    da.v = conv_.as<float>() + 2 * c.kd();
    da.ld_qk = da.ld_v = W;
    da.bs_qkv = size_t(sl) * W;
    da.decay = decay_.as<float>();
    da.beta = beta_.as<float>();
    da.log_decay = 1;
    da.ld_gb = H;
    da.bs_gb = size_t(sl) * H;
    da.n = sl;
    da.key_heads = c.key_heads;
    da.value_heads = H;
    da.dv = c.dv;
    da.state = seg_state_.as<float>();
    da.bs_state = sbytes / 4;
    da.o = o_.as<float>();
    da.ldo = H * c.dv;
    da.bs_o = size_t(sl) * H * c.dv;
    // As for one sequence: the chunked form in fast mode for more than one
    // chunk (when the workspace holds every sequence's chunks), else the
    // token recurrence.
    if (!exact && delta_ws_.ptr && sl > kDeltaChunk &&
        delta_chunk_workspace_bytes(ns, H, sl) <= delta_ws_.bytes)
      launch_delta_chunked(da, ns, delta_ws_.ptr, delta_ws_.bytes, stream_, wide_scan);
    else
      launch_delta_rec128(da, ns, stream_);
    const bool q = precision_ == kInt8Compute;
    launch_gated_norm_quant(o_.as<float>(), base + off[1], ldr, n, H, c.dv, L.norm.as<float>(), c.eps,
                            ofin_.as<float>(), xq_.as<int8_t>(), xs_.as<float>(), ldxs_, q, status(), stream_);
    return;
  }
  launch_conv_silu(raw, ldr, n, tail, tail_rows, start, W, k, L.conv.as<float>(), conv_.as<float>(), stream_);
  launch_delta_prep(conv_.as<float>(), W, n, c.key_heads, c.dk, H, base + off[2], base + off[3], ldr,
                    L.decay_rate.as<float>(), L.dt.as<float>(), decay_.as<float>(), beta_.as<float>(), stream_);
  if (past)
    DG_CUDA(cudaMemcpyAsync(state_[i].ptr, past->state.ptr, sbytes, cudaMemcpyDeviceToDevice, stream_));
  else
    DG_CUDA(cudaMemsetAsync(state_[i].ptr, 0, sbytes, stream_));
  if (!exact && delta_ws_.ptr && n > kDeltaChunk) {
    // Fast mode: the chunked form (64-token chunks); its rounding depends on
    // where chunks start, so prefix continuations match full passes to FP32
    // rounding rather than bit for bit. Exact mode keeps the token recurrence,
    // and so does a pass of one chunk or less (a question after a state),
    // where the chunked form's prep runs one CTA per head.
    DeltaArgs da{};
    da.q = conv_.as<float>();
    da.k = conv_.as<float>() + c.kd();
    da.v = conv_.as<float>() + 2 * c.kd();
    da.ld_qk = da.ld_v = W;
    da.decay = decay_.as<float>();
    da.beta = beta_.as<float>();
    da.log_decay = 1;
    da.ld_gb = H;
    da.n = n;
    da.key_heads = c.key_heads;
    da.value_heads = H;
    da.dv = c.dv;
    da.state = state_[i].as<float>();
    da.o = o_.as<float>();
    da.ldo = H * c.dv;
    launch_delta_chunked(da, 1, delta_ws_.ptr, delta_ws_.bytes, stream_, wide_scan);
  } else {
    launch_delta_recurrence(conv_.as<float>(), n, c.key_heads, c.dk, H, c.dv, decay_.as<float>(),
                            beta_.as<float>(), state_[i].as<float>(), o_.as<float>(), stream_);
  }
  const bool q = precision_ == kInt8Compute;
  launch_gated_norm_quant(o_.as<float>(), base + off[1], ldr, n, H, c.dv, L.norm.as<float>(), c.eps, ofin_.as<float>(),
                          xq_.as<int8_t>(), xs_.as<float>(), ldxs_, q, status(), stream_);
  if (cap) {
    cap->full = false;
    cap->state = DevBuf::pooled_on(sbytes, stream_);
    DG_CUDA(cudaMemcpyAsync(cap->state.ptr, state_[i].ptr, sbytes, cudaMemcpyDeviceToDevice, stream_));
    const int keep = std::min(start + n, k - 1), from_tail = std::max(0, keep - n), from_raw = keep - from_tail;
    cap->tail_rows = keep;
    cap->tail = DevBuf::pooled_on(size_t(std::max(keep, 1)) * W * 4, stream_);
    if (from_tail)
      DG_CUDA(cudaMemcpyAsync(cap->tail.ptr, tail + size_t(tail_rows - from_tail) * W, size_t(from_tail) * W * 4,
                              cudaMemcpyDeviceToDevice, stream_));
    if (from_raw)
      DG_CUDA(cudaMemcpy2DAsync(cap->tail.as<float>() + size_t(from_tail) * W, size_t(W) * 4,
                                raw + size_t(n - from_raw) * ldr, size_t(ldr) * 4, size_t(W) * 4, from_raw,
                                cudaMemcpyDeviceToDevice, stream_));
  }
}

void Engine::layer_fast(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap) {
  const Config& c = c_;
  const Layer& L = layers_[i];
  const int H = c.hidden, I = c.intermediate;
  float* x = x_.as<float>();
  float* nb = n_.as<float>();
  float* mid = mid_.as<float>();
  float* proj = proj_.as<float>();
  // mid = x · Aᵀ of a projection's fused LoRA parts (x: k-wide rows).
  auto lora_a = [&](const float* xin, int k, const DevProj& p) {
    launch_lora_a(xin, k, n, k, p.lora_a.as<float>(), p.lora_rows, mid, 128, exact, stream_, lora_part_.as<float>(),
                  lora_part_.bytes / 4, status(), lora_overlap_);
  };
  launch_norm_quant(x, H, n, H, L.input_norm.as<float>(), c.eps, nb, H, xq_.as<int8_t>(), xs_.as<float>(), ldxs_,
                    status(), stream_);
  dump_codes(n, H);
  lora_a(nb, H, L.in_proj);
  run_proj_fast(L.in_proj, n, mid, proj, ld_proj_, kEpiWrite);
  const float* mixed_in;
  int kin;
  if (L.full) {
    const int d = c.head_dim, kw = c.kw();
    if (seg_len_) {
      // The prefix's keys are read in place; the sequences' own go to kseg_/vseg_.
      launch_qk_norm_rope(proj, ld_proj_, n, c.heads, c.kv_heads, d, L.q_norm.as<float>(), L.k_norm.as<float>(),
                          c.eps, rope_.as<float>(), rope_half_, start, qbuf_.as<float>(), kseg_.as<float>(),
                          vseg_.as<float>(), stream_, seg_len_);
      launch_attention(qbuf_.as<float>(), past ? past->k.as<float>() : kseg_.as<float>(),
                       past ? past->v.as<float>() : vseg_.as<float>(), proj, ld_proj_, n, start, c.heads, c.kv_heads,
                       d, att_.as<float>(), exact, stream_, seg_len_, kseg_.as<float>(), vseg_.as<float>());
    } else {
      if (past) {
        DG_CUDA(cudaMemcpyAsync(kcache_[i].ptr, past->k.ptr, size_t(start) * kw * 4, cudaMemcpyDeviceToDevice, stream_));
        DG_CUDA(cudaMemcpyAsync(vcache_[i].ptr, past->v.ptr, size_t(start) * kw * 4, cudaMemcpyDeviceToDevice, stream_));
      }
      launch_qk_norm_rope(proj, ld_proj_, n, c.heads, c.kv_heads, d, L.q_norm.as<float>(), L.k_norm.as<float>(),
                          c.eps, rope_.as<float>(), rope_half_, start, qbuf_.as<float>(), kcache_[i].as<float>(),
                          vcache_[i].as<float>(), stream_);
      if (!exact && attn_tc_ && attn_ws_.ptr)
        launch_attention_tc(qbuf_.as<float>(), kcache_[i].as<float>(), vcache_[i].as<float>(), proj, ld_proj_, n,
                            start, c.heads, c.kv_heads, d, att_.as<float>(), attn_ws_.as<float>(), attn_ws_.bytes / 4,
                            status(), stream_);
      else
        launch_attention(qbuf_.as<float>(), kcache_[i].as<float>(), vcache_[i].as<float>(), proj, ld_proj_, n, start,
                         c.heads, c.kv_heads, d, att_.as<float>(), exact, stream_);
    }
    launch_norm_quant(att_.as<float>(), c.qw(), n, c.qw(), nullptr, c.eps, nullptr, 0, xq_.as<int8_t>(),
                      xs_.as<float>(), ldxs_, status(), stream_);
    dump_codes(n, c.qw());
    if (cap) {
      cap->full = true;
      cap->k = DevBuf::pooled_on(size_t(start + n) * kw * 4, stream_);
      cap->v = DevBuf::pooled_on(size_t(start + n) * kw * 4, stream_);
      DG_CUDA(cudaMemcpyAsync(cap->k.ptr, kcache_[i].ptr, cap->k.bytes, cudaMemcpyDeviceToDevice, stream_));
      DG_CUDA(cudaMemcpyAsync(cap->v.ptr, vcache_[i].ptr, cap->v.bytes, cudaMemcpyDeviceToDevice, stream_));
    }
    mixed_in = att_.as<float>();
    kin = c.qw();
  } else {
    mixer_tail(i, n, start, past, cap, proj, ld_proj_);
    dump_codes(n, c.vd());
    mixed_in = ofin_.as<float>();
    kin = c.vd();
  }
  lora_a(mixed_in, kin, L.out_proj);
  run_proj_fast(L.out_proj, n, mid, x, H, kEpiAdd);  // x += mixed (residual_norm's add)
  launch_norm_quant(x, H, n, H, L.post_norm.as<float>(), c.eps, nb, H, xq_.as<int8_t>(), xs_.as<float>(), ldxs_,
                    status(), stream_);
  dump_codes(n, H);
  lora_a(nb, H, L.mlp_in);
  run_proj_fast(L.mlp_in, n, mid, h_.as<float>(), I, kEpiSwiGlu);
  launch_norm_quant(h_.as<float>(), I, n, I, nullptr, c.eps, nullptr, 0, xq_.as<int8_t>(), xs_.as<float>(), ldxs_,
                    status(), stream_);
  dump_codes(n, I);
  lora_a(h_.as<float>(), I, L.down);
  run_proj_fast(L.down, n, mid, x, H, kEpiAdd);
}

void Engine::layer_generic(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap) {
  const Config& c = c_;
  const Layer& L = layers_[i];
  const int H = c.hidden, I = c.intermediate;
  const bool q = precision_ == kInt8Compute;
  float* x = x_.as<float>();
  float* nb = n_.as<float>();
  float* proj = proj_.as<float>();
  int8_t* xq = q ? xq_.as<int8_t>() : nullptr;
  launch_norm_quant(x, H, n, H, L.input_norm.as<float>(), c.eps, nb, H, xq, xs_.as<float>(), ldxs_, status(), stream_);
  const int* off = L.in_proj.part_off.data();
  int mlp = 0;
  if (L.full) {
    for (int p = 0; p < 3; ++p) run_proj_generic(L.parts[p], nb, H, n, proj + off[p], ld_proj_, kEpiWrite);
    const int d = c.head_dim, kw = c.kw();
    if (past) {
      DG_CUDA(cudaMemcpyAsync(kcache_[i].ptr, past->k.ptr, size_t(start) * kw * 4, cudaMemcpyDeviceToDevice, stream_));
      DG_CUDA(cudaMemcpyAsync(vcache_[i].ptr, past->v.ptr, size_t(start) * kw * 4, cudaMemcpyDeviceToDevice, stream_));
    }
    launch_qk_norm_rope(proj, ld_proj_, n, c.heads, c.kv_heads, d, L.q_norm.as<float>(), L.k_norm.as<float>(), c.eps,
                        rope_.as<float>(), rope_half_, start, qbuf_.as<float>(), kcache_[i].as<float>(),
                        vcache_[i].as<float>(), stream_);
    launch_attention(qbuf_.as<float>(), kcache_[i].as<float>(), vcache_[i].as<float>(), proj, ld_proj_, n, start,
                     c.heads, c.kv_heads, d, att_.as<float>(), true, stream_);
    if (q) {
      launch_norm_quant(att_.as<float>(), c.qw(), n, c.qw(), nullptr, c.eps, nullptr, 0, xq, xs_.as<float>(), ldxs_,
                        status(), stream_);
    }
    if (cap) {
      cap->full = true;
      cap->k = DevBuf::pooled_on(size_t(start + n) * kw * 4, stream_);
      cap->v = DevBuf::pooled_on(size_t(start + n) * kw * 4, stream_);
      DG_CUDA(cudaMemcpyAsync(cap->k.ptr, kcache_[i].ptr, cap->k.bytes, cudaMemcpyDeviceToDevice, stream_));
      DG_CUDA(cudaMemcpyAsync(cap->v.ptr, vcache_[i].ptr, cap->v.bytes, cudaMemcpyDeviceToDevice, stream_));
    }
    run_proj_generic(L.parts[3], att_.as<float>(), c.qw(), n, x, H, kEpiAdd);
    mlp = 4;
  } else {
    for (int p = 0; p < 4; ++p) run_proj_generic(L.parts[p], nb, H, n, proj + off[p], ld_proj_, kEpiWrite);
    mixer_tail(i, n, start, past, cap, proj, ld_proj_);
    run_proj_generic(L.parts[4], ofin_.as<float>(), c.vd(), n, x, H, kEpiAdd);
    mlp = 5;
  }
  launch_norm_quant(x, H, n, H, L.post_norm.as<float>(), c.eps, nb, H, xq, xs_.as<float>(), ldxs_, status(), stream_);
  run_proj_generic(L.parts[mlp], nb, H, n, h_.as<float>(), I, kEpiWrite);
  run_proj_generic(L.parts[mlp + 1], nb, H, n, h_.as<float>(), I, kEpiSwiGlu);
  if (q) {
    launch_norm_quant(h_.as<float>(), I, n, I, nullptr, c.eps, nullptr, 0, xq, xs_.as<float>(), ldxs_, status(),
                      stream_);
  }
  run_proj_generic(L.parts[mlp + 2], h_.as<float>(), I, n, x, H, kEpiAdd);
}

void Engine::check_status() {
  DeviceStatus st{};
  DG_CUDA(cudaMemcpyAsync(&st, status_.ptr, sizeof(st), cudaMemcpyDeviceToHost, stream_));
  DG_CUDA(cudaStreamSynchronize(stream_));
  if (st.code == kNonFinite) throw DgError("non-finite Qwen hidden states");
  if (st.code == kWaitTimeout)
    throw DgError("device pipeline wait timed out (location " + std::to_string(st.where) + ")");
  if (st.code) throw DgError("device error code " + std::to_string(st.code));
}

void Engine::run_layers(int n, int start, const Prefix* past, Prefix* cap) {
  launch_embed(embedding_.ptr, 0, c_.hidden, ids_.as<uint32_t>(), n, x_.as<float>(), stream_);
  for (int i = 0; i < c_.layers; ++i) {
    const Prefix::LayerState* lp = past ? &past->layers[i] : nullptr;
    Prefix::LayerState* lc = cap ? &cap->layers[i] : nullptr;
    cur_layer_ = i;
    if (fast_)
      layer_fast(i, n, start, lp, lc);
    else
      layer_generic(i, n, start, lp, lc);
  }
  cur_layer_ = -1;
  launch_final_norm(x_.as<float>(), n, c_.hidden, final_norm_.as<float>(), c_.eps, status(), stream_);
}

void Engine::debug_layer(int layer, const float* x_in, int n, float* x_out) {
  if (!finalized_) throw DgError("engine is not finalized");
  if (layer < 0 || layer >= c_.layers) throw DgError("layer index out of range");
  if (n <= 0 || n > 4096) throw DgError("token sequence must contain 1\xe2\x80\x93" "4096 tokens");
  if (n > max_tokens_) throw DgError("token sequence exceeds the engine's max_tokens workspace");
  if (!x_in || !x_out) throw DgError("null argument");
  DG_CUDA(cudaSetDevice(device_));
  const uint64_t launches0 = launch_count();
  const size_t bytes = size_t(n) * c_.hidden * 4;
  DG_CUDA(cudaMemcpyAsync(x_.ptr, x_in, bytes, cudaMemcpyHostToDevice, stream_));
  DG_CUDA(cudaMemsetAsync(status_.ptr, 0, sizeof(DeviceStatus), stream_));
  gemm_ops_pending_.clear();
  fwd_ops_all_ = 0.0;
  fwd_proj_ = 0;
  DG_CUDA(cudaEventRecord(ev0_, stream_));
  cur_layer_ = layer;
  if (fast_)
    layer_fast(layer, n, 0, nullptr, nullptr);
  else
    layer_generic(layer, n, 0, nullptr, nullptr);
  cur_layer_ = -1;
  DG_CUDA(cudaEventRecord(ev1_, stream_));
  DG_CUDA(cudaMemcpyAsync(x_out, x_.ptr, bytes, cudaMemcpyDeviceToHost, stream_));
  check_status();
  DG_CUDA(cudaEventElapsedTime(&last_forward_ms, ev0_, ev1_));
  collect_gemm_timing();
  last_launches = int(launch_count() - launches0);
}

void Engine::dump_codes(int n, int K) {
  if (!dbg_codes_) return;
  DG_CUDA(cudaMemcpyAsync(dbg_codes_ + dbg_off_, xq_.ptr, size_t(n) * K, cudaMemcpyDeviceToHost, stream_));
  dbg_off_ += size_t(n) * K;
}

void Engine::debug_layer_codes(int layer, const float* x_in, int n, float* x_out, int8_t* codes) {
  if (!fast_) throw DgError("quantised codes are recorded on the int8-compute tcgen05 path only");
  if (!codes) throw DgError("null argument");
  dbg_codes_ = codes;
  dbg_off_ = 0;
  try {
    debug_layer(layer, x_in, n, x_out);
  } catch (...) {
    dbg_codes_ = nullptr;
    throw;
  }
  dbg_codes_ = nullptr;
}

void Engine::drop_graphs() {
  for (auto& kv : graphs_)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  graphs_.clear();
}

void Engine::forward(const uint32_t* ids, int n, const Prefix* past, bool capture, float* hidden_out,
                     std::unique_ptr<Prefix>* captured) {
  if (!finalized_) throw DgError("engine is not finalized");
  const int start = past ? past->len : 0;
  if (n <= 0 || start + n > 4096) throw DgError("token sequence must contain 1\xe2\x80\x93" "4096 tokens");
  if (n > max_tokens_) throw DgError("token sequence exceeds the engine's max_tokens workspace");
  for (int t = 0; t < n; ++t)
    if (ids[t] >= uint32_t(c_.vocab)) throw DgError("token " + std::to_string(ids[t]) + " outside vocabulary");
  if (past && int(past->layers.size()) != c_.layers) throw DgError("prefix cache does not match the layer types");
  if (past)
    for (int i = 0; i < c_.layers; ++i)
      if (past->layers[i].full != layers_[i].full) throw DgError("prefix cache does not match the layer types");
  DG_CUDA(cudaSetDevice(device_));
  const uint64_t launches0 = launch_count();
  std::unique_ptr<Prefix> cap;
  if (capture) {
    cap.reset(new Prefix());
    cap->len = start + n;
    cap->layers.resize(c_.layers);
  }
  DG_CUDA(cudaMemcpyAsync(ids_.ptr, ids, size_t(n) * 4, cudaMemcpyHostToDevice, stream_));
  DG_CUDA(cudaMemsetAsync(status_.ptr, 0, sizeof(DeviceStatus), stream_));
  gemm_ops_pending_.clear();
  fwd_ops_all_ = 0.0;
  fwd_proj_ = 0;
  DG_CUDA(cudaEventRecord(ev0_, stream_));
  if (!graphs_on_ || past || capture) {
    run_layers(n, start, past, cap.get());
  } else {
    FwdGraph& g = graphs_[4 * n + (gemm_ev_.empty() ? 0 : 2) + (exact ? 1 : 0)];
    if (g.exec) {
      DG_CUDA(cudaGraphLaunch(g.exec, stream_));
      gemm_ops_pending_ = g.gemm_ops;
      fwd_ops_all_ = g.ops_all;
      fwd_proj_ = g.proj;
      note_launches(g.launches);
    } else if (g.runs++ == 0) {
      run_layers(n, start, nullptr, nullptr);
    } else {
      const uint64_t l0 = launch_count();
      cudaGraph_t graph = nullptr;
      DG_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      try {
        run_layers(n, start, nullptr, nullptr);
      } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
      }
      DG_CUDA(cudaStreamEndCapture(stream_, &graph));
      const cudaError_t e = cudaGraphInstantiate(&g.exec, graph, 0);
      cudaGraphDestroy(graph);
      DG_CUDA(e);
      g.launches = launch_count() - l0;
      g.gemm_ops = gemm_ops_pending_;
      g.ops_all = fwd_ops_all_;
      g.proj = fwd_proj_;
      DG_CUDA(cudaGraphLaunch(g.exec, stream_));
    }
  }
  DG_CUDA(cudaEventRecord(ev1_, stream_));
  if (hidden_out)
    DG_CUDA(cudaMemcpyAsync(hidden_out, x_.ptr, size_t(n) * c_.hidden * 4, cudaMemcpyDeviceToHost, stream_));
  check_status();
  DG_CUDA(cudaEventElapsedTime(&last_forward_ms, ev0_, ev1_));
  collect_gemm_timing();
  last_launches = int(launch_count() - launches0);
  if (capture) *captured = std::move(cap);
}

bool Engine::segments_supported() const {
  return fast_ && c_.head_dim == 256 && c_.dk == 128 && c_.dv == 128 && (c_.kw() * 4) % 16 == 0;
}

void Engine::forward_segments(const uint32_t* ids, int seg_len, int segs, const Prefix* past, float* hidden_out) {
  if (!finalized_) throw DgError("engine is not finalized");
  if (!segments_supported()) throw DgError("segmented forwards need the 2B-shaped tcgen05 path");
  if (segs == 1) return forward(ids, seg_len, past, false, hidden_out, nullptr);
  const int start = past ? past->len : 0;
  if (seg_len <= 0 || segs <= 0 || start + seg_len > 4096)
    throw DgError("token sequence must contain 1\xe2\x80\x93" "4096 tokens");
  const int n = seg_len * segs;
  if (size_t(seg_len) * segs > size_t(max_tokens_)) throw DgError("token sequence exceeds the engine's max_tokens workspace");
  for (int t = 0; t < n; ++t)
    if (ids[t] >= uint32_t(c_.vocab)) throw DgError("token " + std::to_string(ids[t]) + " outside vocabulary");
  if (past && int(past->layers.size()) != c_.layers) throw DgError("prefix cache does not match the layer types");
  if (past)
    for (int i = 0; i < c_.layers; ++i)
      if (past->layers[i].full != layers_[i].full) throw DgError("prefix cache does not match the layer types");
  DG_CUDA(cudaSetDevice(device_));
  const size_t sbytes = size_t(c_.value_heads) * c_.dk * c_.dv * 4;
  if (seg_state_.bytes < sbytes * segs) seg_state_ = DevBuf(sbytes * segs);
  const uint64_t launches0 = launch_count();
  DG_CUDA(cudaMemcpyAsync(ids_.ptr, ids, size_t(n) * 4, cudaMemcpyHostToDevice, stream_));
  DG_CUDA(cudaMemsetAsync(status_.ptr, 0, sizeof(DeviceStatus), stream_));
  gemm_ops_pending_.clear();
  fwd_ops_all_ = 0.0;
  fwd_proj_ = 0;
  DG_CUDA(cudaEventRecord(ev0_, stream_));
  seg_len_ = seg_len;
  segs_ = segs;
  try {
    run_layers(n, start, past, nullptr);
  } catch (...) {
    seg_len_ = 0;
    segs_ = 1;
    throw;
  }
  seg_len_ = 0;
  segs_ = 1;
  DG_CUDA(cudaEventRecord(ev1_, stream_));
  if (hidden_out)
    DG_CUDA(cudaMemcpyAsync(hidden_out, x_.ptr, size_t(n) * c_.hidden * 4, cudaMemcpyDeviceToHost, stream_));
  check_status();
  DG_CUDA(cudaEventElapsedTime(&last_forward_ms, ev0_, ev1_));
  collect_gemm_timing();
  last_launches = int(launch_count() - launches0);
}

void Engine::head_logits(int rows, const size_t* positions, int n_pos, float* logits_out, int row_base) {
  if (c_.pointer_dim <= 0) throw DgError("engine has no pointer head");
  if (n_pos <= 0 || n_pos + 1 > 512) throw DgError("invalid encoding positions or window");
  std::vector<int> idx(n_pos + 1);
  idx[0] = row_base + rows - 1;
  for (int i = 0; i < n_pos; ++i) {
    if (positions[i] >= size_t(rows)) throw DgError("invalid encoding positions or window");
    idx[i + 1] = row_base + int(positions[i]);
  }
  const int H = c_.hidden, P = c_.pointer_dim;
  DG_CUDA(cudaMemcpyAsync(hrow_idx_.ptr, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice, stream_));
  launch_head_norm(x_.as<float>(), H, hrow_idx_.as<int>(), n_pos + 1, head_norm_w_.as<float>(),
                   head_norm_b_.as<float>(), hnorm_.as<float>(), stream_);
  // q = dot_scores(n, Wq[j]) (+ bq inside head_dot): the lane-ordered FP32
  // dot of the LoRA-A kernel, with coalesced weight reads.
  launch_lora_a(hnorm_.as<float>(), H, 1, H, head_q_.w_f32.as<float>(), P, hq_.as<float>(), P, true, stream_);
  launch_lora_a(hnorm_.as<float>() + H, H, n_pos, H, head_k_.w_f32.as<float>(), P, hk_.as<float>(), P, true, stream_);
  launch_head_dot(hq_.as<float>(), hk_.as<float>(), n_pos, P, 1.0f / std::sqrt(float(P)), head_q_.bias.as<float>(),
                  head_k_.bias.as<float>(), hlogits_.as<float>(), stream_);
  DG_CUDA(cudaMemcpyAsync(logits_out, hlogits_.ptr, size_t(n_pos) * 4, cudaMemcpyDeviceToHost, stream_));
  DG_CUDA(cudaStreamSynchronize(stream_));
}

}  // namespace dg
