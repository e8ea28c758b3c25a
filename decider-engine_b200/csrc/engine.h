// Device-resident Qwen3.5 decider torso + pointer head: the executor behind
// the C ABI. One engine = one GPU, one stream, weights resident in HBM.
//
// Replaces qwen::Model (src/qwen.rs:280-505) and Head (src/lib.rs:87-131).
#pragma once
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "gemm_i8.cuh"
#include "launch.h"

namespace dg {

enum Precision { kCheckpoint = 0, kInt8 = 1, kInt8Compute = 2, kInt4 = 3 };

struct Config {
  int hidden = 0, intermediate = 0, layers = 0, vocab = 0, heads = 0, kv_heads = 0, head_dim = 0;
  int conv_kernel = 0, dk = 0, dv = 0, key_heads = 0, value_heads = 0;
  float eps = 1e-6f, rope_theta = 1e7f, partial_rotary = 0.25f;
  std::vector<int> layer_types;  // 1 = full_attention, 0 = linear_attention
  int rank = 0;
  float lora_scale = 0.0f;
  int pointer_dim = 0;           // 0: no pointer head
  int rotary_dim() const { return int(float(head_dim) * partial_rotary); }
  int kd() const { return key_heads * dk; }
  int vd() const { return value_heads * dv; }
  int conv_width() const { return 2 * kd() + vd(); }
  int qw() const { return heads * head_dim; }
  int kw() const { return kv_heads * head_dim; }
  void validate() const;
};

// Device buffer with RAII.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool pooled = false;  // from the device's stream-ordered pool (cudaMallocAsync)
  int device = -1;      // the pool's device (pooled buffers)
  bool borrowed = false;  // a view of another buffer's memory: never freed through this one
  DevBuf() = default;
  // A non-owning view of o's memory (weights shared between engines).
  static DevBuf view_of(const DevBuf& o) {
    DevBuf b;
    b.ptr = o.ptr;
    b.bytes = o.bytes;
    b.borrowed = o.ptr != nullptr;
    return b;
  }
  explicit DevBuf(size_t n);
  // Stream-ordered allocation from the device's default memory pool, for
  // buffers made and dropped per request (prefix caches): no device-wide
  // synchronisation on free, and the pool keeps released memory for reuse.
  static DevBuf pooled_on(size_t n, cudaStream_t s);
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept
      : ptr(o.ptr), bytes(o.bytes), pooled(o.pooled), device(o.device), borrowed(o.borrowed) {
    o.ptr = nullptr;
    o.bytes = 0;
    o.pooled = false;
    o.borrowed = false;
  }
  DevBuf& operator=(DevBuf&& o) noexcept;
  ~DevBuf();
  template <class T> T* as() const { return static_cast<T*>(ptr); }
};

// Host-side staged tensor (FP32, or already quantized projection weights).
// A staged checkpoint tensor, F32 on the host. `quantized` marks a
// projection that read_tensors quantises (src/weights.rs:346-355): it is
// quantised on the device (quantize_weights_device, Data::quantize) when
// its projection is built, straight into the projection's layout.
struct HostTensor {
  std::vector<int64_t> shape;
  std::vector<float> f32;
  bool quantized = false;
  int bits = 0;  // 8 or 4 when quantized
};

// One (possibly fused) projection on the device.
struct DevProj {
  int in = 0, out = 0, out_pad = 0;
  // tcgen05 path (int8-compute, aligned shapes)
  DevBuf wq, ws_t, lora_a, lora_b, chunk_pid;
  WeightMaps maps{};
  int lora_rows = 0;           // rows of lora_a (= projections sharing the input x rank)
  std::vector<int> part_off;     // output column of each fused part
  // generic path
  GenericProj g{};
  DevBuf w_f32, scale_rows, bias;
};

struct Layer {
  bool full = false;
  DevBuf input_norm, post_norm;
  // fast path: fused input projection and single output projection
  DevProj in_proj, out_proj, mlp_in, down;
  // generic path: separate projections in reference order
  std::vector<DevProj> parts;    // DeltaNet: qkv,z,a,b,out ; attention: q,k,v,o ; then gate,up,down
  DevBuf q_norm, k_norm;          // attention
  DevBuf conv, dt, decay_rate, norm;  // DeltaNet (conv tap-major)
};

struct Prefix {
  int len = 0;
  struct LayerState {
    bool full = false;
    DevBuf k, v;          // [len][kw]
    DevBuf tail, state;   // [rows][W], [H][dk][dv]
    int tail_rows = 0;
  };
  std::vector<LayerState> layers;
};

class Engine {
 public:
  Engine(const Config& c, int precision, int device, int max_tokens);
  ~Engine();
  void set_tensor(const std::string& name, int dtype, const std::vector<int64_t>& shape, const void* data);
  void fill_synthetic(uint64_t seed, float stddev);
  void finalize();
  // Instead of staging and finalize: use the weights of `base` (a finalized
  // engine on the same device, same model, precision and token budget) as
  // read-only views. Stream, workspaces, CUDA graphs and prefixes stay this
  // engine's own, so engines that share weights can run forwards
  // concurrently from different host threads. The caller keeps `base`
  // alive while this engine lives.
  void share_weights(const Engine& base);
  // Model::run: hidden [n][hidden] to host (nullable); capture -> new prefix.
  void forward(const uint32_t* ids, int n, const Prefix* past, bool capture, float* hidden_out,
               std::unique_ptr<Prefix>* captured);
  // Model::forward_after for `segs` sequences of seg_len tokens each (ids
  // concatenated), every one continuing `past` (or starting at position 0
  // when past is null): the questions of one request as ONE pass over
  // segs * seg_len rows. Projections, norms and the MLP run once over all
  // rows; RoPE positions, the attention (the prefix's keys plus each
  // sequence's own), the conv (the prefix's tail) and the recurrence (a copy
  // of the prefix state per sequence) keep the sequences apart. In reference
  // order each sequence's rows equal those of forward(its ids, past) bit for
  // bit. hidden_out (nullable) receives [segs * seg_len][hidden]; the rows
  // stay on the device for head_logits with row_base = sequence * seg_len.
  void forward_segments(const uint32_t* ids, int seg_len, int segs, const Prefix* past, float* hidden_out);
  // Segmented forwards need the head_dim-256 attention and dk = dv = 128
  // recurrence kernels (the 2B shape) on the tcgen05 path.
  bool segments_supported() const;
  // Head::logits on the last forward's hidden rows (device-resident):
  // the answer is row row_base + rows - 1, the options rows row_base + positions.
  void head_logits(int rows, const size_t* positions, int n_pos, float* logits_out, int row_base = 0);
  // One decoder layer, teacher-forced: residual rows x_in [n][hidden] (host)
  // at positions 0..n-1 with no prefix -> the layer's output rows (host).
  void debug_layer(int layer, const float* x_in, int n, float* x_out);
  // debug_layer, also copying the int8 codes of the layer's four quantised
  // projection inputs to codes (host, n * (hidden + mixer width + hidden +
  // intermediate) bytes: input norm, mixer output, post norm, SwiGLU rows).
  // int8-compute on the tcgen05 path only.
  void debug_layer_codes(int layer, const float* x_in, int n, float* x_out, int8_t* codes);
  const Config& config() const { return c_; }
  int max_tokens() const { return max_tokens_; }
  // dg_logits_batch runs the equal-length questions of a request as one
  // segmented forward (DG_BATCH_QUESTIONS=0: one forward per question).
  bool batch_questions = true;
  bool fast_path() const { return fast_; }
  int device() const { return device_; }
  int precision() const { return precision_; }
  cudaStream_t stream() const { return stream_; }
  std::mutex mu;
  // Exact FP32 promotion order in the tcgen05 projections (reference order).
  bool exact = true;
  // The chunked DeltaNet scan in 32-column slices (half the CTAs): set for
  // engines that serve batch lanes, where other lanes use the free SMs.
  bool wide_scan = false;
  // Device launches issued by the last forward (kernels only).
  int last_launches = 0;
  // Device time of the last forward's kernels (after the id upload, before
  // the hidden-state download), from CUDA events on the engine stream.
  float last_forward_ms = 0.0f;

 private:
  struct Expected {
    std::vector<int64_t> shape;
    bool projection;
  };
  std::map<std::string, Expected> expected_names() const;
  void stage(const std::string& name, std::vector<int64_t> shape, std::vector<float>&& f32);
  HostTensor take(const std::string& name);
  DevBuf upload_f32(const std::vector<float>& v);
  void build_fast_layer(int i, Layer& L);
  void build_generic_layer(int i, Layer& L);
  DevProj build_generic_proj(const std::string& key, int in, int out, bool lora, bool bias);
  DevProj build_fused(const std::vector<std::string>& keys, const std::vector<int>& outs, int in, bool interleave_mlp);
  void run_proj_fast(const DevProj& p, int M, const float* mid, float* out, int ldo, int epi);
  void run_proj_generic(const DevProj& p, const float* x, int ldx, int M, float* out, int ldo, int epi);
  void layer_fast(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap);
  void layer_generic(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap);
  void mixer_tail(int i, int n, int start, const Prefix::LayerState* past, Prefix::LayerState* cap,
                  const float* raw, int ldr);
  void check_status();
  // The forward's device buffers, sized for max_tokens_ rows (ld_proj: the
  // widest fused input projection).
  void alloc_workspaces(int ld_proj);
  // Debug copy of the quantised activations (xq_) after each quantisation of
  // a debug_layer_codes call; a no-op otherwise.
  int8_t* dbg_codes_ = nullptr;
  size_t dbg_off_ = 0;
  void dump_codes(int n, int K);
  void run_layers(int n, int start, const Prefix* past, Prefix* cap);
  // The kernels of a forward without a prefix (no past, no capture) as one
  // CUDA graph per token count and timing mode: the first such forward runs
  // eagerly (first-use set-up stays outside any capture), the second is
  // captured, later ones replay the graph.
  struct FwdGraph {
    int runs = 0;
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;
    std::vector<double> gemm_ops;
    double ops_all = 0.0;
    uint64_t proj = 0;
  };
  std::map<int, FwdGraph> graphs_;
  bool graphs_on_ = true;
  // Projections wait for their LoRA-A kernels only before the epilogue
  // (GemmArgs::late_dep), so their main loop overlaps LoRA-A; DG_LORA_OVERLAP=0
  // serialises them again.
  bool lora_overlap_ = true;
  void drop_graphs();

  Config c_;
  int precision_, device_, max_tokens_;
  bool fast_ = false, finalized_ = false;
  cudaStream_t stream_ = nullptr;
  bool pool_held_ = false;  // this engine counts as a user of the device's prefix pool settings
  std::map<std::string, HostTensor> staged_;
  std::vector<Layer> layers_;
  DevBuf embedding_, final_norm_, rope_;
  int rope_half_ = 0;
  // pointer head
  DevBuf head_norm_w_, head_norm_b_;
  DevProj head_q_, head_k_;
  // workspace
  int ldxs_ = 0, ld_proj_ = 0;
  DevBuf ids_, x_, n_, xq_, xs_, mid_, proj_, conv_, decay_, beta_, o_, ofin_, h_, qbuf_, att_;
  DevBuf hrows_, hnorm_, hq_, hk_, hlogits_, hrow_idx_;
  std::vector<DevBuf> kcache_, vcache_, state_;
  DevBuf delta_ws_;  // chunked DeltaNet products (fast mode)
  // Segmented forwards (forward_segments): sequence length and count of the
  // running pass (0 / 1 otherwise), the sequences' own K/V rows and one
  // recurrent state per sequence.
  int seg_len_ = 0, segs_ = 1;
  DevBuf kseg_, vseg_, seg_state_;
  // Fast-mode attention on the tensor cores (scores and Vᵀ workspace);
  // DG_ATTN_TC=0 keeps the CUDA-core kernel.
  DevBuf attn_ws_;
  bool attn_tc_ = true;
  DevBuf lora_part_; // split-K LoRA-A partial sums (fast mode)
  DevBuf tc_prod_;   // FP32-weight projections on the tensor cores: the product before the SwiGLU
  DevBuf gemm_split_ws_, gemm_split_cnt_;  // split-K projection partials and tile counters (fast mode)
  DevBuf status_;
  cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
  DeviceStatus* status() const { return status_.as<DeviceStatus>(); }
  // Optional timing of every tcgen05 projection launch (event pairs on the
  // engine stream), read back after each forward.
  std::vector<cudaEvent_t> gemm_ev_;
  std::vector<double> gemm_ops_pending_;
  int gemm_lo_ = 0, gemm_hi_ = 1 << 30, cur_layer_ = -1;
  double fwd_ops_all_ = 0.0;  // projection ops of the current forward
  uint64_t fwd_proj_ = 0;     // projection launches of the current forward
  void collect_gemm_timing();

 public:
  struct GemmTiming {
    double ms = 0.0, ops = 0.0;  // timed launches: summed time and algorithmic ops (2*M*N*K)
    uint64_t launches = 0;
    double ops_all = 0.0;        // every projection launch of the timed forwards
    uint64_t launches_all = 0;
  } gemm_timing;
  // Times the projections of layers [first_layer, first_layer + layers) only.
  void set_gemm_timing(bool on, int first_layer = 0, int layers = 1 << 30);
};

// While any engine lives on a device, that device's default stream-ordered
// pool keeps up to 4 GiB of released prefix blocks; the last engine restores
// the pool's release threshold and trims it.
void prefix_pool_acquire(int device);
void prefix_pool_release(int device);

// LoadLimits (src/loading.rs:8-24): allocation budgets checked before any
// payload is read or any memory taken. Defaults: 2 GiB per tensor, 12 GiB of
// weights and conversion scratch, 2 GiB of forward workspace.
struct LoadLimits {
  uint64_t max_tensor_bytes = uint64_t(2) << 30;
  uint64_t max_weight_bytes = uint64_t(12) << 30;
  uint64_t max_workspace_bytes = uint64_t(2) << 30;
};

// Checkpoint directory in the reference's layout (loader.cu): the validated
// model config (rank, LoRA scale, pointer dim included; max_length of the
// decision window when max_length_out is given), the architecture's budget
// check (Config::validate_layout), and the tensors of the safetensors files
// charged to a budget and streamed into an engine.
void read_checkpoint_config(const std::string& dir, Config& c, int& pointer_dim, int* max_length_out = nullptr);
void validate_layout(const Config& c, int tokens, int rank, int pointer, const LoadLimits& limits);
void ensure_checkpoint_budget(const std::string& dir, const LoadLimits& limits);
void load_checkpoint_tensors(Engine& e, const std::string& dir, const LoadLimits& limits = LoadLimits());

}  // namespace dg
