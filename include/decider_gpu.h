/*
 * decider_gpu.h — C ABI of the B200 (sm_100a) prefill engine for the Strands
 * Decider 2B classifier. Drop-in device backend for decider-engine's model
 * seam: qwen::Model (load / forward / prefill / forward_after,
 * src/qwen.rs:291-424) and Head::logits (src/lib.rs:116-131). Host logic
 * (prompting, tokenizer, limits, schema, readout) stays with the caller.
 *
 * Conventions: every function returns 0 on success or a nonzero status, with
 * the message in dg_last_error() (thread-local). All pointers are HOST
 * pointers unless a name says `_device`; callers own every buffer they pass.
 * No call keeps a pointer to caller memory after it returns.
 */
#ifndef DECIDER_GPU_H
#define DECIDER_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct dg_engine dg_engine;
typedef struct dg_prefix dg_prefix;
typedef struct dg_linear dg_linear;

/* Precision switch, Precision (src/lib.rs:48-66). */
enum { DG_CHECKPOINT = 0, DG_INT8 = 1, DG_INT8_COMPUTE = 2, DG_INT4 = 3 };
/* Tensor dtypes accepted by dg_engine_set_tensor (safetensors F32/BF16/F16,
 * Data::read, src/weights.rs:147-194). */
enum { DG_F32 = 0, DG_BF16 = 1, DG_F16 = 2 };

/* Qwen3.5 text_config fields read by the forward pass (Config,
 * src/qwen.rs:8-34), the LoRA rank and alpha/r scale (src/lib.rs:300-358) and
 * the pointer-head width (src/lib.rs:72-86; 0 = no head). */
typedef struct dg_model_config {
  int32_t hidden_size, intermediate_size, num_hidden_layers, vocab_size;
  int32_t num_attention_heads, num_key_value_heads, head_dim;
  int32_t linear_conv_kernel_dim, linear_key_head_dim, linear_value_head_dim;
  int32_t linear_num_key_heads, linear_num_value_heads;
  float rms_norm_eps, rope_theta, partial_rotary_factor;
  const int32_t* layer_types; /* num_hidden_layers entries: 1 full_attention, 0 linear_attention */
  int32_t lora_rank;
  float lora_scale;
  int32_t pointer_dim;
} dg_model_config;

/* Last error message of this thread ("" if none). */
const char* dg_last_error(void);
/* Number of kernel launches this library has issued in this process. */
uint64_t dg_launch_count(void);

/* ---- engine lifecycle: replaces Model::load + Head::load
 * (src/qwen.rs:291-406, src/lib.rs:94-105). Tensors use the checkpoint names
 * without the "model.language_model." prefix; adapter tensors keep
 * "base_model.model."; pointer-head tensors are "head.<name>". Projection
 * weights ("layers.*_proj.weight") are quantised per `precision` exactly as
 * Data::quantize (src/weights.rs:98-146), on the device when the engine is
 * finalized. max_tokens bounds the rows of one forward call (1..4096). */
int dg_engine_create(const dg_model_config* cfg, int precision, int device, int max_tokens, dg_engine** out);
int dg_engine_set_tensor(dg_engine* e, const char* name, int dtype, const int64_t* shape, int ndim,
                         const void* data);
/* Fills every tensor not yet set with seeded N(0, stddev^2) values (norm
 * weights 1, biases 0): synthetic checkpoints of a given architecture. */
int dg_engine_fill_synthetic(dg_engine* e, uint64_t seed, float stddev);
int dg_engine_finalize(dg_engine* e);
/* A second engine on the base's device that reads the base's weights
 * (finalized, read-only; no copy) and has its own stream, forward buffers,
 * CUDA graphs and prefixes; it starts in the base's arithmetic mode. Engines that share weights may run forward,
 * logits and batch calls concurrently from different host threads (one call
 * at a time per engine): on one GPU, two or three request streams overlap
 * each other's latency-bound kernels. A prefix belongs to the engine that
 * made it. The weights stay alive until the base and every sibling have
 * been freed, in any order. No counterpart in the reference, whose engine
 * serves one forward at a time. */
int dg_engine_create_sibling(dg_engine* base, dg_engine** out);
/* 1 when the tcgen05 INT8 path serves the projections, 0 for the generic kernels. */
int dg_engine_fast_path(const dg_engine* e);
/* 1 (default): every FP32 sum in the reference's order (the tcgen05 INT8
 * promotion in group order, the other precisions' projections in dot_scores
 * lane order, the token recurrence, the CUDA-core attention). 0: the fast
 * mode: fused multiply-adds in the promotion, the chunked delta rule,
 * attention and LoRA products on the tensor cores (3 x TF32), and the
 * weight-only precisions' projections on the tensor cores. */
int dg_engine_set_exact(dg_engine* e, int exact);
void dg_engine_free(dg_engine* e);
/* Model::load + Head::load from a checkpoint directory in the reference's
 * layout (src/lib.rs:287-367): validates strands_decider_config.json (or
 * hobson_config.json, src/lib.rs:188-222), base/config.json's text_config
 * (src/qwen.rs:133-188) and lora/adapter_config.json (src/lib.rs:300-358),
 * then streams base/model.safetensors (without its "model.language_model."
 * prefix), lora/adapter_model.safetensors and head.safetensors (prefixed
 * "head.") into a new engine and finalizes it. Equivalent to
 * dg_engine_create + dg_engine_set_tensor for every tensor + dg_engine_finalize. */
int dg_engine_load(const char* dir, int precision, int device, int max_tokens, dg_engine** out);
/* LoadLimits (src/loading.rs:8-24): allocation budgets, in bytes, checked at
 * the checkpoint boundary before any payload is read or any device memory is
 * taken. Defaults (dg_load_limits_default): 2 GiB per tensor, 12 GiB of
 * weights and conversion scratch, 2 GiB of forward workspace. */
typedef struct dg_load_limits {
  uint64_t max_tensor_bytes;
  uint64_t max_weight_bytes;
  uint64_t max_workspace_bytes;
} dg_load_limits;
void dg_load_limits_default(dg_load_limits* out);
/* NativeEngine::load_with_limits (src/lib.rs:287-367): dg_engine_load with
 * explicit budgets (limits NULL: the defaults). Before the engine is created
 * it runs the reference's checks in its order: Config::validate_layout
 * (src/qwen.rs:37-135: the architecture's FP32 weight estimate, LoRA
 * included, and the forward workspace for max_length tokens), then
 * WeightBudget::charge (src/loading.rs:61-80) of every tensor in the adapter,
 * head and base files (base: model.safetensors, or the shards of
 * model.safetensors.index.json) from their headers. Over-budget checkpoints
 * fail with the reference's messages ("{name}: allocation of {bytes} bytes
 * exceeds budget {limit}", "{name}: dimension product overflow"), with no
 * device memory taken. dg_engine_load is this call with the defaults. */
int dg_engine_load_with_limits(const char* dir, int precision, const dg_load_limits* limits, int device,
                               int max_tokens, dg_engine** out);
/* The validated model config of a checkpoint directory (no device needed):
 * fills *cfg, with cfg->layer_types pointing at the caller's buffer of
 * max_layers entries (0 DeltaNet, 1 attention). */
int dg_read_checkpoint_config(const char* dir, dg_model_config* cfg, int32_t* layer_types, int max_layers);
/* The engine's CUDA stream (cudaStream_t) for callers that time or order work. */
void* dg_engine_stream(const dg_engine* e);
/* Device time (ms) of the last forward's kernels, between the id upload and
 * the result download; and the number of kernels that forward launched. */
float dg_engine_last_forward_ms(const dg_engine* e);
int dg_engine_last_launches(const dg_engine* e);
/* Measurement aid (no counterpart in the reference): with timing enabled,
 * every tcgen05 projection launch of a forward is bracketed by CUDA events on
 * the engine stream; dg_engine_gemm_time returns the summed launch time (ms),
 * the summed algorithmic ops (2*M*N*K) and the launch count since the last
 * dg_engine_gemm_timing call, which also resets them. */
int dg_engine_gemm_timing(dg_engine* e, int enable);
int dg_engine_gemm_time(const dg_engine* e, double* ms, double* ops, uint64_t* launches);
/* As dg_engine_gemm_timing(e, 1), but only the projections of layers
 * [first_layer, first_layer + layers) get events (a sample that perturbs the
 * forward less); dg_engine_gemm_time_all returns the algorithmic ops and launch
 * count of every projection of the timed forwards, sampled or not. */
int dg_engine_gemm_timing_layers(dg_engine* e, int first_layer, int layers);
int dg_engine_gemm_time_all(const dg_engine* e, double* ops_all, uint64_t* launches_all);

/* Measurement aid (no counterpart in the reference): the dense INT8
 * tensor-core rate of `device` in TOP/s, from a timed launch of one CTA per SM
 * issuing `iters` x 4 back-to-back tcgen05.mma.kind::i8 of 128 x 256 x 32
 * (iters 1..4194304; ~2^16 runs for about 10 ms); ms_out (nullable) gets the
 * launch's duration. */
int dg_measure_i8_peak(int device, int iters, double* tops_out, float* ms_out);

/* ---- forward passes: Model::forward / prefill / forward_after
 * (src/qwen.rs:407-424). `past` may be NULL. hidden_out (nullable) receives
 * [n][hidden_size] FP32. Errors mirror the reference's messages:
 * "token sequence must contain 1–4096 tokens", "token {id} outside
 * vocabulary", "non-finite Qwen hidden states", "prefix cache does not match
 * the layer types". */
int dg_forward_hidden(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t n, float* hidden_out);
int dg_prefill(dg_engine* e, const uint32_t* ids, size_t n, dg_prefix** out);
/* One decoder layer teacher-forced, for per-layer parity: the body of the
 * layer loop of Model::run (src/qwen.rs:470-494: input norm, Full::forward or
 * Delta::forward, residual_norm, SwiGLU MLP with the residual add) applied
 * to the caller's residual rows x_in [n][hidden_size] at positions 0..n-1
 * with no prefix; x_out receives the layer's output rows [n][hidden_size].
 * Runs in the engine's current arithmetic mode. */
int dg_debug_layer(dg_engine* e, int layer, const float* x_in, size_t n, float* x_out);
/* dg_debug_layer, also returning the int8 codes of the layer's four quantised
 * projection inputs (QuantizedInputs::new, src/tensor.rs:315-353), for the
 * per-layer parity protocol's check of which rows flipped a code: codes_out
 * receives n x (hidden_size + mixer width + hidden_size + intermediate_size)
 * bytes, the blocks [n][hidden] of the normalised input rows (q/k/v or
 * qkv/z/a/b), [n][mixer width] of the mixer output (o_proj or out_proj input;
 * heads x head_dim or DeltaNet value heads x value dim), [n][hidden] of the
 * normalised post-mixer rows (gate/up) and [n][intermediate] of the SwiGLU
 * rows (down_proj). int8-compute engines on the tcgen05 path only. */
int dg_debug_layer_codes(dg_engine* e, int layer, const float* x_in, size_t n, float* x_out, int8_t* codes_out);
/* Model::forward_after for `segs` sequences of seg_len tokens each, ids
 * concatenated ([segs][seg_len]), every one continuing `past` (nullable: from
 * position 0), run as ONE forward over segs * seg_len rows (the questions of
 * one request; dg_logits_batch uses it for equal-length questions). Each
 * sequence's hidden rows equal those of dg_forward_hidden(past, its ids) (bit
 * for bit in reference order); hidden_out (nullable) receives
 * [segs * seg_len][hidden_size]. Needs the 2B-shaped int8-compute path
 * (head_dim 256, DeltaNet heads of 128) and segs * seg_len <= max_tokens. */
int dg_forward_segments_hidden(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t seg_len, size_t segs,
                               float* hidden_out);
size_t dg_prefix_len(const dg_prefix* p);
void dg_prefix_free(dg_prefix* p);

/* ---- pointer logits: NativeEngine::logits (src/lib.rs:400-419) =
 * forward(_after) + Head::logits. opt_pos are positions inside `ids` (already
 * relative to the prefix when `past` is given); logits_out has n_opt floats.
 * The answer row is the last token. */
int dg_logits(dg_engine* e, const dg_prefix* past, const uint32_t* ids, size_t n, const size_t* opt_pos,
              size_t n_opt, float* logits_out);

/* ---- batched requests: the throughput form of NativeEngine::evaluate
 * (src/lib.rs:477-559), which prefills a request's state once
 * (src/lib.rs:515-522, Model::prefill src/qwen.rs:413) and reads every
 * question of the request after it (Model::forward_after src/qwen.rs:422 +
 * Head::logits src/lib.rs:116-131). One request:
 *   past        nullable: an existing prefix (dg_prefill) the questions continue;
 *   state_ids   n_state tokens prefilled once and shared by the questions
 *               (n_state 0: none; not combined with `past`);
 *   questions   each a token sequence after the state with its option
 *               positions (relative to the question's own ids).
 * A request with neither past nor state and one question is one plain
 * forward. logits_out receives the n_opt logits of every question of every
 * request, concatenated in order. status_out (nullable, [n_requests]) gets
 * 0 or 1 per request and request_ms (nullable) the device time of that
 * request's forwards; a failed request's logits are unspecified and the
 * batch continues with the next request. Returns 0 when every request
 * succeeded, otherwise 1 with dg_last_error() holding the first failure's
 * message (in request order). With one lane (the default) the requests run
 * in order on the engine's stream; with dg_engine_set_lanes(e, k) they are
 * dealt to k lanes (the engine and k - 1 engines sharing its weights,
 * longest processing time first; a request that continues a prefix stays on
 * the engine that made it), each lane running its share in order from its
 * own host thread, so their kernels overlap on the device. Results do not
 * depend on the lane a request ran on. To spread a batch over several GPUs,
 * give each device's engine its share (one host thread or process per GPU). */
/* Lanes of dg_logits_batch (1 to 8; 1 = the engine alone). Each extra lane
 * is an engine on the same device reading this engine's weights (see
 * dg_engine_create_sibling) with its own stream and forward buffers (about
 * 1.2 GB at max_tokens 4096 for the 2B model). dg_engine_set_exact applies
 * to every lane. Set the lanes between calls: not while another thread runs
 * a call on this engine. */
int dg_engine_set_lanes(dg_engine* e, int lanes);
int dg_engine_lanes(const dg_engine* e);
/* Device time of the last dg_logits_batch call from its first kernel to the
 * end of its last lane (CUDA events; host gaps between requests included). */
float dg_engine_last_batch_ms(const dg_engine* e);
typedef struct dg_question {
  const uint32_t* ids;
  size_t n;
  const size_t* opt_pos;
  size_t n_opt;
} dg_question;
typedef struct dg_request {
  const dg_prefix* past;
  const uint32_t* state_ids;
  size_t n_state;
  const dg_question* questions;
  size_t n_questions;
} dg_request;
int dg_logits_batch(dg_engine* e, const dg_request* requests, size_t n_requests, float* logits_out, int* status_out,
                    float* request_ms);

/* ---- isolated INT8 projection: the reference's
 * linear_int8 + Adapter::combine (src/tensor.rs:379-456,109-117) with
 * load-time weight quantisation (src/weights.rs:98-146). w: [n][k] FP32;
 * lora_a [rank][k], lora_b [n][rank] (nullable when rank == 0; rank 0 or 32);
 * k % 128 == 0. */
int dg_linear_create(const float* w, int n, int k, const float* lora_a, const float* lora_b, int rank,
                     float lora_scale, int device, dg_linear** out);
/* y[m][n] = projection of x[m][k] (host buffers; copies inside). */
int dg_linear_forward(dg_linear* l, const float* x, int m, float* y);
/* Same on device buffers; group_dots_device (nullable) receives the exact
 * int32 group dots [k/64][m][n] the tensor cores produced. */
int dg_linear_forward_device(dg_linear* l, const float* x_device, int m, float* y_device, int32_t* group_dots_device);
/* Allocation-free form of dg_linear_forward_device (no counterpart in the
 * reference, whose projection is CPU code). For hosts that must not allocate
 * device memory while serving a request: those that reserve their whole
 * device-memory budget at start-up, where an allocation in mid-request can
 * fail under memory pressure, and latency-bound callers for which
 * cudaMalloc/cudaFree cost too much (cudaFree waits for the device). Same
 * kernels and results as dg_linear_forward_device without the group-dot dump;
 * its scratch is one fixed 8 MiB area of static device memory per device, so
 * it allocates nothing. Limits and rules:
 *  - m rows must fit that area: about m*k + m*(k/16 + 128) bytes, plus
 *    m*n_pad*4 when n % 256 != 0; larger calls fail with an error naming the
 *    bytes needed (split the rows over several calls);
 *  - the first call on each device resolves the area's address (with that
 *    device current); make that first call before beginning any stream
 *    capture; the address is kept for the process, so do not use this call
 *    across a cudaDeviceReset of that device;
 *  - calls on one device share the area, so they must not overlap in time,
 *    from several threads or several handles alike: serialise them.
 * Runs on, and synchronises, the handle's stream (dg_linear_stream). */
int dg_linear_forward_device_noalloc(dg_linear* l, const float* x_device, int m, float* y_device);
/* Quantised activations of the last call: xq [m][k] int8 and scales [k/64][m] (host). */
int dg_linear_last_quantized(dg_linear* l, int m, int8_t* xq, float* xs);
int dg_linear_set_exact(dg_linear* l, int exact);
/* Failure-path test aid with no counterpart in the reference: with
 * skip_group >= 0 (0 .. k/64 - 1), the handle's next projection launches
 * leave out the tensor cores' completion signal of that 64-wide K group and
 * bound every pipeline wait by wait_ns (1 ns .. 1 s) instead of 2 s, so the
 * wait for the group runs out: the kernel records the timeout in its status
 * word, lets its copies in flight land, frees its tensor memory and returns,
 * and the call fails with "device pipeline wait timed out" and the wait's
 * location. skip_group < 0 restores normal launches. */
int dg_linear_test_wait_fault(dg_linear* l, int skip_group, uint64_t wait_ns);
/* The CUDA stream the projection runs on (cudaStream_t). */
void* dg_linear_stream(const dg_linear* l);
/* Device time of the last dg_linear_forward / dg_linear_forward_device call,
 * from CUDA events on the handle's stream, in milliseconds: total_ms from the
 * activation quantiser to the end of the projection kernel, gemm_ms the
 * projection kernel alone (either pointer nullable). A measurement aid with
 * no counterpart in the reference. */
int dg_linear_last_times(const dg_linear* l, float* total_ms, float* gemm_ms);
void dg_linear_free(dg_linear* l);

/* ---- isolated gated delta rule: Recurrence::head's
 * state update (src/qwen.rs:846-866) for `batch` sequences x `heads` heads of
 * `t` tokens, dk = dv = 128, q and k already L2-normalised (q also scaled by
 * 1/sqrt(dk)). Device buffers: q, k, v [batch][t][heads][128]; g, beta
 * [batch][t][heads] with decay = exp(g); state [batch][heads][128][128] is
 * read as the initial state and left as the final one; o receives q^T S. */
int dg_gated_delta_rule_device(const float* q, const float* k, const float* v, const float* g, const float* beta,
                               int batch, int t, int heads, float* state, float* o, void* stream);
/* The same rule in its chunked form (64-token chunks: intra-chunk products in
 * parallel, one sequential pass over chunks). `workspace` is a device buffer
 * of at least dg_gated_delta_chunk_workspace_bytes(batch, t, heads) bytes,
 * owned by the caller. */
size_t dg_gated_delta_chunk_workspace_bytes(int batch, int t, int heads);
int dg_gated_delta_rule_chunked_device(const float* q, const float* k, const float* v, const float* g,
                                       const float* beta, int batch, int t, int heads, float* state, float* o,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* ---- weight quantisation on the device: Data::quantize
 * (src/weights.rs:98-146), which the reference runs on the host while
 * read_tensors loads a projection (src/weights.rs:346-355); the engine runs
 * it on the device as it builds each projection. Device buffers: w [rows]
 * [width] F32; bits 8: values [rows][width] (one int8 code per byte), bits 4:
 * ceil(rows * width / 2) bytes (value i in the low nibble of byte i / 2 when
 * i is even, the high nibble when odd, as code + 8); scales [rows]
 * [ceil(width / 64)]. Per group of 64: scale = max |w| / bound (127 or 7),
 * at least FLT_MIN, 1 for an all-zero group; code = clamp(round(w / scale)).
 * Bit for bit the reference's values. Runs on `stream` and synchronises it;
 * bits other than 4 / 8 or width 0 is an error. */
int dg_quantize_weights_device(const float* w, size_t rows, size_t width, int bits, uint8_t* values, float* scales,
                               void* stream);

/* ---- isolated gated causal attention (causal_attention and the output
 * gate of Full::forward, src/qwen.rs:581-643), a measurement and test entry
 * with no counterpart in the reference's API. Device buffers: q [n][heads][d]
 * (normalised, rotated), kc / vc [offset + n][kv_heads * d] (the prefix's
 * keys then the rows' own), gate rows of ld_gate floats with head h's gate at
 * column h * 2d + d; out [n][heads][d]. tensor_cores = 1: the fast-mode
 * tensor-core path (3 x TF32 tcgen05 products, head_dim 256; workspace of
 * dg_attention_workspace_bytes, owned by the caller); 0: the CUDA-core kernel
 * of reference-order mode (workspace unused). Runs on `stream` (a
 * cudaStream_t, NULL for the default stream) and synchronises it. */
size_t dg_attention_workspace_bytes(int heads, int kv_heads, int d, int n);
int dg_attention_device(const float* q, const float* kc, const float* vc, const float* gate, int ld_gate, int n,
                        int offset, int heads, int kv_heads, int d, float* out, int tensor_cores, void* workspace,
                        size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DECIDER_GPU_H */
