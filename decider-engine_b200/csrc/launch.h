// Host-side launchers of the decider GPU kernels (all on the given stream).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace dg {

struct GemmArgs;

// ---- tensor maps (driver entry point resolved at run time; no -lcuda)
void make_tmap_i8_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint32_t box_inner, uint32_t box_outer);

// ---- INT8 tensor-core projection (tcgen05), gemm_i8.cu
// Tensor maps of one int8 weight matrix [n][k] for each output-tile width.
// lb: the LoRA-B rows [n][32] (rank 32), read by the tensor-core LoRA path.
struct WeightMaps {
  CUtensorMap bn128{}, bn64{}, lb{};
  bool has_lb = false;
};
void make_weight_maps(WeightMaps* maps, const void* wq, int k, int n, const float* lora_b = nullptr, int rank = 0);
// rank: 0 or 32. epi: kEpiWrite/kEpiAdd/kEpiSwiGlu. exact: reference FP32 order.
// The tile width is chosen per shape (gemm_i8_choose_bn) so the grid fills
// the 148 SMs with the fewest waves.
void launch_gemm_i8(const CUtensorMap& map_a, const WeightMaps& w, const GemmArgs& args, int rank, int epi,
                    bool exact, cudaStream_t stream);
int gemm_i8_choose_bn(int M, int N, int epi);
// Split-K: tiles of a grid that may be split (one counter each), and the
// workspace that bounds (splits x M x N <= 148 x 128 x 128 floats).
constexpr int kGemmSplitTiles = 148;
constexpr size_t kGemmSplitFloats = size_t(148) * 128 * 128;
int gemm_i8_choose_splits(const GemmArgs& args, int bn, bool exact);

// ---- dense tcgen05 kind::i8 throughput of `device` (tc_peak.cu): TOP/s of
// `iters` x 4 MMAs of 128 x 256 x 32 per SM, one CTA per SM; ms_out gets the
// timed launch's duration.
double measure_i8_peak(int device, int iters, float* ms_out);

// ---- elementwise / normalisation / quantisation, kernels.cu
// Row-wise: optional centred RMSNorm (gamma != nullptr: x * (inv * (1 + g))),
// optional FP32 output, optional group-64 quantisation into xq [M][K] and
// xs [G][ldxs]. Non-finite quantisation inputs are reported.
void launch_norm_quant(const float* x, int ldx, int M, int K, const float* gamma, float eps, float* n_out,
                       int ldn, int8_t* xq, float* xs, int ldxs, DeviceStatus* st, cudaStream_t s);
// DeltaNet gated norm fused with quantisation: per value head, o = rms(o, w)
// (non-centred) * silu(z); writes FP32 and the group-64 quantisation.
void launch_gated_norm_quant(const float* o, const float* z, int ldz, int M, int heads, int dv,
                             const float* w, float eps, float* out, int8_t* xq, float* xs, int ldxs,
                             bool quantize, DeviceStatus* st, cudaStream_t s);
// mid[m][r] = dot_scores(x[m], A[r]) for r < R (reference lane order when exact).
// Fast mode with `partial` (lora_a_partial_floats(M) floats) splits K over
// CTAs and reduces the slices in a fixed order.
void launch_lora_a(const float* x, int ldx, int M, int K, const float* A, int R, float* mid, int ldm,
                   bool exact, cudaStream_t s, float* partial = nullptr, size_t partial_floats = 0,
                   DeviceStatus* st = nullptr, bool overlap = false);
// overlap: the next launch is a projection with GemmArgs::late_dep set; the
// LoRA-A kernels then run as its programmatic prerequisites on fewer SMs, so
// that projection's main loop runs beside them.
// Tensor-core LoRA A (lora_a_tc.cu): R <= 128, K % 32 == 0, 16-byte aligned
// rows; the slices of each 128-row tile go to `partial`, then a fixed-order sum.
bool lora_a_tc_supported(const float* x, int ldx, int K, const float* A, int R, int ldm);
size_t lora_a_tc_partial_floats(int max_rows);
void launch_lora_a_tc(const float* x, int ldx, int M, int K, const float* A, int R, float* mid, int ldm,
                      float* partial, size_t partial_floats, DeviceStatus* st, cudaStream_t s, bool overlap = false);
// mid[m][r] = sum over z of partial[z][m][r], as four chains added pairwise.
void launch_lora_a_reduce(const float* partial, int slices, int M, int R, float* mid, int ldm, cudaStream_t s,
                          bool pdl = false);
inline size_t lora_a_partial_floats(int max_rows) {
  const size_t simt = (size_t(148 * 64) + size_t(max_rows)) * 128;
  const size_t tc = lora_a_tc_partial_floats(max_rows);
  return simt > tc ? simt : tc;
}
// Generic SIMT projection for any shape and precision (reference order):
// precision 0: w f32; 1: int8 weight-only; 2: int8-compute; 3: int4.
struct GenericProj {
  int precision, in, out;
  const float* w;        // precision 0
  const uint8_t* wq;     // precision 1-3 (int4 packed as the reference)
  const float* wscale;   // [out][G]
  const float* bias;     // nullable
  const float* lora_b;   // [out][rank], nullable
  int rank;
  float lora_scale;
};
void launch_proj_generic(const GenericProj& p, const float* x, int ldx, const int8_t* xq, const float* xs,
                         int ldxs, const float* mid, int ldm, int M, float* out, int ldo, int epi,
                         cudaStream_t s);
// Finishes a projection whose product v (+ bias) is in `prod` (row stride
// ldp): out = silu(out) * (v + bias) for kEpiSwiGlu, out = v + bias
// otherwise (in place when prod == out). Bias nullable.
void launch_proj_finish(const float* prod, int ldp, const float* bias, float* out, int ldo, int M, int N, int epi,
                        cudaStream_t s);
void launch_embed(const void* table, int dtype, int hidden, const uint32_t* ids, int n, float* x,
                  cudaStream_t s);
// Causal depthwise conv (tap-major weights [k][W]) + SiLU, continuing from a
// tail of `tail_rows` raw rows that precede position `start`.
void launch_conv_silu(const float* raw, int ldr, int n, const float* tail, int tail_rows, int start, int W,
                      int kernel, const float* taps, float* out, cudaStream_t s, int segs = 1);
// dst[i] = src for i < copies (bytes % 16 == 0, 16-byte aligned): one prefix
// state per sequence of a segmented forward.
void launch_broadcast_copy(void* dst, const void* src, size_t bytes, int copies, cudaStream_t s);
// Per token: q/k L2 norms (q also / sqrt(dk)), log decay g = rate * softplus(a + dt)
// (the decay is exp(g)), beta = sigmoid(b). Normalises conv[:, :2kd] in place.
void launch_delta_prep(float* conv, int W, int n, int key_heads, int dk, int value_heads, const float* a,
                       const float* b, int ldab, const float* decay_rate, const float* dt, float* decay,
                       float* beta, cudaStream_t s);
// Gated delta rule over n tokens for every value head (decay given as its log),
// state [H][dk][dv] updated in place; o [n][H*dv] receives q^T S per token.
void launch_delta_recurrence(const float* conv, int n, int key_heads, int dk, int value_heads, int dv,
                             const float* decay, const float* beta, float* state, float* o,
                             cudaStream_t s);
// Strided operands of the dk == 128 recurrence kernel; blockIdx.y indexes
// independent sequences (batch strides in floats).
struct DeltaArgs {
  const float *q, *k, *v;
  int ld_qk, ld_v;
  size_t bs_qkv;
  const float *decay, *beta;   // decay is exp(g) already, or g itself when log_decay != 0
  int log_decay;
  int ld_gb;
  size_t bs_gb;
  int n, key_heads, value_heads, dv;
  float* state;
  size_t bs_state;
  float* o;
  int ldo;
  size_t bs_o;
};
void launch_delta_rec128(const DeltaArgs& a, int batch, cudaStream_t s);
// Chunked form (64-token chunks, dk = dv = 128) of the same rule; needs a
// device workspace of delta_chunk_workspace_bytes(batch, heads, n).
size_t delta_chunk_workspace_bytes(int batch, int heads, int n);
constexpr int kDeltaChunk = 64;  // tokens per chunk of the chunked form
// wide: 32-column scan slices (half the scan CTAs, the same work per thread)
// even when the batch alone would not fill two waves of them; an engine that
// shares the GPU with other lanes asks for them.
void launch_delta_chunked(const DeltaArgs& a, int batch, void* workspace, size_t workspace_bytes, cudaStream_t s,
                          bool wide = false);
void launch_exp(const float* g, float* out, size_t n, cudaStream_t s);
// Split q|gate per head, centred RMSNorm of q and k, partial RoPE from the
// precomputed table, append k/v to the cache at `start`. seg_len > 0: the n
// rows are n / seg_len sequences of seg_len tokens each at positions start..,
// and row t's k/v go to row t of kcache / vcache.
void launch_qk_norm_rope(const float* qkv, int ldq, int n, int heads, int kv_heads, int d, const float* qn,
                         const float* kn, float eps, const float* rope, int half, int start, float* q_out,
                         float* kcache, float* vcache, cudaStream_t s, int seg_len = 0);
// `exact` (reference-order mode) keeps the key split fixed, so prefix
// continuations stay bit-identical to full forwards. seg_len > 0 (head_dim
// 256): n / seg_len sequences of seg_len rows continuing the same `offset`
// prefix keys in kcache / vcache, their own keys in kc_own / vc_own (row t of
// the n rows).
void launch_attention(const float* q, const float* kcache, const float* vcache, const float* gate_src,
                      int ld_gate, int n, int offset, int heads, int kv_heads, int d, float* out, bool exact,
                      cudaStream_t s, int seg_len = 0, const float* kc_own = nullptr, const float* vc_own = nullptr);
// ---- causal attention on the tensor cores, fast mode (attn_tc.cu)
// C[m][n] = alpha * sum_k A[m][k] * B[n][k] (then + C when accumulate, then
// * sigmoid(gate[m][n])), FP32 operands as 3 x TF32 on tcgen05. Batch z =
// outer * inner_count + inner offsets A by outer * a_outer + inner * a_inner,
// B by outer * b_outer + (inner / b_inner_div) * b_inner, C and the gate
// alike. diag >= 0: row m sees columns n <= diag + m only; tiles wholly past
// that are skipped (k_causal = 0), or the K range is cut there (k_causal = 1:
// the K index is the key). K % 32 == 0; operands 16-byte aligned.
struct TcGemmArgs {
  const float* A = nullptr;
  int lda = 0;
  long a_outer = 0, a_inner = 0;
  const float* B = nullptr;
  int ldb = 0;
  long b_outer = 0, b_inner = 0;
  int b_inner_div = 1;
  float* C = nullptr;
  int ldc = 0;
  long c_outer = 0, c_inner = 0;
  const float* gate = nullptr;
  int ldg = 0;
  long g_outer = 0, g_inner = 0;
  int M = 0, N = 0, K = 0;
  float alpha = 1.0f;
  int inner_count = 1;
  int diag = -1;
  int k_causal = 0;
  int accumulate = 0;
  DeviceStatus* status = nullptr;
};
void launch_tc_gemm(const TcGemmArgs& g, int batches, cudaStream_t s);
// Query rows per pass of launch_attention_tc (bounds its score workspace).
constexpr int kAttnTcChunk = 1024;
size_t attention_tc_workspace_floats(int heads, int kv_heads, int d, int max_rows);
bool attention_tc_supported(int d, int heads, int kv_heads);
// Gated causal attention of n query rows at positions offset.. against the
// offset + n keys of kcache / vcache ([keys][kv_heads * d]); q [n][heads][d];
// the gate is column h * 2d + d + c of gate_src's rows; out [n][heads][d].
// ws: attention_tc_workspace_floats floats (scores and Vᵀ).
void launch_attention_tc(const float* q, const float* kc, const float* vc, const float* gate_src, int ld_gate, int n,
                         int offset, int heads, int kv_heads, int d, float* out, float* ws, size_t ws_floats,
                         DeviceStatus* st, cudaStream_t s);

// Centred RMSNorm over rows, in place, plus a non-finite check.
void launch_final_norm(float* x, int M, int K, const float* gamma, float eps, DeviceStatus* st,
                       cudaStream_t s);
// Pointer-head LayerNorm (eps 1e-5, weight and bias) of selected rows.
void launch_head_norm(const float* hidden, int K, const int* rows, int n_rows, const float* w, const float* b,
                      float* out, cudaStream_t s);
// logits[i] = dot_scores(q + bq, k_i + bk) * scale (biases nullable).
void launch_head_dot(const float* q, const float* k, int n_keys, int dim, float scale, const float* bq,
                     const float* bk, float* logits, cudaStream_t s);

// Data::quantize of an F32 [rows][width] device tensor (bits 8 or 4), group
// 64 along the width. Plain layout (layout null): q [rows][width] bytes for
// 8 bits, ceil(rows * width / 2) packed bytes for 4 bits; scales
// [rows][ceil(width / 64)]. An 8-bit layout may map row j to output row
// (j / rb) * rs + ro + j % rb (q_row bytes per output row) and its scales to
// scales[out_row * s_row + group * s_group].
struct QuantLayout {
  size_t q_row, s_row, s_group;
  int rb, rs, ro;
};
QuantLayout quant_plain_layout(size_t rows, size_t width);
void quantize_weights_device(const float* w, size_t rows, size_t width, int bits, uint8_t* q, float* scales,
                             const QuantLayout* layout, cudaStream_t s);
// The FP32 values the reference reads from plain-layout quantised weights
// (Data::row: code times its group's scale), out [rows][width].
void dequantize_weights_device(const uint8_t* q, const float* scales, size_t rows, size_t width, int bits,
                               float* out, cudaStream_t s);

}  // namespace dg
