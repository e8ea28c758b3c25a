// Mixer kernels of the Qwen3.5 torso: DeltaNet conv / recurrence, gated GQA
// attention with partial RoPE, final norm and the pointer head.
#include <cstdint>
#include <cfloat>

#include <algorithm>

#include "launch.h"

namespace dg {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// convolve, src/qwen.rs:712-756: per channel, taps in order from a zero sum,
// skipping taps before the sequence start, then SiLU.
// One thread per channel and 16 consecutive tokens: the window of raw inputs
// (16 + kernel - 1 rows) is loaded once and every tap reuses it.
constexpr int CONV_T = 16, CONV_KMAX = 8;
__global__ void conv_silu_kernel(const float* __restrict__ raw, int ldr, const float* __restrict__ tail, int tail_rows,
                                 int n, int start, int W, int kernel, const float* __restrict__ taps,
                                 float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int c = blockIdx.x * blockDim.x + threadIdx.x, t0 = blockIdx.y * CONV_T;
  if (c >= W) return;
  raw += size_t(blockIdx.z) * n * ldr;  // segment z of equal-length sequences (same tail)
  out += size_t(blockIdx.z) * n * W;
  float w[CONV_KMAX];
  float win[CONV_T + CONV_KMAX - 1];
#pragma unroll
  for (int j = 0; j < CONV_KMAX; ++j) w[j] = j < kernel ? taps[size_t(j) * W + c] : 0.0f;
  // win[i] holds the input at absolute position start + t0 - (kernel - 1) + i.
#pragma unroll
  for (int i = 0; i < CONV_T + CONV_KMAX - 1; ++i) {
    const int source = start + t0 - (kernel - 1) + i;  // absolute position
    float v = 0.0f;
    if (i < CONV_T + kernel - 1 && source >= 0 && source < start + n) {
      v = source >= start ? raw[size_t(source - start) * ldr + c] : tail[size_t(source + tail_rows - start) * W + c];
    }
    win[i] = v;
  }
#pragma unroll
  for (int tt = 0; tt < CONV_T; ++tt) {
    const int t = t0 + tt;
    if (t >= n) break;
    const int position = start + t;
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < CONV_KMAX; ++j) {
      if (j >= kernel || position + j + 1 < kernel) continue;
      // source = position + j + 1 - kernel  ->  window index tt + j
      sum = sum + win[tt + j] * w[j];
    }
    out[size_t(t) * W + c] = silu_f(sum);
  }
}

// Recurrence::head prologue (src/qwen.rs:832-845) for one token: L2 norms of
// q (then / sqrt(dk)) and k per key head, in place; decay and beta per value head.
__global__ void delta_prep_kernel(float* __restrict__ conv, int W, int key_heads, int dk, int value_heads,
                                  const float* __restrict__ a, const float* __restrict__ b, int ldab,
                                  const float* __restrict__ rate, const float* __restrict__ dt, float* __restrict__ decay,
                                  float* __restrict__ beta) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  float* row = conv + size_t(t) * W;
  const float rdk = sqrtf(float(dk));
  for (int v = warp; v < 2 * key_heads; v += nwarps) {
    float* x = row + v * dk;  // v < key_heads: q of head v; else k of head v - key_heads
    float ss = 0.0f;
    for (int i = lane; i < dk; i += 32) ss = __fmaf_rn(x[i], x[i], ss);
    ss = warp_sum(ss);
    float norm = 1.0f / sqrtf(ss + 1e-6f);
    if (v < key_heads) norm = norm / rdk;
    for (int i = lane; i < dk; i += 32) x[i] = x[i] * norm;
  }
  for (int h = threadIdx.x; h < value_heads; h += blockDim.x) {
    decay[size_t(t) * value_heads + h] = rate[h] * softplus_f(a[size_t(t) * ldab + h] + dt[h]);  // log of the decay
    beta[size_t(t) * value_heads + h] = sigmoid_f(b[size_t(t) * ldab + h]);
  }
}

// Gated delta rule, generic shapes: one thread per (value head, value column),
// the reference's per-column arithmetic order (src/qwen.rs:846-866).
__global__ void delta_rec_generic_kernel(const float* __restrict__ conv, int n, int W, int key_heads, int dk,
                                         int value_heads, int dv, const float* __restrict__ decay,
                                         const float* __restrict__ beta, float* __restrict__ state,
                                         float* __restrict__ o) {
  griddep_wait();
  griddep_launch();
  const int id = blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= value_heads * dv) return;
  const int h = id / dv, j = id % dv, kh = h / (value_heads / key_heads), kd = key_heads * dk;
  float* S = state + size_t(h) * dk * dv;
  for (int t = 0; t < n; ++t) {
    const float* q = conv + size_t(t) * W + kh * dk;
    const float* k = conv + size_t(t) * W + kd + kh * dk;
    const float v = conv[size_t(t) * W + 2 * kd + h * dv + j];
    const float dec = expf(decay[size_t(t) * value_heads + h]), be = beta[size_t(t) * value_heads + h];
    float delta = 0.0f;
    for (int i = 0; i < dk; ++i) {
      const float s = S[size_t(i) * dv + j] * dec;
      S[size_t(i) * dv + j] = s;
      delta = delta + k[i] * s;
    }
    delta = (v - delta) * be;
    float out = 0.0f;
    for (int i = 0; i < dk; ++i) {
      const float s = S[size_t(i) * dv + j] + k[i] * delta;
      S[size_t(i) * dv + j] = s;
      out = out + q[i] * s;
    }
    o[size_t(t) * value_heads * dv + h * dv + j] = out;
  }
}

// Gated delta rule for dk == 128. A CTA of 4 warps owns 16 value columns of
// one head of one sequence; each warp owns 4 columns and lane l holds state
// rows 4l..4l+3 of them in registers. Tokens are staged through shared memory
// in chunks of 32 with cp.async, double-buffered, so the serial per-token
// chain (decay, k^T S reduction, delta, rank-1 update, q^T S reduction) never
// waits on global memory. Operands are strided so the same kernel serves the
// model (q|k|v rows of the conv output) and the isolated batched recurrence.
constexpr int REC_T = 32, REC_COLS = 16;
struct RecStage {
  float q[REC_T][128];
  float k[REC_T][128];
  float v[REC_T][REC_COLS];
  float decay[REC_T];
  float beta[REC_T];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(128) delta_rec128_kernel(DeltaArgs a) {
  griddep_wait();
  griddep_launch();
  constexpr int DK = 128;
  extern __shared__ __align__(16) uint8_t rec_smem[];
  RecStage* st = reinterpret_cast<RecStage*>(rec_smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int groups16 = a.dv / REC_COLS;
  const size_t bi = blockIdx.y;
  const int h = blockIdx.x / groups16, c0 = (blockIdx.x % groups16) * REC_COLS;
  const int kh = h / (a.value_heads / a.key_heads), j0 = c0 + warp * 4;
  const float* qb = a.q + bi * a.bs_qkv + kh * DK;
  const float* kb = a.k + bi * a.bs_qkv + kh * DK;
  const float* vb = a.v + bi * a.bs_qkv + h * a.dv + c0;
  const float* db = a.decay + bi * a.bs_gb + h;
  const float* bb = a.beta + bi * a.bs_gb + h;
  float* ob = a.o + bi * a.bs_o + h * a.dv + j0;
  float* S = a.state + bi * a.bs_state + size_t(h) * DK * a.dv;
  const int dv = a.dv, n = a.n;
  const int chunks = (n + REC_T - 1) / REC_T;

  auto stage = [&](int chunk, int buf) {
    const int t0 = chunk * REC_T, tn = min(REC_T, n - t0);
    RecStage& sg = st[buf];
    for (int i = threadIdx.x; i < tn * 32; i += 128) {  // q and k: 32 float4 per token each
      const int t = i / 32, c = (i % 32) * 4;
      cp_async16(&sg.q[t][c], qb + size_t(t0 + t) * a.ld_qk + c);
      cp_async16(&sg.k[t][c], kb + size_t(t0 + t) * a.ld_qk + c);
    }
    for (int i = threadIdx.x; i < tn * (REC_COLS / 4); i += 128) {
      const int t = i / (REC_COLS / 4), c = (i % (REC_COLS / 4)) * 4;
      cp_async16(&sg.v[t][c], vb + size_t(t0 + t) * a.ld_v + c);
    }
    cp_async_commit();
    for (int t = threadIdx.x; t < tn; t += 128) {
      const float d = db[size_t(t0 + t) * a.ld_gb];
      sg.decay[t] = a.log_decay ? expf(d) : d;
      sg.beta[t] = bb[size_t(t0 + t) * a.ld_gb];
    }
  };

  float s[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float4 v = *reinterpret_cast<const float4*>(S + size_t(lane * 4 + r) * dv + j0);
    s[r][0] = v.x; s[r][1] = v.y; s[r][2] = v.z; s[r][3] = v.w;
  }
  if (chunks > 0) stage(0, 0);
  for (int ch = 0; ch < chunks; ++ch) {
    cp_async_wait_all();
    __syncthreads();  // chunk ch is resident; the other buffer is free
    if (ch + 1 < chunks) stage(ch + 1, (ch + 1) & 1);
    const RecStage& sg = st[ch & 1];
    const int t0 = ch * REC_T, tn = min(REC_T, n - t0);
    for (int t = 0; t < tn; ++t) {
      const float4 kq4 = *reinterpret_cast<const float4*>(&sg.k[t][lane * 4]);
      const float4 qq4 = *reinterpret_cast<const float4*>(&sg.q[t][lane * 4]);
      const float4 vv4 = *reinterpret_cast<const float4*>(&sg.v[t][warp * 4]);
      const float kk[4] = {kq4.x, kq4.y, kq4.z, kq4.w}, qv[4] = {qq4.x, qq4.y, qq4.z, qq4.w};
      const float v[4] = {vv4.x, vv4.y, vv4.z, vv4.w};
      const float d0 = sg.decay[t], b0 = sg.beta[t];
      float p[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float acc = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          s[r][c] = s[r][c] * d0;
          acc = __fmaf_rn(kk[r], s[r][c], acc);
        }
        p[c] = acc;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int c = 0; c < 4; ++c) p[c] += __shfl_xor_sync(0xffffffffu, p[c], off);
      float out[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float delta = (v[c] - p[c]) * b0;
        float acc = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          s[r][c] = __fmaf_rn(kk[r], delta, s[r][c]);
          acc = __fmaf_rn(qv[r], s[r][c], acc);
        }
        out[c] = acc;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int c = 0; c < 4; ++c) out[c] += __shfl_xor_sync(0xffffffffu, out[c], off);
      if (lane == 0)
        *reinterpret_cast<float4*>(ob + size_t(t0 + t) * a.ldo) = make_float4(out[0], out[1], out[2], out[3]);
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
    *reinterpret_cast<float4*>(S + size_t(lane * 4 + r) * dv + j0) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
}

__global__ void exp_kernel(const float* __restrict__ g, float* __restrict__ out, size_t n) {
  griddep_wait();
  griddep_launch();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = expf(g[i]);
}

}  // namespace

// Four adjacent channels per thread (float4 loads and stores; W, ldr % 4 == 0,
// 16-byte aligned rows); per channel the same window and order as
// conv_silu_kernel, so the outputs are bit-identical.
__global__ void __launch_bounds__(128) conv_silu4_kernel(const float* __restrict__ raw, int ldr,
                                                         const float* __restrict__ tail, int tail_rows, int n,
                                                         int start, int W, int kernel,
                                                         const float* __restrict__ taps, float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x), t0 = blockIdx.y * CONV_T;
  if (c >= W) return;
  raw += size_t(blockIdx.z) * n * ldr;  // segment z of equal-length sequences (same tail)
  out += size_t(blockIdx.z) * n * W;
  float4 w[CONV_KMAX];
#pragma unroll
  for (int j = 0; j < CONV_KMAX; ++j)
    w[j] = j < kernel ? __ldg(reinterpret_cast<const float4*>(taps + size_t(j) * W + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 win[CONV_T + CONV_KMAX - 1];
#pragma unroll
  for (int i = 0; i < CONV_T + CONV_KMAX - 1; ++i) {
    const int source = start + t0 - (kernel - 1) + i;  // absolute position
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < CONV_T + kernel - 1 && source >= 0 && source < start + n) {
      const float* src = source >= start ? raw + size_t(source - start) * ldr + c
                                         : tail + size_t(source + tail_rows - start) * W + c;
      v = *reinterpret_cast<const float4*>(src);
    }
    win[i] = v;
  }
#pragma unroll
  for (int tt = 0; tt < CONV_T; ++tt) {
    const int t = t0 + tt;
    if (t >= n) break;
    const int position = start + t;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < CONV_KMAX; ++j) {
      if (j >= kernel || position + j + 1 < kernel) continue;
      sum.x = sum.x + win[tt + j].x * w[j].x;
      sum.y = sum.y + win[tt + j].y * w[j].y;
      sum.z = sum.z + win[tt + j].z * w[j].z;
      sum.w = sum.w + win[tt + j].w * w[j].w;
    }
    *reinterpret_cast<float4*>(out + size_t(t) * W + c) =
        make_float4(silu_f(sum.x), silu_f(sum.y), silu_f(sum.z), silu_f(sum.w));
  }
}
void launch_conv_silu(const float* raw, int ldr, int n, const float* tail, int tail_rows, int start, int W, int kernel,
                      const float* taps, float* out, cudaStream_t s, int segs) {
  if (n <= 0 || segs <= 0) return;
  if (kernel < 1 || kernel > CONV_KMAX) throw CudaError("conv: kernel width must be 1..8");
  const bool vec = W % 4 == 0 && ldr % 4 == 0 && reinterpret_cast<uintptr_t>(raw) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(taps) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   (tail_rows == 0 || reinterpret_cast<uintptr_t>(tail) % 16 == 0);
  if (vec) {
    dim3 grid((W / 4 + 127) / 128, (n + CONV_T - 1) / CONV_T, segs);
    launch_pdl(conv_silu4_kernel, dim3(grid), dim3(128), 0, s, raw, ldr, tail, tail_rows, n, start, W, kernel, taps,
               out);
  } else {
    dim3 grid((W + 255) / 256, (n + CONV_T - 1) / CONV_T, segs);
    launch_pdl(conv_silu_kernel, dim3(grid), dim3(256), 0, s, raw, ldr, tail, tail_rows, n, start, W, kernel, taps,
               out);
  }
  DG_CUDA(cudaGetLastError());
}

void launch_delta_prep(float* conv, int W, int n, int key_heads, int dk, int value_heads, const float* a,
                       const float* b, int ldab, const float* decay_rate, const float* dt, float* decay, float* beta,
                       cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(delta_prep_kernel, dim3(n), dim3(256), 0, s, conv, W, key_heads, dk, value_heads, a, b, ldab, decay_rate, dt, decay, beta);
  DG_CUDA(cudaGetLastError());
}

void launch_delta_recurrence(const float* conv, int n, int key_heads, int dk, int value_heads, int dv,
                             const float* decay, const float* beta, float* state, float* o, cudaStream_t s) {
  if (n <= 0) return;
  const int W = 2 * key_heads * dk + value_heads * dv;
  if (dk == 128 && dv % REC_COLS == 0) {
    DeltaArgs a{};
    a.q = conv;
    a.k = conv + key_heads * dk;
    a.v = conv + 2 * key_heads * dk;
    a.ld_qk = a.ld_v = W;
    a.decay = decay;
    a.log_decay = 1;
    a.beta = beta;
    a.ld_gb = value_heads;
    a.n = n;
    a.key_heads = key_heads;
    a.value_heads = value_heads;
    a.dv = dv;
    a.state = state;
    a.o = o;
    a.ldo = value_heads * dv;
    launch_delta_rec128(a, 1, s);
  } else {
    const int threads = value_heads * dv;
    launch_pdl(delta_rec_generic_kernel, dim3((threads + 127) / 128), dim3(128), 0, s, conv, n, W, key_heads, dk, value_heads, dv, decay,
                                                                   beta, state, o);
    DG_CUDA(cudaGetLastError());
  }
}

void launch_delta_rec128(const DeltaArgs& a, int batch, cudaStream_t s) {
  if (a.n <= 0 || batch <= 0) return;
  if (a.dv % REC_COLS) throw CudaError("delta_rec128: value width must be a multiple of 16");
  static std::atomic<uint64_t> configured{0};
  const int smem = 2 * sizeof(RecStage);
  once_per_device(configured, [&] {
    DG_CUDA(cudaFuncSetAttribute(delta_rec128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  });
  dim3 grid(a.value_heads * (a.dv / REC_COLS), batch);
  launch_pdl(delta_rec128_kernel, dim3(grid), dim3(128), smem, s, a);
  DG_CUDA(cudaGetLastError());
}

__global__ void broadcast_copy_kernel(float4* __restrict__ dst, const float4* __restrict__ src, size_t n4, int copies) {
  griddep_wait();
  griddep_launch();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n4; i += size_t(gridDim.x) * blockDim.x) {
    const float4 v = src[i];
    for (int c = 0; c < copies; ++c) dst[size_t(c) * n4 + i] = v;
  }
}

void launch_broadcast_copy(void* dst, const void* src, size_t bytes, int copies, cudaStream_t s) {
  if (!bytes || copies <= 0) return;
  if (bytes % 16 || reinterpret_cast<uintptr_t>(dst) % 16 || reinterpret_cast<uintptr_t>(src) % 16)
    throw CudaError("broadcast_copy: 16-byte aligned whole float4 rows only");
  const size_t n4 = bytes / 16;
  const int blocks = int(std::min<size_t>((n4 + 255) / 256, 592));
  launch_pdl(broadcast_copy_kernel, dim3(blocks), dim3(256), 0, s, reinterpret_cast<float4*>(dst),
             reinterpret_cast<const float4*>(src), n4, copies);
  DG_CUDA(cudaGetLastError());
}

void launch_exp(const float* g, float* out, size_t n, cudaStream_t s) {
  if (!n) return;
  launch_pdl(exp_kernel, dim3(592), dim3(256), 0, s, g, out, n);
  DG_CUDA(cudaGetLastError());
}


}  // namespace dg
