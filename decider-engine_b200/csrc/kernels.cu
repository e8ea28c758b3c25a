// Normalisation, quantisation, LoRA-A, generic projection and embedding kernels.
// Compiled with -fmad=false (see common.cuh): reference-order arithmetic by default.
#include <cfloat>

#include "launch.h"

namespace dg {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide sum for blockDim.x == 256 (8 warps); all threads get the result.
__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < 8 ? red[l] : 0.0f;
  t = warp_sum(t);
  return t;
}

// QuantizedInputs::new per 64-wide group (src/tensor.rs:328-339): scale =
// max|v|/127 (at least FLT_MIN; 1.0 for an all-zero group), q = round(v/scale)
// clamped to +-127. `vals` points at the group in shared memory; one warp
// quantises one group of `len` <= 64 values.
__device__ __forceinline__ void quantize_group_warp(const float* vals, int len, int8_t* q_out, float* scale_out,
                                                    bool* nonfinite) {
  const int l = threadIdx.x % 32;
  float a = l < len ? vals[l] : 0.0f, b = l + 32 < len ? vals[l + 32] : 0.0f;
  bool bad = !isfinite(a) || !isfinite(b);
  if (__any_sync(0xffffffffu, bad)) *nonfinite = true;
  float mx = warp_max(fmaxf(fabsf(a), fabsf(b)));
  float scale = mx == 0.0f ? 1.0f : fmaxf(mx / 127.0f, FLT_MIN);
  if (l < len) q_out[l] = int8_t(fminf(fmaxf(roundf(a / scale), -127.0f), 127.0f));
  if (l + 32 < len) q_out[l + 32] = int8_t(fminf(fmaxf(roundf(b / scale), -127.0f), 127.0f));
  if (l == 0) *scale_out = scale;
}

// Warp-per-row variant for K % 128 == 0: lane l holds float4 l + 32 i of the
// row, so no shared memory or block barrier is needed. With gamma (NV float4
// per lane kept in registers) the centred RMSNorm comes first.
template <int NV>
__global__ void __launch_bounds__(256) norm_quant_warp_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                              const float* __restrict__ gamma, float eps,
                                                              float* __restrict__ n_out, int ldn,
                                                              int8_t* __restrict__ xq, float* __restrict__ xs,
                                                              int ldxs, DeviceStatus* st) {
  griddep_wait();
  griddep_launch();
  const int m = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
  if (m >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + size_t(m) * ldx);
  const int nv = K / 128;
  bool bad = false;
  if (NV > 0) {
    // The row and gamma are loaded up front so every load is in flight at once.
    float4 v[NV > 0 ? NV : 1], gv[NV > 0 ? NV : 1];
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[i] = xr[lane + 32 * i];
      gv[i] = __ldg(g4 + lane + 32 * i);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      ss = __fmaf_rn(v[i].x, v[i].x, ss);
      ss = __fmaf_rn(v[i].y, v[i].y, ss);
      ss = __fmaf_rn(v[i].z, v[i].z, ss);
      ss = __fmaf_rn(v[i].w, v[i].w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / float(K) + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 g = gv[i];
      v[i].x = v[i].x * (inv * (1.0f + g.x));
      v[i].y = v[i].y * (inv * (1.0f + g.y));
      v[i].z = v[i].z * (inv * (1.0f + g.z));
      v[i].w = v[i].w * (inv * (1.0f + g.w));
      if (n_out) reinterpret_cast<float4*>(n_out + size_t(m) * ldn)[lane + 32 * i] = v[i];
      if (xq) {
        const int col = 4 * (lane + 32 * i);
        quantize_vec4_halfwarp(v[i], xq + size_t(m) * K + col, xs + size_t(col / 64) * ldxs + m, (lane & 15) == 0,
                               &bad);
      }
    }
  } else {
    // Quantisation only: blockIdx.y selects a 512-column segment of the row.
    const int i0 = blockIdx.y * 4, i1 = min(nv, i0 + 4);
#pragma unroll 4
    for (int i = i0; i < i1; ++i) {
      const float4 v = xr[lane + 32 * i];
      if (n_out) reinterpret_cast<float4*>(n_out + size_t(m) * ldn)[lane + 32 * i] = v;
      const int col = 4 * (lane + 32 * i);
      quantize_vec4_halfwarp(v, xq + size_t(m) * K + col, xs + size_t(col / 64) * ldxs + m, (lane & 15) == 0, &bad);
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) report(st, kNonFinite, 1);
}

// One 256-thread CTA per row.
__global__ void norm_quant_kernel(const float* __restrict__ x, int ldx, int K, const float* __restrict__ gamma,
                                  float eps, float* __restrict__ n_out, int ldn, int8_t* __restrict__ xq,
                                  float* __restrict__ xs, int ldxs, DeviceStatus* st) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float row[];
  __shared__ float red[8];
  const int m = blockIdx.x;
  const float* xr = x + size_t(m) * ldx;
  float ss = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = xr[k];
    row[k] = v;
    ss = __fmaf_rn(v, v, ss);
  }
  if (gamma) {
    // rms, src/qwen.rs:208-217: v * (inv * (1 + g)), inv = 1/sqrt(mean(v^2) + eps).
    const float total = block_sum_256(ss, red);
    const float inv = 1.0f / sqrtf(total / float(K) + eps);
    for (int k = threadIdx.x; k < K; k += 256) row[k] = row[k] * (inv * (1.0f + gamma[k]));
  }
  __syncthreads();
  if (n_out)
    for (int k = threadIdx.x; k < K; k += 256) n_out[size_t(m) * ldn + k] = row[k];
  if (xq) {
    __shared__ bool nonfinite;
    if (threadIdx.x == 0) nonfinite = false;
    __syncthreads();
    const int G = (K + 63) / 64;
    for (int g = threadIdx.x / 32; g < G; g += 8) {
      const int len = min(64, K - g * 64);
      quantize_group_warp(row + g * 64, len, xq + size_t(m) * K + g * 64, xs + size_t(g) * ldxs + m, &nonfinite);
    }
    __syncthreads();
    if (threadIdx.x == 0 && nonfinite) report(st, kNonFinite, 1);
  }
}

// Recurrence::head's output step (src/qwen.rs:867-873): per value head,
// o = rms(o, w) (non-centred weight) then o *= silu(z). One CTA per token.
__global__ void gated_norm_quant_kernel(const float* __restrict__ o, const float* __restrict__ z, int ldz, int heads,
                                        int dv, const float* __restrict__ w, float eps, float* __restrict__ out,
                                        int8_t* __restrict__ xq, float* __restrict__ xs, int ldxs, int quantize,
                                        DeviceStatus* st) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float row[];
  const int m = blockIdx.x, K = heads * dv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int h = warp; h < heads; h += 8) {
    const float* oh = o + size_t(m) * K + h * dv;
    float ss = 0.0f;
    for (int j = lane; j < dv; j += 32) ss = __fmaf_rn(oh[j], oh[j], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(dv) + eps);
    for (int j = lane; j < dv; j += 32) {
      const float v = oh[j] * (inv * w[j]);
      row[h * dv + j] = v * silu_f(z[size_t(m) * ldz + h * dv + j]);
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += 256) out[size_t(m) * K + k] = row[k];
  if (quantize) {
    __shared__ bool nonfinite;
    if (threadIdx.x == 0) nonfinite = false;
    __syncthreads();
    const int G = (K + 63) / 64;
    for (int g = warp; g < G; g += 8)
      quantize_group_warp(row + g * 64, min(64, K - g * 64), xq + size_t(m) * K + g * 64, xs + size_t(g) * ldxs + m,
                          &nonfinite);
    __syncthreads();
    if (threadIdx.x == 0 && nonfinite) report(st, kNonFinite, 2);
  }
}

// dv == 128: one warp per (row, head). Lane l holds elements l + 32 i
// (i < 4) of the head, in the same order as gated_norm_quant_kernel, so the
// sum of squares and every output are bit-identical; the head's two 64-wide
// quantisation groups are elements {l, l + 32} and {l + 64, l + 96}, quantised
// straight from registers (the scale depends only on the group maximum).
__global__ void __launch_bounds__(256) gated_norm_quant_warp_kernel(const float* __restrict__ o,
                                                                    const float* __restrict__ z, int ldz, int M,
                                                                    int heads, const float* __restrict__ w, float eps,
                                                                    float* __restrict__ out, int8_t* __restrict__ xq,
                                                                    float* __restrict__ xs, int ldxs, int quantize,
                                                                    DeviceStatus* st) {
  griddep_wait();
  griddep_launch();
  constexpr int DV = 128;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
  if (gw >= M * heads) return;
  const int m = gw / heads, h = gw % heads, K = heads * DV;
  const float* oh = o + size_t(m) * K + h * DV;
  const float* zh = z + size_t(m) * ldz + h * DV;
  float a[4], zv[4], wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[i] = oh[lane + 32 * i];
    zv[i] = zh[lane + 32 * i];
    wv[i] = __ldg(w + lane + 32 * i);
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = __fmaf_rn(a[i], a[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(DV) + eps);
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = a[i] * (inv * wv[i]) * silu_f(zv[i]);
    out[size_t(m) * K + h * DV + lane + 32 * i] = v[i];
  }
  if (!quantize) return;
  bool bad = false;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const float p0 = v[2 * g], p1 = v[2 * g + 1];
    bad |= !isfinite(p0) || !isfinite(p1);
    const float mx = warp_max(fmaxf(fabsf(p0), fabsf(p1)));
    const float scale = mx == 0.0f ? 1.0f : fmaxf(mx / 127.0f, FLT_MIN);
    int8_t* q = xq + size_t(m) * K + h * DV + 64 * g;
    q[lane] = int8_t(fminf(fmaxf(roundf(p0 / scale), -127.0f), 127.0f));
    q[lane + 32] = int8_t(fminf(fmaxf(roundf(p1 / scale), -127.0f), 127.0f));
    if (lane == 0) xs[size_t((h * DV) / 64 + g) * ldxs + m] = scale;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) report(st, kNonFinite, 2);
}

// LoRA A: mid[m][r] = dot_scores(x[m], A[r]) in the reference's order
// (src/tensor.rs:6-25): eight lanes over k % 8, each a sequential
// multiply-then-add chain, the lanes summed from -0.0 in order, then the tail.
// A thread runs lane `i` of a 4-row x 4-output tile (16 chains sharing 8 loads
// per step); the eight lanes of a tile are eight consecutive threads.
// TM = 1 serves the few rows of the pointer head: more loads in flight per
// thread instead of three padding rows.
template <bool EXACT, int TM = 4, int TR = 4>
__global__ void __launch_bounds__(256) lora_a_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                     const float* __restrict__ A, int R, float* __restrict__ mid,
                                                     int ldm) {
  griddep_wait();
  griddep_launch();
  const long gid = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane8 = int(gid & 7);
  const long tile = gid >> 3;
  const int rtiles = (R + TR - 1) / TR;
  const int m0 = int(tile / rtiles) * TM, r0 = int(tile % rtiles) * TR;
  const float* xr[TM];
  const float* ar[TR];
#pragma unroll
  for (int a = 0; a < TM; ++a) xr[a] = x + size_t(min(m0 + a, M - 1)) * ldx;
#pragma unroll
  for (int b = 0; b < TR; ++b) ar[b] = A + size_t(min(r0 + b, R - 1)) * K;
  const int kfull = (K / 8) * 8;
  float acc[TM][TR];
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TR; ++b) acc[a][b] = 0.0f;
  if (m0 < M) {
#pragma unroll(TM == 1 ? 16 : 2)
    for (int k = lane8; k < kfull; k += 8) {
      float xv[TM], av[TR];
#pragma unroll
      for (int a = 0; a < TM; ++a) xv[a] = __ldg(xr[a] + k);
#pragma unroll
      for (int b = 0; b < TR; ++b) av[b] = __ldg(ar[b] + k);
#pragma unroll
      for (int a = 0; a < TM; ++a)
#pragma unroll
        for (int b = 0; b < TR; ++b) {
          if (EXACT)
            acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(xv[a], av[b]));
          else
            acc[a][b] = __fmaf_rn(xv[a], av[b], acc[a][b]);
        }
    }
  }
  // Each lane finalises two of the 16 outputs: the eight lane partials summed
  // in lane order from -0.0, then the tail.
  const int base = threadIdx.x & ~7;
#pragma unroll
  for (int o = 0; o < TM * TR; ++o) {
    const int a = o / TR, b = o % TR;
    float s = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc[a][b], base + l));
    if ((o >> 1) == lane8) {
      const int m = m0 + a, r = r0 + b;
      if (m < M && r < R) {
        for (int k = kfull; k < K; ++k) s = __fadd_rn(s, __fmul_rn(xr[a][k], ar[b][k]));
        mid[size_t(m) * ldm + r] = s;
      }
    }
  }
}

// LoRA A, fast mode (fused multiply-add, free summation order): one warp per
// 4-row x 4-output tile, the 32 lanes striding K so loads stay coalesced and
// plenty of chains are in flight; a butterfly reduction combines the lanes.
__global__ void __launch_bounds__(256) lora_a_fast_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                          const float* __restrict__ A, int R, float* __restrict__ mid,
                                                          int ldm) {
  griddep_wait();
  griddep_launch();
  constexpr int TM = 4, TR = 4;
  const long tile = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int rtiles = (R + TR - 1) / TR;
  const int m0 = int(tile / rtiles) * TM, r0 = int(tile % rtiles) * TR;
  if (m0 >= M) return;  // whole warp leaves together
  const float* xr[TM];
  const float* ar[TR];
#pragma unroll
  for (int a = 0; a < TM; ++a) xr[a] = x + size_t(min(m0 + a, M - 1)) * ldx;
#pragma unroll
  for (int b = 0; b < TR; ++b) ar[b] = A + size_t(min(r0 + b, R - 1)) * K;
  float acc[TM][TR];
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TR; ++b) acc[a][b] = 0.0f;
#pragma unroll 4
  for (int k = lane; k < K; k += 32) {
    float xv[TM], av[TR];
#pragma unroll
    for (int a = 0; a < TM; ++a) xv[a] = __ldg(xr[a] + k);
#pragma unroll
    for (int b = 0; b < TR; ++b) av[b] = __ldg(ar[b] + k);
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TR; ++b) acc[a][b] = __fmaf_rn(xv[a], av[b], acc[a][b]);
  }
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TR; ++b) {
      float v = acc[a][b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[a][b] = v;
    }
  if (lane < TM * TR) {
    const int a = lane / TR, b = lane % TR, m = m0 + a, r = r0 + b;
    float v = 0.0f;
#pragma unroll
    for (int o = 0; o < TM * TR; ++o)
      if (o == lane) v = acc[o / TR][o % TR];
    if (m < M && r < R) mid[size_t(m) * ldm + r] = v;
  }
}

// 16-byte global -> shared copy; src_bytes 0 fills the destination with zeros.
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_groups() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// LoRA A, fast mode: partial[slice] = x · Aᵀ over one K slice, split so the
// skinny [M x R] output still fills the GPU; lora_a_reduce_kernel adds the
// slices in a fixed order (deterministic). CTA = TM rows x RT outputs; 32-wide
// K chunks go to shared memory K-contiguous (double-buffered cp.async). Each
// thread owns 4 rows x OPT outputs, the outputs strided by NOG so the 16-byte
// loads of one warp fall on distinct banks, and consumes four k per load: a
// 16-byte load feeds 4 to 8 FMAs.
template <int TM, int RT>
struct LoraTile {
  static constexpr int KC = 32, LD = KC + 4;  // floats per staged row (16-byte aligned)
  static constexpr int NOG = 1024 / TM;       // output groups (threads per row group)
  static constexpr int OPT = RT / NOG;        // outputs per thread
  static constexpr int STAGE = (TM + RT) * LD;
  static constexpr int SMEM = 2 * STAGE * 4;
  static_assert(OPT >= 1 && RT % NOG == 0, "tile shape");
};

template <int TM, int RT>
__global__ void __launch_bounds__(256) lora_a_splitk_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                            const float* __restrict__ A, int R,
                                                            float* __restrict__ partial, int kslice) {
  griddep_wait();
  griddep_launch();
  using T = LoraTile<TM, RT>;
  constexpr int LD = T::LD, NOG = T::NOG, OPT = T::OPT, KC = T::KC;
  extern __shared__ __align__(16) float lora_smem[];
  const int tid = threadIdx.x, og = tid % NOG, rg = tid / NOG;
  const int m_base = blockIdx.x * TM, r_base = blockIdx.y * RT;
  const int k0 = blockIdx.z * kslice, k1 = min(K, k0 + kslice);
  const int chunks = (k1 - k0) / KC;  // kslice and K are multiples of 32
  auto stage_x = [&](int b) { return lora_smem + b * T::STAGE; };
  auto stage_a = [&](int b) { return lora_smem + b * T::STAGE + TM * LD; };
  auto load = [&](int c, int b) {
    const int kc = k0 + c * KC;
    for (int i = tid; i < (TM + RT) * (KC / 4); i += 256) {
      const int row = i / (KC / 4), k4 = (i % (KC / 4)) * 4;
      if (row < TM) {
        const int m = m_base + row;
        const float* src = m < M ? x + size_t(m) * ldx + kc + k4 : x;
        cp_async16_zfill(stage_x(b) + row * LD + k4, src, m < M ? 16 : 0);
      } else {
        const int r = r_base + row - TM;
        const float* src = r < R ? A + size_t(r) * K + kc + k4 : A;
        cp_async16_zfill(stage_a(b) + (row - TM) * LD + k4, src, r < R ? 16 : 0);
      }
    }
    cp_async_commit_group();
  };
  float acc[4][OPT];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int o = 0; o < OPT; ++o) acc[a][o] = 0.0f;
  if (chunks > 0) load(0, 0);
  for (int c = 0; c < chunks; ++c) {
    if (c + 1 < chunks) {
      load(c + 1, (c + 1) & 1);
      cp_async_wait_groups<1>();
    } else {
      cp_async_wait_groups<0>();
    }
    __syncthreads();
    const float* xs = stage_x(c & 1) + rg * 4 * LD;
    const float* as = stage_a(c & 1) + og * LD;
#pragma unroll
    for (int k4 = 0; k4 < KC; k4 += 4) {
      float4 xv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xv[a] = *reinterpret_cast<const float4*>(xs + a * LD + k4);
#pragma unroll
      for (int o = 0; o < OPT; ++o) {
        const float4 av = *reinterpret_cast<const float4*>(as + o * NOG * LD + k4);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          acc[a][o] = __fmaf_rn(xv[a].x, av.x, acc[a][o]);
          acc[a][o] = __fmaf_rn(xv[a].y, av.y, acc[a][o]);
          acc[a][o] = __fmaf_rn(xv[a].z, av.z, acc[a][o]);
          acc[a][o] = __fmaf_rn(xv[a].w, av.w, acc[a][o]);
        }
      }
    }
    __syncthreads();  // the buffer is refilled two chunks on
  }
  float* out = partial + size_t(blockIdx.z) * M * R;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int m = m_base + rg * 4 + a;
    if (m >= M) continue;
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const int r = r_base + og + o * NOG;
      if (r < R) out[size_t(m) * R + r] = acc[a][o];
    }
  }
}

// Sums the split-K slices partial[z][M][R] into mid (row stride ldm): slice
// z goes to chain z % 8 and the chains are added pairwise in a fixed order,
// so the result is deterministic.
__global__ void __launch_bounds__(128) lora_a_reduce_kernel(const float* __restrict__ partial, int slices, int M,
                                                            int R, float* __restrict__ mid, int ldm) {
  // Trigger first: a projection launched as this kernel's dependent may start
  // its main loop while the LoRA-A pass still runs (it waits for this kernel
  // before reading mid). This kernel itself waits before touching memory.
  griddep_launch();
  griddep_wait();
  // One thread per four outputs; eight slices in flight per round, added in
  // a fixed order (deterministic).
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int n4 = M * R / 4;
  if (i >= n4) return;
  const float4* p4 = reinterpret_cast<const float4*>(partial);
  float4 c[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) c[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  auto add = [](float4& a, const float4 b) { a = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); };
  int z = 0;
  for (; z + 8 <= slices; z += 8) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldg(p4 + size_t(z + j) * n4 + i);
#pragma unroll
    for (int j = 0; j < 8; ++j) add(c[j], v[j]);
  }
#pragma unroll
  for (int j = 0; j < 7; ++j)
    if (z + j < slices) add(c[j], __ldg(p4 + size_t(z + j) * n4 + i));
  add(c[0], c[1]);
  add(c[2], c[3]);
  add(c[4], c[5]);
  add(c[6], c[7]);
  add(c[0], c[2]);
  add(c[4], c[6]);
  add(c[0], c[4]);
  const int e = 4 * i;
  *reinterpret_cast<float4*>(mid + size_t(e / R) * ldm + e % R) = c[0];
}


}  // namespace

void launch_lora_a_reduce(const float* partial, int slices, int M, int R, float* mid, int ldm, cudaStream_t s,
                          bool pdl) {
  if (R % 4 || ldm % 4 || reinterpret_cast<uintptr_t>(mid) % 16 || reinterpret_cast<uintptr_t>(partial) % 16)
    throw CudaError("lora_a_reduce: rank, row stride and buffers must be 16-byte aligned");
  launch_k(pdl || pdl_enabled(), lora_a_reduce_kernel, dim3((M * R / 4 + 127) / 128), dim3(128), 0, s, partial, slices,
           M, R, mid, ldm);
  DG_CUDA(cudaGetLastError());
}

namespace {

template <int TM, int RT>
void launch_lora_splitk(const float* x, int ldx, int M, int K, const float* A, int R, float* mid, int ldm,
                        float* partial, size_t partial_floats, cudaStream_t s) {
  using T = LoraTile<TM, RT>;
  static std::atomic<uint64_t> configured{0};  // per instantiation
  once_per_device(configured, [] {
    DG_CUDA(cudaFuncSetAttribute(lora_a_splitk_kernel<TM, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 T::SMEM));
  });
  const int gx = (M + TM - 1) / TM, gy = (R + RT - 1) / RT;
  const int slices = std::max(1, std::min(K / T::KC, (148 + gx * gy - 1) / (gx * gy)));
  const int kslice = ((K + slices - 1) / slices + T::KC - 1) / T::KC * T::KC;
  const int used = (K + kslice - 1) / kslice;
  if (size_t(used) * M * R > partial_floats) throw CudaError("lora_a: split-K workspace too small");
  launch_pdl(lora_a_splitk_kernel<TM, RT>, dim3(dim3(gx, gy, used)), dim3(256), T::SMEM, s, x, ldx, M, K, A, R, partial, kslice);
  DG_CUDA(cudaGetLastError());
  launch_lora_a_reduce(partial, used, M, R, mid, ldm, s);
}

__device__ __forceinline__ float dequant(const uint8_t* wq, const float* wscale, int precision, int n, int k, int K) {
  const int G = (K + 63) / 64;
  const float sc = wscale[size_t(n) * G + k / 64];
  if (precision == 3) {
    const size_t i = size_t(n) * K + k;
    const int nib = (wq[i / 2] >> (4 * (i % 2))) & 15;
    return (float(nib) - 8.0f) * sc;
  }
  return float(int8_t(wq[size_t(n) * K + k])) * sc;
}

// Generic projection: one thread per output (m, n), reference arithmetic
// (linear_int8 scaled dots or dot_scores over expanded weights, + bias or 0.0,
// Adapter::combine, Epilogue::store).
__global__ void proj_generic_kernel(GenericProj p, const float* __restrict__ x, int ldx, const int8_t* __restrict__ xq,
                                    const float* __restrict__ xs, int ldxs, const float* __restrict__ mid, int ldm,
                                    int M, float* __restrict__ out, int ldo, int epi) {
  griddep_wait();
  griddep_launch();
  const int n = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  if (n >= p.out || m >= M) return;
  const int K = p.in;
  float base;
  if (p.precision == 2) {
    const int G = (K + 63) / 64;
    float sum = 0.0f;
    for (int g = 0; g < G; ++g) {
      int dot = 0;
      const int len = min(64, K - g * 64);
      for (int k = 0; k < len; ++k)
        dot += int(xq[size_t(m) * K + g * 64 + k]) * int(int8_t(p.wq[size_t(n) * K + g * 64 + k]));
      sum = sum + float(dot) * (xs[size_t(g) * ldxs + m] * p.wscale[size_t(n) * G + g]);
    }
    base = sum;
  } else {
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int kfull = (K / 8) * 8;
    const float* xr = x + size_t(m) * ldx;
    for (int k = 0; k < kfull; ++k) {
      const float w = p.precision == 0 ? p.w[size_t(n) * K + k] : dequant(p.wq, p.wscale, p.precision, n, k, K);
      lanes[k & 7] = lanes[k & 7] + xr[k] * w;
    }
    float s = -0.0f;
    for (int l = 0; l < 8; ++l) s = s + lanes[l];
    for (int k = kfull; k < K; ++k) {
      const float w = p.precision == 0 ? p.w[size_t(n) * K + k] : dequant(p.wq, p.wscale, p.precision, n, k, K);
      s = s + xr[k] * w;
    }
    base = s;
  }
  base = base + (p.bias ? p.bias[n] : 0.0f);
  float v = base;
  if (p.lora_b) {
    const float* mr = mid + size_t(m) * ldm;
    const float* br = p.lora_b + size_t(n) * p.rank;
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int rfull = (p.rank / 8) * 8;
    for (int r = 0; r < rfull; ++r) lanes[r & 7] = lanes[r & 7] + mr[r] * br[r];
    float d = -0.0f;
    for (int l = 0; l < 8; ++l) d = d + lanes[l];
    for (int r = rfull; r < p.rank; ++r) d = d + mr[r] * br[r];
    d = d + 0.0f;
    v = base + p.lora_scale * d;
  }
  float* o = out + size_t(m) * ldo + n;
  if (epi == kEpiWrite)
    *o = v;
  else if (epi == kEpiAdd)
    *o = *o + v;
  else
    *o = silu_f(*o) * v;
}

__global__ void embed_kernel(const void* table, int dtype, int hidden, const uint32_t* ids, float* x) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const size_t row = size_t(ids[t]) * hidden;
  for (int k = threadIdx.x; k < hidden; k += blockDim.x) {
    float v;
    if (dtype == 0)
      v = static_cast<const float*>(table)[row + k];
    else
      v = __uint_as_float(uint32_t(static_cast<const uint16_t*>(table)[row + k]) << 16);
    x[size_t(t) * hidden + k] = v;
  }
}

}  // namespace

void launch_norm_quant(const float* x, int ldx, int M, int K, const float* gamma, float eps, float* n_out, int ldn,
                       int8_t* xq, float* xs, int ldxs, DeviceStatus* st, cudaStream_t s) {
  if (M <= 0) return;
  if (K > 12288) throw CudaError("norm_quant: row too wide");
  const bool aligned = K % 128 == 0 && ldx % 4 == 0 && (!n_out || ldn % 4 == 0) &&
                       reinterpret_cast<uintptr_t>(x) % 16 == 0;
  const int blocks = (M + 7) / 8;
  if (aligned && !gamma && xq) {
    launch_pdl(norm_quant_warp_kernel<0>, dim3(dim3(blocks, (K / 128 + 3) / 4)), dim3(256), 0, s, x, ldx, M, K, nullptr, eps, n_out, ldn,
                                                                            xq, xs, ldxs, st);
  } else if (aligned && gamma && K == 2048) {
    // Two rows (warps) per CTA: 256 CTAs at 512 tokens spread over every SM.
    launch_pdl(norm_quant_warp_kernel<16>, dim3((M + 1) / 2), dim3(64), 0, s, x, ldx, M, K, gamma, eps, n_out, ldn, xq, xs, ldxs, st);
  } else {
    launch_pdl(norm_quant_kernel, dim3(M), dim3(256), K * sizeof(float), s, x, ldx, K, gamma, eps, n_out, ldn, xq, xs, ldxs, st);
  }
  DG_CUDA(cudaGetLastError());
}

void launch_gated_norm_quant(const float* o, const float* z, int ldz, int M, int heads, int dv, const float* w,
                             float eps, float* out, int8_t* xq, float* xs, int ldxs, bool quantize, DeviceStatus* st,
                             cudaStream_t s) {
  if (M <= 0) return;
  if (dv == 128) {
    const long warps = long(M) * heads;
    launch_pdl(gated_norm_quant_warp_kernel, dim3(int((warps + 7) / 8)), dim3(256), 0, s, o, z, ldz, M, heads, w, eps,
               out, xq, xs, ldxs, quantize ? 1 : 0, st);
  } else {
    launch_pdl(gated_norm_quant_kernel, dim3(M), dim3(256), heads * dv * sizeof(float), s, o, z, ldz, heads, dv, w,
               eps, out, xq, xs, ldxs, quantize ? 1 : 0, st);
  }
  DG_CUDA(cudaGetLastError());
}

void launch_lora_a(const float* x, int ldx, int M, int K, const float* A, int R, float* mid, int ldm, bool exact,
                   cudaStream_t s, float* partial, size_t partial_floats, DeviceStatus* st, bool overlap) {
  if (M <= 0 || R <= 0) return;
  const long threads = long((M + 3) / 4) * ((R + 3) / 4) * 8;
  const int blocks = int((threads + 255) / 256);
  if (exact && M <= 16) {
    // One row x one output per group of eight lanes: the head's few rows
    // still spread over R * M * 8 threads, in blocks of 64 so that they
    // reach many SMs, each lane with 16 steps of loads in flight (the chain
    // of one output lane is K / 8 dependent adds; its loads are not).
    const long t1 = long(M) * R * 8;
    launch_pdl(lora_a_kernel<true, 1, 1>, dim3(int((t1 + 63) / 64)), dim3(64), 0, s, x, ldx, M, K, A, R, mid, ldm);
  } else if (exact) {
    launch_k(overlap || pdl_enabled(), lora_a_kernel<true>, dim3(blocks), dim3(256), 0, s, x, ldx, M, K, A, R, mid,
             ldm);
  } else if (partial && lora_a_tc_supported(x, ldx, K, A, R, ldm)) {
    launch_lora_a_tc(x, ldx, M, K, A, R, mid, ldm, partial, partial_floats, st, s, overlap);
  } else if (partial && K % 32 == 0 && ldx % 4 == 0 && R % 4 == 0 && ldm % 4 == 0 &&
             reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0) {
    if (R <= 32)
      launch_lora_splitk<128, 32>(x, ldx, M, K, A, R, mid, ldm, partial, partial_floats, s);
    else if (R <= 64)
      launch_lora_splitk<64, 64>(x, ldx, M, K, A, R, mid, ldm, partial, partial_floats, s);
    else
      launch_lora_splitk<64, 128>(x, ldx, M, K, A, R, mid, ldm, partial, partial_floats, s);
  } else {
    const long warps = long((M + 3) / 4) * ((R + 3) / 4);
    launch_pdl(lora_a_fast_kernel, dim3(int((warps * 32 + 255) / 256)), dim3(256), 0, s, x, ldx, M, K, A, R, mid, ldm);
  }
  DG_CUDA(cudaGetLastError());
}

// The generic projection's FP32-dot precisions (checkpoint, int8 and int4
// weights, FP32 activations) as a tiled kernel: CTA = 32 rows x 64 outputs,
// 32-wide K chunks of x and of the (dequantised) weights in shared memory;
// thread (tid / 16, tid % 16) owns rows 2 t, 2 t + 1 and outputs c, c + 16,
// c + 32, c + 48, each with the eight dot_scores lanes of the reference
// (src/tensor.rs:6-25): lane k % 8 adds x[k] * w[k] in order of k, the lanes
// are summed in order from -0.0. Same arithmetic per output as
// proj_generic_kernel, bit for bit; K % 32 == 0.
constexpr int PGT_M = 32, PGT_N = 64, PGT_K = 32, PGT_LD = PGT_K + 1;
__global__ void __launch_bounds__(256) proj_generic_tiled_kernel(GenericProj p, const float* __restrict__ x, int ldx,
                                                                 const float* __restrict__ mid, int ldm, int M,
                                                                 float* __restrict__ out, int ldo, int epi) {
  griddep_wait();
  griddep_launch();
  __shared__ float xs_t[PGT_M][PGT_LD];
  __shared__ float ws_t[PGT_N][PGT_LD];
  const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
  const int m0 = blockIdx.y * PGT_M, n0 = blockIdx.x * PGT_N, K = p.in;
  float lanes[2][4][8];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int l = 0; l < 8; ++l) lanes[i][j][l] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += PGT_K) {
    __syncthreads();
    for (int i = tid; i < PGT_M * PGT_K; i += 256) {
      const int r = i / PGT_K, k = i % PGT_K;
      xs_t[r][k] = m0 + r < M ? x[size_t(m0 + r) * ldx + k0 + k] : 0.0f;
    }
    for (int i = tid; i < PGT_N * PGT_K; i += 256) {
      const int r = i / PGT_K, k = i % PGT_K, n = n0 + r;
      float w = 0.0f;
      if (n < p.out) w = p.precision == 0 ? p.w[size_t(n) * K + k0 + k] : dequant(p.wq, p.wscale, p.precision, n, k0 + k, K);
      ws_t[r][k] = w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < PGT_K; ++k) {
      const float a0 = xs_t[2 * tm][k], a1 = xs_t[2 * tm + 1][k];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float w = ws_t[tn + 16 * j][k];
        lanes[0][j][k & 7] = lanes[0][j][k & 7] + a0 * w;
        lanes[1][j][k & 7] = lanes[1][j][k & 7] + a1 * w;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int m = m0 + 2 * tm + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tn + 16 * j;
      if (m >= M || n >= p.out) continue;
      float sum = -0.0f;
#pragma unroll
      for (int l = 0; l < 8; ++l) sum = sum + lanes[i][j][l];
      const float base = sum + (p.bias ? p.bias[n] : 0.0f);
      float v = base;
      if (p.lora_b) {
        const float* mr = mid + size_t(m) * ldm;
        const float* br = p.lora_b + size_t(n) * p.rank;
        float ln[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int rfull = (p.rank / 8) * 8;
        for (int r = 0; r < rfull; ++r) ln[r & 7] = ln[r & 7] + mr[r] * br[r];
        float d = -0.0f;
        for (int l = 0; l < 8; ++l) d = d + ln[l];
        for (int r = rfull; r < p.rank; ++r) d = d + mr[r] * br[r];
        d = d + 0.0f;
        v = base + p.lora_scale * d;
      }
      float* o = out + size_t(m) * ldo + n;
      if (epi == kEpiWrite)
        *o = v;
      else if (epi == kEpiAdd)
        *o = *o + v;
      else
        *o = silu_f(*o) * v;
    }
  }
}

void launch_proj_generic(const GenericProj& p, const float* x, int ldx, const int8_t* xq, const float* xs, int ldxs,
                         const float* mid, int ldm, int M, float* out, int ldo, int epi, cudaStream_t s) {
  if (M <= 0) return;
  if (p.precision != 2 && p.in % PGT_K == 0) {
    dim3 grid((p.out + PGT_N - 1) / PGT_N, (M + PGT_M - 1) / PGT_M);
    launch_pdl(proj_generic_tiled_kernel, dim3(grid), dim3(256), 0, s, p, x, ldx, mid, ldm, M, out, ldo, epi);
  } else {
    dim3 grid((p.out + 127) / 128, M);
    launch_pdl(proj_generic_kernel, dim3(grid), dim3(128), 0, s, p, x, ldx, xq, xs, ldxs, mid, ldm, M, out, ldo, epi);
  }
  DG_CUDA(cudaGetLastError());
}

namespace {
__global__ void __launch_bounds__(256) proj_finish_kernel(const float* __restrict__ prod, int ldp,
                                                          const float* __restrict__ bias, float* out, int ldo,
                                                          int M, int N, int epi) {
  griddep_wait();
  griddep_launch();
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(M) * N) return;
  const int m = int(i / N), n = int(i % N);
  float v = prod[size_t(m) * ldp + n];
  if (bias) v = v + bias[n];
  float* o = out + size_t(m) * ldo + n;
  *o = epi == kEpiSwiGlu ? silu_f(*o) * v : v;
}
}  // namespace

void launch_proj_finish(const float* prod, int ldp, const float* bias, float* out, int ldo, int M, int N, int epi,
                        cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  const long total = long(M) * N;
  launch_pdl(proj_finish_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, prod, ldp, bias, out, ldo, M,
             N, epi);
  DG_CUDA(cudaGetLastError());
}

void launch_embed(const void* table, int dtype, int hidden, const uint32_t* ids, int n, float* x, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(embed_kernel, dim3(n), dim3(256), 0, s, table, dtype, hidden, ids, x);
  DG_CUDA(cudaGetLastError());
}

}  // namespace dg
