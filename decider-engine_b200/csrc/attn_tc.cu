// Causal GQA attention on the tensor cores, fast (FMA) mode: the product of
// Full::forward's causal_attention (src/qwen.rs:590-643) and the output gate
// (src/qwen.rs:581-583) as three kernels per query chunk:
//   1. S = Q·Kᵀ / sqrt(d)         tc_gemm_kernel (3 x TF32 tcgen05, FP32 accumulate)
//   2. P = softmax(S), causal     softmax_rows_kernel (one warp per row)
//   3. out = (P·V) · sigmoid(gate) tc_gemm_kernel with the gate in its epilogue
// plus a transpose of V into Vᵀ [kv head][d][keys] so both products read
// K-major operands.
//
// tc_gemm_kernel: C[m][n] = alpha · Σ_k A[m][k] · B[n][k] (+ C, · sigmoid(G)),
// FP32 in and out. CTA = 128 x 128 output tile; 32-wide K chunks are gathered
// by all 256 threads (16-byte loads, the next chunk in flight while the
// current one is stored), split into the TF32 part (low 13 mantissa bits
// cleared) and the remainder, and stored in the 128-byte-swizzled K-major
// layout; one thread issues the chunk's tcgen05.mma kind::tf32 (M = N = 128,
// K = 8): hi·hi into one TMEM accumulator, the correction hi·lo + lo·hi into
// a second. The tensor core's FP32 accumulation does not round to nearest, so
// long chains of it drift: each chunk therefore starts fresh accumulators
// (two buffers of the pair, alternating), and once its MMAs complete every
// thread reads its rows' values and adds main + correction into its FP32
// register sums, rounding to nearest. Error per product about 2^-21; per
// output, a few TF32-chain steps plus the FP32 sum of the chunks.
// Batches (grid.z) index heads and sequences through per-operand offsets.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace dg {
namespace {

constexpr int kTcThreads = 256;
constexpr int kTcSlot = 4 * 16384;                 // A hi, A lo, B hi, B lo: 128 rows x 128 B each
constexpr int kTcSmem = 2 * kTcSlot + 64 + 1024;   // two slots, barriers, 1024-byte alignment

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(TcGemmArgs g) {
  extern __shared__ __align__(1024) uint8_t tc_raw[];
  uint8_t* sm = tc_raw + ((1024u - (smem_addr(tc_raw) & 1023u)) & 1023u);
  uint64_t* done = reinterpret_cast<uint64_t*>(sm + 2 * kTcSlot);  // [2]: MMAs of the slot's chunk complete
  uint32_t* holder = reinterpret_cast<uint32_t*>(done + 2);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * 128;
  const int outer = int(blockIdx.z) / g.inner_count, inner = int(blockIdx.z) % g.inner_count;
  // Causal tiles: row m sees columns (keys) up to diag + m.
  if (g.diag >= 0 && !g.k_causal && n0 > g.diag + m0 + 127) return;  // the whole tile is masked
  int kend = g.K;
  if (g.diag >= 0 && g.k_causal) kend = min(g.K, (g.diag + m0 + 128 + 31) / 32 * 32);
  const int nch = max(0, kend) / 32;
  const float* A = g.A + outer * g.a_outer + inner * g.a_inner;
  const float* B = g.B + outer * g.b_outer + (inner / g.b_inner_div) * g.b_inner;
  if (tid == 0) {
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(holder, 512);  // [2 buffers][main, correction] x 128 columns
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  griddep_wait();  // set-up above touched only shared memory and TMEM
  griddep_launch();
  constexpr uint32_t idesc = idesc_tf32(128, 128);
  // 16-byte pieces of one chunk: 128 A rows then 128 B rows, 8 pieces each.
  auto gather = [&](float4 (&v)[8], int k) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * kTcThreads, r = i >> 3, j = i & 7;
      v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (r < 128) {
        if (m0 + r < g.M) v[u] = ldg4(A + size_t(m0 + r) * g.lda + k + 4 * j);
      } else if (n0 + r - 128 < g.N) {
        v[u] = ldg4(B + size_t(n0 + r - 128) * g.ldb + k + 4 * j);
      }
    }
  };
  // Warps w and w + 4 read TMEM lanes 32 (w % 4) ..: columns 0-63 and 64-127.
  const int q = warp & 3, half = warp >> 2;
  const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16) + uint32_t(half * 64);
  float acc[64];
#pragma unroll
  for (int e = 0; e < 64; ++e) acc[e] = 0.0f;
  bool ok = true;
  // Adds chunk c's products (buffer c & 1) into acc once its MMAs are complete.
  auto take = [&](int c) {
    const int b = c & 1;
    ok = mbar_wait_bounded(&done[b], (c >> 1) & 1, g.status, 500 + b, nullptr) && ok;
    tc_fence_after();
    const uint32_t base = lane_base + uint32_t(b * 256);
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t dm[16], dc[16];
      tmem_ld16x2_sync(base + uint32_t(16 * cc), base + 128u + uint32_t(16 * cc), dm, dc);
#pragma unroll
      for (int e = 0; e < 16; ++e)
        acc[16 * cc + e] = acc[16 * cc + e] + (__uint_as_float(dm[e]) + __uint_as_float(dc[e]));
    }
    tc_fence_before();
  };
  float4 v[8];
  if (nch > 0) gather(v, 0);
  for (int c = 0; c < nch; ++c) {
    const int b = c & 1;
    uint8_t* s = sm + b * kTcSlot;
    float4 w[8];
    if (c + 1 < nch) gather(w, 32 * (c + 1));
    // Slot and accumulator buffer b were last used by chunk c - 2: add its
    // products, which also frees both.
    if (c >= 2) take(c - 2);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * kTcThreads, r = i >> 3, j = i & 7;
      const int rr = r & 127;
      uint8_t* hi = s + (r < 128 ? 0 : 32768);
      uint8_t* lo = hi + 16384;
      // 128-byte swizzle: 16-byte piece j of row rr sits at piece j ^ (rr % 8).
      const int off = rr * 128 + ((j ^ (rr & 7)) << 4);
      const float4 h = make_float4(tf32_hi(v[u].x), tf32_hi(v[u].y), tf32_hi(v[u].z), tf32_hi(v[u].w));
      *reinterpret_cast<float4*>(hi + off) = h;
      *reinterpret_cast<float4*>(lo + off) = make_float4(v[u].x - h.x, v[u].y - h.y, v[u].z - h.z, v[u].w - h.w);
    }
    fence_proxy_async_smem();  // generic-proxy stores, read by the MMAs (async proxy)
    __syncthreads();
    if (tid == 0) {
      if (ok) {
        tc_fence_after();
        const uint32_t aa = smem_addr(s), ba = aa + 32768;
        const uint32_t dmain = tmem + uint32_t(b * 256), dcorr = dmain + 128u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t ah = aa + kk * 32, al = ah + 16384, bh = ba + kk * 32, bl = bh + 16384;
          mma_tf32(dmain, smem_desc_sw128(ah), smem_desc_sw128(bh), idesc, kk > 0 ? 1u : 0u);
          mma_tf32(dcorr, smem_desc_sw128(ah), smem_desc_sw128(bl), idesc, kk > 0 ? 1u : 0u);
          mma_tf32(dcorr, smem_desc_sw128(al), smem_desc_sw128(bh), idesc, 1u);
        }
      }
      mma_commit(&done[b]);  // also after a failed wait, so that every later wait ends
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = w[u];
  }
  if (nch >= 2) take(nch - 2);
  if (nch >= 1) take(nch - 1);
  {
    const int r = q * 32 + lane, m = m0 + r;
    float* C = g.C + outer * g.c_outer + inner * g.c_inner + size_t(m) * g.ldc;
    const float* G = g.gate ? g.gate + outer * g.g_outer + inner * g.g_inner + size_t(m) * g.ldg : nullptr;
    const bool has = nch > 0 && ok;  // no chunk: the product is zero
    if (m < g.M) {
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const int n = n0 + half * 64 + e;
        if (n < g.N) {
          float val = has ? acc[e] * g.alpha : 0.0f;
          if (g.accumulate) val = C[n] + val;
          if (G) val = val * sigmoid_f(G[n]);
          C[n] = val;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Row softmax in place over S [heads][M][ld]: row m of head h keeps columns
// [0, min(N, diag + m + 1)) (the causal window), P = exp(s - max) / Σ, and
// zeros up to ld (the padded K extent of the P·V product). One warp per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float* __restrict__ S, int ld, long head_stride, int M,
                                                           int N, int diag, int heads) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x % 32;
  if (row >= M * heads) return;
  const int h = row / M, m = row % M;
  float* s = S + h * head_stride + size_t(m) * ld;
  const int lim = min(N, diag + m + 1);
  float mx = -INFINITY;
  for (int j = lane; j < lim; j += 32) mx = fmaxf(mx, s[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.0f;
  for (int j = lane; j < lim; j += 32) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  for (int j = lane; j < ld; j += 32) s[j] = j < lim ? s[j] * inv : 0.0f;
}

// Vᵀ [kv][d][ld] from V rows [L][kv * d] (keys 0..L-1, zero to ld), in
// 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) transpose_v_kernel(const float* __restrict__ V, int L, int kv, int d,
                                                          float* __restrict__ Vt, int ld) {
  griddep_wait();
  griddep_launch();
  __shared__ float tile[32][33];
  const int k0 = blockIdx.x * 32, c0 = blockIdx.y * 32, kh = blockIdx.z;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  for (int r = ty; r < 32; r += 8) {
    const int key = k0 + r;
    tile[r][tx] = key < L ? V[size_t(key) * kv * d + kh * d + c0 + tx] : 0.0f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int key = k0 + tx;
    if (key < ld) Vt[(size_t(kh) * d + c0 + r) * ld + key] = tile[tx][r];
  }
}

}  // namespace

void launch_tc_gemm(const TcGemmArgs& g, int batches, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || batches <= 0) return;
  if (g.K % 32 || g.lda % 4 || g.ldb % 4 || reinterpret_cast<uintptr_t>(g.A) % 16 ||
      reinterpret_cast<uintptr_t>(g.B) % 16 || g.a_outer % 4 || g.a_inner % 4 || g.b_outer % 4 || g.b_inner % 4 ||
      g.inner_count <= 0 || g.b_inner_div <= 0)
    throw CudaError("tc_gemm: K must be a multiple of 32 and the operands 16-byte aligned");
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    DG_CUDA(cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
  });
  dim3 grid((g.M + 127) / 128, (g.N + 127) / 128, batches);
  launch_pdl(tc_gemm_kernel, grid, dim3(kTcThreads), kTcSmem, s, g);
  DG_CUDA(cudaGetLastError());
}

size_t attention_tc_workspace_floats(int heads, int kv_heads, int d, int max_rows) {
  const size_t qc = size_t(std::min(max_rows, kAttnTcChunk));
  return size_t(heads) * qc * 4096 + size_t(kv_heads) * d * 4096;
}

bool attention_tc_supported(int d, int heads, int kv_heads) {
  return d == 256 && kv_heads > 0 && heads % kv_heads == 0;
}

void launch_attention_tc(const float* q, const float* kc, const float* vc, const float* gate_src, int ld_gate, int n,
                         int offset, int heads, int kv_heads, int d, float* out, float* ws, size_t ws_floats,
                         DeviceStatus* st, cudaStream_t s) {
  if (n <= 0) return;
  const int L = offset + n, ld = (L + 31) / 32 * 32, kw = kv_heads * d;
  const int qc = std::min(n, kAttnTcChunk);
  if (!attention_tc_supported(d, heads, kv_heads) || L > 4096 ||
      size_t(heads) * qc * ld + size_t(kv_heads) * d * ld > ws_floats)
    throw CudaError("attention_tc: unsupported shape or workspace too small");
  float* S = ws;                                   // [heads][qc][ld]
  float* Vt = ws + size_t(heads) * qc * ld;        // [kv][d][ld]
  launch_pdl(transpose_v_kernel, dim3(ld / 32, d / 32, kv_heads), dim3(256), 0, s, vc, L, kv_heads, d, Vt, ld);
  DG_CUDA(cudaGetLastError());
  const int group = heads / kv_heads;
  for (int q0 = 0; q0 < n; q0 += qc) {
    const int rows = std::min(qc, n - q0), keys = offset + q0 + rows;
    // S[h][m][j] = q[q0 + m][h] · k[j][h / group] / sqrt(d)
    TcGemmArgs a{};
    a.A = q + size_t(q0) * heads * d;
    a.lda = heads * d;
    a.a_inner = d;
    a.B = kc;
    a.ldb = kw;
    a.b_inner = d;
    a.b_inner_div = group;
    a.C = S;
    a.ldc = ld;
    a.c_inner = long(qc) * ld;
    a.M = rows;
    a.N = keys;
    a.K = d;
    a.alpha = 1.0f / sqrtf(float(d));
    a.inner_count = heads;
    a.diag = offset + q0;
    a.status = st;
    launch_tc_gemm(a, heads, s);
    launch_pdl(softmax_rows_kernel, dim3((rows * heads + 7) / 8), dim3(256), 0, s, S, ld, long(qc) * ld, rows, keys,
               offset + q0, heads);
    DG_CUDA(cudaGetLastError());
    // out[q0 + m][h][c] = (Σ_j P[h][m][j] · Vt[h / group][c][j]) · sigmoid(gate[q0 + m][h][d + c])
    TcGemmArgs b{};
    b.A = S;
    b.lda = ld;
    b.a_inner = long(qc) * ld;
    b.B = Vt;
    b.ldb = ld;
    b.b_inner = long(d) * ld;
    b.b_inner_div = group;
    b.C = out + size_t(q0) * heads * d;
    b.ldc = heads * d;
    b.c_inner = d;
    b.M = rows;
    b.N = d;
    b.K = ld;
    b.alpha = 1.0f;
    b.inner_count = heads;
    b.diag = offset + q0;
    b.k_causal = 1;
    b.gate = gate_src + size_t(q0) * ld_gate + d;
    b.ldg = ld_gate;
    b.g_inner = 2 * d;
    b.status = st;
    launch_tc_gemm(b, heads, s);
  }
}

}  // namespace dg
