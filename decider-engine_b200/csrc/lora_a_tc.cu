// LoRA A on the tensor cores, fast mode: mid = x · Aᵀ for the fused LoRA
// parts of one projection (x [M][K] FP32, A [R][K] FP32, R <= 128), the
// counterpart of the reference's per-row Adapter::scores (src/tensor.rs:6-25,
// 272-288) computed as one skinny GEMM.
//
// Split K over the grid so the skinny [M x R] product still fills the GPU:
// CTA (t, z) owns rows 128 t .. 128 t + 127 and the K slice z. Per 32-wide K
// chunk its 256 threads gather the x rows and A rows into registers
// (coalesced 16-byte loads; the next one or two chunks' loads are in flight
// while the current chunk is stored), split every value into its TF32 part (low 13
// mantissa bits cleared) and the remainder, and store both in the
// 128-byte-swizzled K-major layout the tensor cores read; one thread issues
// hi·hi + hi·lo + lo·hi as tcgen05.mma kind::tf32 (M = 128, N = R rounded up
// to 16) into one TMEM accumulator; two chunk slots alternate. The partial
// product goes to partial[z][M][R] and lora_a_reduce_kernel adds the slices
// in a fixed order (deterministic).
#include "common.cuh"
#include "launch.h"

namespace dg {
namespace {

constexpr int kLaThreads = 256;

__host__ __device__ constexpr int lora_tc_slot_bytes(int np) { return 2 * 16384 + 2 * np * 128; }
__host__ __device__ constexpr int lora_tc_smem_bytes(int np) { return 2 * lora_tc_slot_bytes(np) + 64 + 1024; }

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float tf32_part(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// Gathers 32-wide K chunk `k` of the x rows m0.. and the A rows into v.
__device__ __forceinline__ void lora_tc_gather(float4 (&v)[8], const float* __restrict__ x, int ldx, int M, int m0,
                                               const float* __restrict__ A, int R, int K, int k, int items, int tid) {
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i = tid + u * kLaThreads;
    v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (i < items) {
      const int r = i >> 3, j = i & 7;
      if (r < 128) {
        if (m0 + r < M) v[u] = ldg4(x + size_t(m0 + r) * ldx + k + 4 * j);
      } else if (r - 128 < R) {
        v[u] = ldg4(A + size_t(r - 128) * K + k + 4 * j);
      }
    }
  }
}

// DEPTH: chunks of loads in flight ahead of the one being stored (2 for
// CTAs of at most four chunks, where the first loads dominate; 1 otherwise,
// measured slightly faster for longer slices).
template <int DEPTH>
__global__ void __launch_bounds__(kLaThreads, 1)
    lora_a_tc_kernel(const float* __restrict__ x, int ldx, int M, int K, const float* __restrict__ A, int R, int NP,
                     float* __restrict__ partial, int kslice, DeviceStatus* st) {
  extern __shared__ __align__(1024) uint8_t la_raw[];
  uint8_t* sm = la_raw + ((1024u - (smem_addr(la_raw) & 1023u)) & 1023u);
  const int slot = lora_tc_slot_bytes(NP);
  uint64_t* done = reinterpret_cast<uint64_t*>(sm + 2 * slot);  // [2]: MMAs of the slot's chunk complete
  uint32_t* holder = reinterpret_cast<uint32_t*>(done + 2);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int m0 = blockIdx.x * 128;
  const int k0 = blockIdx.y * kslice;
  const int nch = max(0, min(K, k0 + kslice) - k0) / 32;
  const uint32_t ncols = NP <= 32 ? 32u : NP <= 64 ? 64u : 128u;
  if (tid == 0) {
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(holder, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  griddep_wait();  // set-up above touched only shared memory and TMEM
  griddep_launch();
  const uint32_t idesc = idesc_tf32(128, uint32_t(NP));
  const int items = (128 + NP) * 8;  // 16-byte pieces per chunk: x rows, then A rows
  bool ok = true;
  float4 v[8], w[8];
  if (nch > 0) lora_tc_gather(v, x, ldx, M, m0, A, R, K, k0, items, tid);
  if (DEPTH == 2 && nch > 1) lora_tc_gather(w, x, ldx, M, m0, A, R, K, k0 + 32, items, tid);
  for (int c = 0; c < nch; ++c) {
    const int b = c & 1;
    uint8_t* s = sm + b * slot;
    float4 nxt[8];
    if (c + DEPTH < nch) lora_tc_gather(nxt, x, ldx, M, m0, A, R, K, k0 + 32 * (c + DEPTH), items, tid);
    // The slot was last read by the MMAs of chunk c - 2.
    if (c >= 2) ok = mbar_wait_bounded(&done[b], ((c - 2) >> 1) & 1, st, 400 + b, nullptr) && ok;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * kLaThreads;
      if (i < items) {
        const int r = i >> 3, j = i & 7;
        const bool is_x = r < 128;
        const int rr = is_x ? r : r - 128;
        uint8_t* hi = s + (is_x ? 0 : 32768);
        uint8_t* lo = hi + (is_x ? 16384 : NP * 128);
        // 128-byte swizzle: 16-byte piece j of row rr sits at piece j ^ (rr % 8).
        const int off = rr * 128 + ((j ^ (rr & 7)) << 4);
        const float4 h = make_float4(tf32_part(v[u].x), tf32_part(v[u].y), tf32_part(v[u].z), tf32_part(v[u].w));
        *reinterpret_cast<float4*>(hi + off) = h;
        *reinterpret_cast<float4*>(lo + off) = make_float4(v[u].x - h.x, v[u].y - h.y, v[u].z - h.z, v[u].w - h.w);
      }
    }
    fence_proxy_async_smem();  // generic-proxy stores, read by the MMAs (async proxy)
    __syncthreads();
    if (tid == 0) {
      if (ok) {
        tc_fence_after();
        const uint32_t xa = smem_addr(s), aa = xa + 32768;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t xh = xa + kk * 32, xl = xh + 16384, ah = aa + kk * 32, al = ah + NP * 128;
          mma_tf32(tmem, smem_desc_sw128(xh), smem_desc_sw128(ah), idesc, (c > 0 || kk > 0) ? 1u : 0u);
          mma_tf32(tmem, smem_desc_sw128(xh), smem_desc_sw128(al), idesc, 1u);
          mma_tf32(tmem, smem_desc_sw128(xl), smem_desc_sw128(ah), idesc, 1u);
        }
      }
      mma_commit(&done[b]);  // also after a failed wait, so that every later wait ends
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (DEPTH == 2) {
        v[u] = w[u];
        w[u] = nxt[u];
      } else {
        v[u] = nxt[u];
      }
    }
  }
  // The last commit covers every MMA of the issuing thread.
  if (nch > 0 && !mbar_wait_bounded(&done[(nch - 1) & 1], ((nch - 1) >> 1) & 1, st, 410, nullptr)) ok = false;
  tc_fence_after();
  if (warp < 4) {
    const int r = warp * 32 + lane, m = m0 + r;
    float* out = partial + size_t(blockIdx.y) * M * R + size_t(m) * R;
    for (int cc = 0; cc < NP / 16; ++cc) {
      uint32_t d[16];
      tmem_ld16_sync(tmem + (uint32_t(warp * 32) << 16) + uint32_t(16 * cc), d);
      if (m < M) {
        const bool has = nch > 0 && ok;  // an empty slice contributes zero
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          const int col = 16 * cc + e;
          if (col < R)
            *reinterpret_cast<float4*>(out + col) =
                has ? make_float4(__uint_as_float(d[e]), __uint_as_float(d[e + 1]), __uint_as_float(d[e + 2]),
                                  __uint_as_float(d[e + 3]))
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

}  // namespace

size_t lora_a_tc_partial_floats(int max_rows) {
  const size_t mt = size_t(max_rows + 127) / 128;
  return (148 + mt) * 128 * 128;
}

bool lora_a_tc_supported(const float* x, int ldx, int K, const float* A, int R, int ldm) {
  return R > 0 && R <= 128 && R % 4 == 0 && K % 32 == 0 && ldx % 4 == 0 && ldm % 4 == 0 &&
         reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0;
}

void launch_lora_a_tc(const float* x, int ldx, int M, int K, const float* A, int R, float* mid, int ldm,
                      float* partial, size_t partial_floats, DeviceStatus* st, cudaStream_t s, bool overlap) {
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    DG_CUDA(cudaFuncSetAttribute(lora_a_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 lora_tc_smem_bytes(128)));
    DG_CUDA(cudaFuncSetAttribute(lora_a_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 lora_tc_smem_bytes(128)));
  });
  const int NP = (R + 15) / 16 * 16;
  const int mt = (M + 127) / 128;
  // The grid fills the GPU. With `overlap` the kernels are launched as
  // programmatic prerequisites of the next projection (measured: confining
  // them to a third of the SMs instead delays that projection's first wave
  // by more than it gains).
  const int splits = std::max(1, std::min(K / 32, (148 + mt - 1) / mt));
  const int kslice = ((K + splits - 1) / splits + 31) / 32 * 32;
  const int used = (K + kslice - 1) / kslice;
  if (size_t(used) * M * R > partial_floats) throw CudaError("lora_a: split-K workspace too small");
  launch_k(overlap || pdl_enabled(), kslice / 32 <= 4 ? lora_a_tc_kernel<2> : lora_a_tc_kernel<1>, dim3(mt, used),
           dim3(kLaThreads), lora_tc_smem_bytes(NP), s, x, ldx, M, K, A, R, NP, partial, kslice, st);
  DG_CUDA(cudaGetLastError());
  launch_lora_a_reduce(partial, used, M, R, mid, ldm, s, overlap);
}

}  // namespace dg
