// Group-64 INT8 projection on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's linear_int8 / Kernel::scaled_dot / Adapter::combine /
// write_columns chain (src/tensor.rs:379-456,109-117,272-288; src/int8.rs:55-61):
//
//   out[m,n] = EPI( Σ_g float(dot_g(xq[m], wq[n])) * (xs[m,g] * ws[n,g])  + 0.0
//                   + lora_scale * (dot_scores(mid[m, pid(n)], lora_b[n]) + 0.0) )
//
// One CTA owns a 128 x 256 output tile; 12 warps (3 warpgroups):
//   warp 0      TMA producer: int8 A/B tiles (128-byte swizzle) plus the two
//               groups' activation and weight scales, 3-stage ring;
//   warp 1      TMEM allocator and single-thread MMA issuer: per 64-wide K group,
//               two tcgen05.mma kind::i8 (K=32) into a fresh int32 accumulator,
//               double-buffered in TMEM (2 x 256 columns);
//   warps 2-3   no role (the block is sized in whole warpgroups);
//   warps 4-11  promotion/epilogue: per group, tcgen05.ld the exact int32 dots,
//               scale them in FP32 in group order (reference order when EXACT).
//               After the last group the FP32 sums move to shared memory (the
//               drained stage ring), and each thread finishes its row: LoRA-B,
//               the epilogue and the store.
// Every wait is bounded (mbar_wait_bounded); a stall records kWaitTimeout.
#pragma once
#include "common.cuh"

namespace dg {

struct GemmArgs {
  int M, N, K;              // N is a multiple of 256, K a multiple of 128
  const float* xs;          // activation scales [K/64][ldxs]
  int ldxs;                 // >= round_up(M, 128)
  const float* ws;          // weight scales [K/64][N]
  const float* lora_mid;    // [M][ld_mid] LoRA-A outputs (nullable when R == 0)
  int ld_mid;
  const float* lora_b;      // [N][R]
  const int* chunk_pid;     // [N/32] LoRA block index of each 32-column chunk
  float lora_scale;
  float* out;               // WRITE/ADD: [M][ldo] (N columns); SWIGLU: [M][ldo] (N/2 columns)
  int ldo;
  DeviceStatus* status;
  int32_t* dots;            // optional debug dump of the exact group dots [K/64][M][N]
};

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 128;    // BK bytes = two 64-wide groups
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
constexpr int WS_OFF = A_BYTES + B_BYTES;            // [2][BN] floats
constexpr int XS_OFF = WS_OFF + 2 * BN * 4;          // [2][BM] floats
constexpr int STAGE_BYTES = XS_OFF + 2 * BM * 4;     // 52224 = 51 KiB
constexpr int STAGE_TX = STAGE_BYTES;
constexpr int LORA_OFF = STAGES * STAGE_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4, EPI_WARPS = 8;
constexpr int ACC_LD = BN + 1;                       // padded row stride of the FP32 sums in smem
constexpr uint32_t TMEM_COLS = 512;
static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment for SWIZZLE_128B");
static_assert(BM * ACC_LD * 4 <= STAGES * STAGE_BYTES, "FP32 sums must fit in the drained stage ring");
__host__ __device__ constexpr int lora_bytes(int R) { return BN * R * 4; }
__host__ __device__ constexpr int bar_off(int R) { return LORA_OFF + lora_bytes(R); }
__host__ __device__ constexpr int smem_bytes(int R) { return bar_off(R) + 128 + 1024; }
}  // namespace gemm

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(gemm::EPI_WARPS * 32) : "memory");
}

template <int R, int EPI, bool EXACT>
__global__ void __launch_bounds__(gemm::NUM_THREADS, 1)
    gemm_i8_g64_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       GemmArgs p) {
  using namespace gemm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_off(R));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* lora_smem = reinterpret_cast<float*>(smem + LORA_OFF);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int G = p.K / 64, KS = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  if (R > 0 && warp >= EPI_WARP0) {
    // Stage this tile's LoRA-B rows [BN][R] (contiguous in global memory).
    const float4* src = reinterpret_cast<const float4*>(p.lora_b + size_t(n0) * R);
    float4* dst = reinterpret_cast<float4*>(lora_smem);
    for (int i = threadIdx.x - EPI_WARP0 * 32; i < BN * R / 4; i += EPI_WARPS * 32) dst[i] = src[i];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int issued = 0;
      for (int ks = 0; ks < KS; ++ks) {
        const int s = ks % STAGES, use = ks / STAGES;
        if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, p.status, 100 + s, abort_flag)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], STAGE_TX);
        tma_load_2d(st, &map_a, &full[s], ks * BK, m0);
        tma_load_2d(st + A_BYTES, &map_b, &full[s], ks * BK, n0);
        for (int j = 0; j < 2; ++j) {
          const int g = 2 * ks + j;
          bulk_load(st + WS_OFF + j * BN * 4, p.ws + size_t(g) * p.N + n0, BN * 4, &full[s]);
          bulk_load(st + XS_OFF + j * BM * 4, p.xs + size_t(g) * p.ldxs + m0, BM * 4, &full[s]);
        }
        issued = ks + 1;
      }
      if (*abort_flag) {
        // Let this CTA's copies in flight land before the CTA exits.
        for (int ks = (issued > STAGES ? issued - STAGES : 0); ks < issued; ++ks)
          mbar_wait_bounded(&full[ks % STAGES], (ks / STAGES) & 1, p.status, 190, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      bool ok = true;
      for (int g = 0; g < G && ok; ++g) {
        const int ks = g / 2, s = ks % STAGES, b = g & 1, use = g / 2;
        if ((g & 1) == 0) ok = mbar_wait_bounded(&full[s], (ks / STAGES) & 1, p.status, 200 + s, abort_flag);
        if (ok && use > 0) ok = mbar_wait_bounded(&tempty[b], (use - 1) & 1, p.status, 210 + b, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_addr(smem + s * STAGE_BYTES) + (g & 1) * 64;
        const uint32_t b_addr = a_addr + A_BYTES;
        const uint32_t d = tmem_base + uint32_t(b * BN);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          mma_i8(d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), idesc, kk);
        mma_commit(&tfull[b]);
        if (g & 1) mma_commit(&empty[s]);
      }
      // All MMAs of this thread have completed once mma_done flips.
      mma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status, 220, nullptr);
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- promotion (warps 4..11)
    const int q = warp & 3;                       // TMEM lane quarter this warp may read
    const int half = (warp - EPI_WARP0) >> 2;     // which 128 columns of the tile
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
    bool ok = true;
    for (int g = 0; g < G; ++g) {
      const int ks = g / 2, s = ks % STAGES, b = g & 1, use = g / 2;
      ok = mbar_wait_bounded(&full[s], (ks / STAGES) & 1, p.status, 300 + s, abort_flag) &&
           mbar_wait_bounded(&tfull[b], use & 1, p.status, 310 + b, abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint8_t* st = smem + s * STAGE_BYTES;
      const float xsg = reinterpret_cast<const float*>(st + XS_OFF)[(g & 1) * BM + row];
      const float* wsg = reinterpret_cast<const float*>(st + WS_OFF) + (g & 1) * BN + half * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t d[16];
        tmem_ld_32x32b_x16(lane_addr + uint32_t(b * BN + half * 128 + c * 16), d);
        tmem_wait_ld();
        if (p.dots != nullptr && m < p.M) {
          int4* dd = reinterpret_cast<int4*>(p.dots + (size_t(g) * p.M + m) * p.N + n0 + half * 128 + c * 16);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4)
            dd[j4] = make_int4(int(d[j4 * 4]), int(d[j4 * 4 + 1]), int(d[j4 * 4 + 2]), int(d[j4 * 4 + 3]));
        }
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const float4 w4 = reinterpret_cast<const float4*>(wsg + c * 16)[j4];
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j4 * 4 + e;
            const float sc = xsg * wv[e];
            const float fd = i32_to_f32_small(int32_t(d[j]));
            if (EXACT)
              acc[c * 16 + j] = __fadd_rn(acc[c * 16 + j], __fmul_rn(fd, sc));
            else
              acc[c * 16 + j] = __fmaf_rn(fd, sc, acc[c * 16 + j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[b]);
        if (g & 1) mbar_arrive(&empty[s]);
      }
    }
    // ---------------- epilogue: sums to shared memory, then per-row finish.
    // All stages are drained once every promotion warp has left the loop.
    epi_bar_sync();
    float* accs = reinterpret_cast<float*>(smem) + size_t(row) * ACC_LD + half * 128;
    if (ok) {
      // Bias-free projections add 0.0 as the reference does (src/tensor.rs:437).
#pragma unroll
      for (int j = 0; j < 128; ++j) accs[j] = __fadd_rn(acc[j], 0.0f);
    }
    __syncwarp();
    if (ok && m < p.M) {
      float vals[32];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col0 = half * 128 + c * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] = accs[c * 32 + j];
        if (R > 0) {
          const int pid = p.chunk_pid[(n0 + col0) >> 5];
          float mid[R > 0 ? R : 1];
          const float4* mp = reinterpret_cast<const float4*>(p.lora_mid + size_t(m) * p.ld_mid + pid * R);
#pragma unroll
          for (int r4 = 0; r4 < R / 4; ++r4) {
            const float4 v = mp[r4];
            mid[r4 * 4] = v.x; mid[r4 * 4 + 1] = v.y; mid[r4 * 4 + 2] = v.z; mid[r4 * 4 + 3] = v.w;
          }
#pragma unroll 4
          for (int j = 0; j < 32; ++j) {
            const float4* bl = reinterpret_cast<const float4*>(lora_smem + (col0 + j) * R);
            if (EXACT) {
              // dot_scores order (src/tensor.rs:6-25): eight lanes, then their sum.
              float lanes[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) lanes[i] = 0.0f;
#pragma unroll
              for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 w = bl[r4];
                const float wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int r = r4 * 4 + e;
                  lanes[r & 7] = __fadd_rn(lanes[r & 7], __fmul_rn(mid[r], wv[e]));
                }
              }
              float delta = -0.0f;
#pragma unroll
              for (int i = 0; i < 8; ++i) delta = __fadd_rn(delta, lanes[i]);
              delta = __fadd_rn(delta, 0.0f);
              vals[j] = __fadd_rn(vals[j], __fmul_rn(p.lora_scale, delta));
            } else {
              float delta = 0.0f;
#pragma unroll
              for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 w = bl[r4];
                delta = __fmaf_rn(mid[r4 * 4], w.x, delta);
                delta = __fmaf_rn(mid[r4 * 4 + 1], w.y, delta);
                delta = __fmaf_rn(mid[r4 * 4 + 2], w.z, delta);
                delta = __fmaf_rn(mid[r4 * 4 + 3], w.w, delta);
              }
              vals[j] = __fmaf_rn(p.lora_scale, delta, vals[j]);
            }
          }
        }
        if (EPI == kEpiSwiGlu) {
          // Columns [0,64) of this half hold gate, [64,128) the matching up
          // values: keep the gate chunks in shared memory, combine on up chunks.
          if (c < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) accs[c * 32 + j] = vals[j];
          } else {
            float* o = p.out + size_t(m) * p.ldo + (n0 >> 1) + half * 64 + (c - 2) * 32;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              float4 v;
              v.x = silu_f(accs[(c - 2) * 32 + j4 * 4 + 0]) * vals[j4 * 4 + 0];
              v.y = silu_f(accs[(c - 2) * 32 + j4 * 4 + 1]) * vals[j4 * 4 + 1];
              v.z = silu_f(accs[(c - 2) * 32 + j4 * 4 + 2]) * vals[j4 * 4 + 2];
              v.w = silu_f(accs[(c - 2) * 32 + j4 * 4 + 3]) * vals[j4 * 4 + 3];
              reinterpret_cast<float4*>(o)[j4] = v;
            }
          }
        } else {
          float4* o = reinterpret_cast<float4*>(p.out + size_t(m) * p.ldo + n0 + col0);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            float4 v = make_float4(vals[j4 * 4], vals[j4 * 4 + 1], vals[j4 * 4 + 2], vals[j4 * 4 + 3]);
            if (EPI == kEpiAdd) {
              const float4 old = o[j4];
              v.x = __fadd_rn(old.x, v.x); v.y = __fadd_rn(old.y, v.y);
              v.z = __fadd_rn(old.z, v.z); v.w = __fadd_rn(old.w, v.w);
            }
            o[j4] = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace dg
