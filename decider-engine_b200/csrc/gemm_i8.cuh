// Group-64 INT8 projection on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's linear_int8 / Kernel::scaled_dot / Adapter::combine /
// write_columns chain (src/tensor.rs:379-456,109-117,272-288; src/int8.rs:55-61):
//
//   out[m,n] = EPI( Σ_g float(dot_g(xq[m], wq[n])) * (xs[m,g] * ws[n,g])  + 0.0
//                   + lora_scale * (dot_scores(mid[m, pid(n)], lora_b[n]) + 0.0) )
//
// One CTA owns a 128 x BN output tile (BN = 256, or 64 for narrow outputs so
// more SMs share the work); 20 warps (5 warpgroups):
//   warp 0      TMA producer: int8 A/B tiles (128-byte swizzle) plus the two
//               groups' activation and weight scales, multi-stage ring;
//   warp 1      TMEM allocator and single-thread MMA issuer: per 64-wide K group,
//               two tcgen05.mma kind::i8 (K=32) into a fresh int32 accumulator,
//               double-buffered in TMEM (2 x BN columns);
//   warps 2-3   no role (the block is sized in whole warpgroups);
//   warps 4-19  promotion/epilogue, four per TMEM lane quarter, each owning a
//               quarter of the tile's columns: per group, tcgen05.ld the exact int32 dots and
//               scale them in FP32 in group order with packed f32x2 arithmetic
//               (each lane op IEEE-rounded: reference order when EXACT, fused
//               multiply-add otherwise). After the last group the FP32 sums move
//               to shared memory (the drained stage ring) and each thread finishes
//               its row: LoRA-B, the epilogue and the store.
// Every wait is bounded (mbar_wait_bounded); a stall records kWaitTimeout.
#pragma once
#include "common.cuh"

namespace dg {

struct GemmArgs {
  int M, N, K;              // N is a multiple of BN, K a multiple of 128
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

template <int BN_>
struct GemmShape {
  static constexpr int BM = 128, BN = BN_, BK = 128;  // BK bytes = two 64-wide groups
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
  static constexpr int WS_OFF = A_BYTES + B_BYTES;                  // [2][BN] floats
  static constexpr int XS_OFF = WS_OFF + 2 * BN * 4;                // [2][BM] floats
  static constexpr int STAGE_BYTES = (XS_OFF + 2 * BM * 4 + 1023) / 1024 * 1024;
  static constexpr int STAGES = BN == 256 ? 3 : (BN == 128 ? 5 : 6);
  static constexpr int LORA_OFF = STAGES * STAGE_BYTES;
  static constexpr int NUM_THREADS = 640;
  static constexpr int EPI_WARP0 = 4, EPI_WARPS = 16;
  static constexpr int HALF = BN / (EPI_WARPS / 4);                 // columns per epilogue warp
  static constexpr int ACC_LD = BN + 1;                             // padded smem row stride
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static_assert(BM * ACC_LD * 4 <= STAGES * STAGE_BYTES, "FP32 sums must fit in the drained stage ring");
  __host__ __device__ static constexpr int lora_bytes(int R) { return BN * R * 4; }
  __host__ __device__ static constexpr int bar_off(int R) { return LORA_OFF + lora_bytes(R); }
  __host__ __device__ static constexpr int smem_bytes(int R) { return bar_off(R) + 128 + 1024; }
};

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 512;" ::: "memory");  // the 16 promotion warps
}

// DUMP: also write the raw int32 group dots to p.dots (parity checks only).
template <int BN, int R, int EPI, bool EXACT, bool DUMP>
__global__ void __launch_bounds__(640, 1)
    gemm_i8_g64_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       GemmArgs p) {
  using S = GemmShape<BN>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES, STAGE_BYTES = S::STAGE_BYTES, HALF = S::HALF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::bar_off(R));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* lora_smem = reinterpret_cast<float*>(smem + S::LORA_OFF);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int G = p.K / 64, KS = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + S::EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], S::EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::TMEM_COLS);
    tmem_relinquish();
  }
  if (R > 0 && warp >= S::EPI_WARP0) {
    // Stage this tile's LoRA-B rows [BN][R] (contiguous in global memory).
    const float4* src = reinterpret_cast<const float4*>(p.lora_b + size_t(n0) * R);
    float4* dst = reinterpret_cast<float4*>(lora_smem);
    for (int i = threadIdx.x - S::EPI_WARP0 * 32; i < BN * R / 4; i += S::EPI_WARPS * 32) dst[i] = src[i];
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
        mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES + 2 * BN * 4 + 2 * BM * 4);
        tma_load_2d(st, &map_a, &full[s], ks * BK, m0);
        tma_load_2d(st + S::A_BYTES, &map_b, &full[s], ks * BK, n0);
        for (int j = 0; j < 2; ++j) {
          const int g = 2 * ks + j;
          bulk_load(st + S::WS_OFF + j * BN * 4, p.ws + size_t(g) * p.N + n0, BN * 4, &full[s]);
          bulk_load(st + S::XS_OFF + j * BM * 4, p.xs + size_t(g) * p.ldxs + m0, BM * 4, &full[s]);
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
        const uint32_t b_addr = a_addr + S::A_BYTES;
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
  } else if (warp >= S::EPI_WARP0) {
    // ---------------- promotion (warps 4..19)
    const int q = warp & 3;                          // TMEM lane quarter this warp may read
    const int half = (warp - S::EPI_WARP0) >> 2;     // which quarter of the tile's columns
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    float2 acc[HALF / 2];
#pragma unroll
    for (int j = 0; j < HALF / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    bool ok = true;
    for (int g = 0; g < G; ++g) {
      const int ks = g / 2, s = ks % STAGES, b = g & 1, use = g / 2;
      ok = mbar_wait_bounded(&full[s], (ks / STAGES) & 1, p.status, 300 + s, abort_flag) &&
           mbar_wait_bounded(&tfull[b], use & 1, p.status, 310 + b, abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint8_t* st = smem + s * STAGE_BYTES;
      const float xsg = reinterpret_cast<const float*>(st + S::XS_OFF)[(g & 1) * BM + row];
      const float2 xs2 = make_float2(xsg, xsg);
      const float* wsg = reinterpret_cast<const float*>(st + S::WS_OFF) + (g & 1) * BN + half * HALF;
#pragma unroll
      for (int c = 0; c < HALF / 8; ++c) {
        uint32_t d[8];
        tmem_ld_32x32b_x8(lane_addr + uint32_t(b * BN + half * HALF + c * 8), d);
        tmem_wait_ld();
        if (DUMP && m < p.M) {
          int4* dd = reinterpret_cast<int4*>(p.dots + (size_t(g) * p.M + m) * p.N + n0 + half * HALF + c * 8);
#pragma unroll
          for (int j4 = 0; j4 < 2; ++j4)
            dd[j4] = make_int4(int(d[j4 * 4]), int(d[j4 * 4 + 1]), int(d[j4 * 4 + 2]), int(d[j4 * 4 + 3]));
        }
#pragma unroll
        for (int j4 = 0; j4 < 2; ++j4) {
          const float4 w4 = reinterpret_cast<const float4*>(wsg + c * 8)[j4];
          const float2 wlo = make_float2(w4.x, w4.y), whi = make_float2(w4.z, w4.w);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = j4 * 4 + e * 2;
            // Exact int32 -> float: bits of 1.5 * 2^23 + dot, minus 1.5 * 2^23.
            float2 fd = make_float2(__int_as_float(int32_t(d[j]) + 0x4B400000),
                                    __int_as_float(int32_t(d[j + 1]) + 0x4B400000));
            float2& a2 = acc[(c * 8 + j) / 2];
            const float2 w2 = e ? whi : wlo;
            if (EXACT) {
              // Reference order with scalar IEEE operations (src/int8.rs:58):
              // sum + float(dot) * (xs * ws), rounded after every step.
              a2.x = __fadd_rn(a2.x, __fmul_rn(__fadd_rn(fd.x, -12582912.0f), __fmul_rn(xsg, w2.x)));
              a2.y = __fadd_rn(a2.y, __fmul_rn(__fadd_rn(fd.y, -12582912.0f), __fmul_rn(xsg, w2.y)));
            } else {
              fd = add2_rn(fd, neg_magic);
              a2 = fma2_rn(fd, mul2_rn(xs2, w2), a2);
            }
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
    float* accs = reinterpret_cast<float*>(smem) + size_t(row) * S::ACC_LD + half * HALF;
    if (ok) {
      // Bias-free projections add 0.0 as the reference does (src/tensor.rs:437).
#pragma unroll
      for (int j = 0; j < HALF / 2; ++j) {
        accs[2 * j] = __fadd_rn(acc[j].x, 0.0f);
        accs[2 * j + 1] = __fadd_rn(acc[j].y, 0.0f);
      }
    }
    __syncwarp();
    if (ok && m < p.M) {
      constexpr int CH = HALF < 16 ? HALF : 16;  // columns finished per pass
      float vals[CH];
#pragma unroll 1
      for (int c = 0; c < HALF / CH; ++c) {
        const int col0 = half * HALF + c * CH;
#pragma unroll
        for (int j = 0; j < CH; ++j) vals[j] = accs[c * CH + j];
        if (R > 0) {
          const int pid = p.chunk_pid[(n0 + col0) >> 4];
          float mid[R > 0 ? R : 1];
          const float4* mp = reinterpret_cast<const float4*>(p.lora_mid + size_t(m) * p.ld_mid + pid * R);
#pragma unroll
          for (int r4 = 0; r4 < R / 4; ++r4) {
            const float4 v = mp[r4];
            mid[r4 * 4] = v.x; mid[r4 * 4 + 1] = v.y; mid[r4 * 4 + 2] = v.z; mid[r4 * 4 + 3] = v.w;
          }
#pragma unroll 2
          for (int j = 0; j < CH; j += 2) {
            // Two columns at a time: .x for column j, .y for column j + 1.
            const float4* b0 = reinterpret_cast<const float4*>(lora_smem + (col0 + j) * R);
            const float4* b1 = reinterpret_cast<const float4*>(lora_smem + (col0 + j + 1) * R);
            float2 delta;
            if (EXACT) {
              // dot_scores order (src/tensor.rs:6-25): eight lanes, then their sum.
              float2 lanes[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) lanes[i] = make_float2(0.0f, 0.0f);
#pragma unroll
              for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 w0 = b0[r4], w1 = b1[r4];
                const float2 wv[4] = {make_float2(w0.x, w1.x), make_float2(w0.y, w1.y), make_float2(w0.z, w1.z),
                                      make_float2(w0.w, w1.w)};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int r = r4 * 4 + e;
                  lanes[r & 7].x = __fadd_rn(lanes[r & 7].x, __fmul_rn(mid[r], wv[e].x));
                  lanes[r & 7].y = __fadd_rn(lanes[r & 7].y, __fmul_rn(mid[r], wv[e].y));
                }
              }
              delta = make_float2(-0.0f, -0.0f);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                delta.x = __fadd_rn(delta.x, lanes[i].x);
                delta.y = __fadd_rn(delta.y, lanes[i].y);
              }
              delta.x = __fadd_rn(delta.x, 0.0f);
              delta.y = __fadd_rn(delta.y, 0.0f);
              vals[j] = __fadd_rn(vals[j], __fmul_rn(p.lora_scale, delta.x));
              vals[j + 1] = __fadd_rn(vals[j + 1], __fmul_rn(p.lora_scale, delta.y));
            } else {
              delta = make_float2(0.0f, 0.0f);
#pragma unroll
              for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 w0 = b0[r4], w1 = b1[r4];
                delta = fma2_rn(make_float2(mid[r4 * 4], mid[r4 * 4]), make_float2(w0.x, w1.x), delta);
                delta = fma2_rn(make_float2(mid[r4 * 4 + 1], mid[r4 * 4 + 1]), make_float2(w0.y, w1.y), delta);
                delta = fma2_rn(make_float2(mid[r4 * 4 + 2], mid[r4 * 4 + 2]), make_float2(w0.z, w1.z), delta);
                delta = fma2_rn(make_float2(mid[r4 * 4 + 3], mid[r4 * 4 + 3]), make_float2(w0.w, w1.w), delta);
              }
              vals[j] = __fmaf_rn(p.lora_scale, delta.x, vals[j]);
              vals[j + 1] = __fmaf_rn(p.lora_scale, delta.y, vals[j + 1]);
            }
          }
        }
        if (EPI == kEpiSwiGlu) {
          // Fused columns come in pairs of 16-wide chunks: 16 gate columns,
          // then the 16 matching up columns (outputs (n0 + col0) / 2 ...).
          // Keep each gate pass in shared memory and combine on the up pass.
          static_assert(CH == 16, "SwiGLU pairs 16-column chunks");
          if ((c & 1) == 0) {
#pragma unroll
            for (int j = 0; j < CH; ++j) accs[c * CH + j] = vals[j];
          } else {
            const float* gate = accs + (c - 1) * CH;
            float* o = p.out + size_t(m) * p.ldo + ((n0 + col0 - CH) >> 1);
#pragma unroll
            for (int j4 = 0; j4 < CH / 4; ++j4) {
              float4 v;
              v.x = silu_f(gate[j4 * 4 + 0]) * vals[j4 * 4 + 0];
              v.y = silu_f(gate[j4 * 4 + 1]) * vals[j4 * 4 + 1];
              v.z = silu_f(gate[j4 * 4 + 2]) * vals[j4 * 4 + 2];
              v.w = silu_f(gate[j4 * 4 + 3]) * vals[j4 * 4 + 3];
              reinterpret_cast<float4*>(o)[j4] = v;
            }
          }
        } else {
          float4* o = reinterpret_cast<float4*>(p.out + size_t(m) * p.ldo + n0 + col0);
#pragma unroll
          for (int j4 = 0; j4 < CH / 4; ++j4) {
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
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace dg
