// Group-64 INT8 projection on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's linear_int8 / Kernel::scaled_dot / Adapter::combine /
// write_columns chain (src/tensor.rs:379-456,109-117,272-288; src/int8.rs:55-61):
//
//   out[m,n] = EPI( Σ_g float(dot_g(xq[m], wq[n])) * (xs[m,g] * ws[n,g])  + 0.0
//                   + lora_scale * (dot_scores(mid[m, pid(n)], lora_b[n]) + 0.0) )
//
// One CTA owns a 128 x BN output tile (BN = 128, or 64 for narrow outputs so
// more SMs share the work); 18 warps:
//   warp 0      TMA producer: int8 A/B tiles (128-byte swizzle) plus the two
//               groups' activation and weight scales of each 128-wide K stage;
//               with tensor-core LoRA-B, also the LoRA operand tiles, which
//               the whole warp splits into TF32 parts before the loop ends;
//   warp 1      TMEM allocator and single-thread MMA issuer: per stage, two
//               64-wide groups, each two tcgen05.mma kind::i8 (K=32) into its
//               own int32 accumulator (the first overwrites, the second adds);
//               512 TMEM columns hold 512/BN group accumulators, so the MMAs
//               run up to 512/BN - 1 groups ahead of the promotion;
//   warps 2-17  promotion and epilogue. Main loop: four warps per TMEM lane
//               quarter (warp % 4), each owning a quarter of the tile's
//               columns; per group they tcgen05.ld the accumulator, free it for
//               the next MMA, and scale it in FP32 in group order (reference
//               order when EXACT, fused multiply-add otherwise).
//               Epilogue: the FP32 sums go to shared memory (the drained stage
//               ring) and leave in row-contiguous copies; with CUDA-core LoRA-B
//               each thread first finishes a 4-row x (BN/16)-column block as a
//               register-tiled rank-R product over the tile's LoRA-A rows.
// Every wait is bounded (mbar_wait_bounded); a stall records kWaitTimeout.
#pragma once
#include "common.cuh"

namespace dg {

struct GemmArgs {
  int M, N, K;              // N is a multiple of BN, K a multiple of 128
  const float* xs;          // activation scales [K/64][ldxs]
  int ldxs;                 // >= round_up(M, 128)
  const float* ws;          // weight scales [K/64][N]
  const float* lora_mid;    // [M][ld_mid] LoRA-A outputs of all fused parts (nullable when R == 0)
  int ld_mid;
  const float* lora_b;      // [N][R]
  const int* chunk_pid;     // [N/16] LoRA part of each 16-column chunk (non-decreasing per tile
                            // except SwiGLU's alternating gate/up chunks)
  float lora_scale;
  float* out;               // WRITE/ADD: [M][ldo] (N columns); SWIGLU: [M][ldo] (N/2 columns)
  int ldo;
  DeviceStatus* status;
  int32_t* dots;            // optional debug dump of the exact group dots [K/64][M][N]
  // Launched as a programmatic dependent of the LoRA-A kernels that produce
  // lora_mid, whose own waits already ordered the activations: wait for the
  // previous kernel only before reading lora_mid and writing out, so the main
  // loop overlaps the LoRA-A pass.
  int late_dep;
  // Split-K (FMA mode, grid.z > 1 splits of the K stages): each split stores
  // its raw partial sums in split_ws [split][M][N]; the last split of a tile
  // to arrive (split_cnt[tile], zero between launches) adds them in split
  // order and runs the epilogue.
  float* split_ws;
  int* split_cnt;
  size_t split_ws_floats;  // capacity of split_ws
  int splits;              // set by launch_gemm_i8 (1: no split)
  // Failure-path test aid (0 / 0 in normal launches): test_skip_commit = g + 1
  // makes the MMA issuer leave out the completion signal of group g, so the
  // promotion warps' wait for it runs out; wait_ns replaces the 2 s budget
  // of the pipeline's bounded waits.
  int test_skip_commit;
  unsigned long long wait_ns;
};

template <int BN_>
struct GemmShape {
  static_assert(BN_ == 64 || BN_ == 128, "tile width");
  static constexpr int BM = 128, BN = BN_, BK = 128;  // BK bytes = two 64-wide groups
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
  static constexpr int WS_OFF = A_BYTES + B_BYTES;                  // [2][BN] floats
  static constexpr int XS_OFF = WS_OFF + 2 * BN * 4;                // [2][BM] floats
  static constexpr int STAGE_BYTES = (XS_OFF + 2 * BM * 4 + 1023) / 1024 * 1024;
  static constexpr int STAGES = BN == 128 ? 5 : 6;
  static constexpr int RING = STAGES * STAGE_BYTES;
  static constexpr int NUM_THREADS = 576;
  static constexpr int EPI_WARP0 = 2, EPI_WARPS = 16, EPI_THREADS = EPI_WARPS * 32;
  static constexpr int HALF = BN / 4;           // main loop: columns per promotion warp
  static constexpr int NBUF = 512 / BN;         // group accumulators in TMEM (MMAs run NBUF - 1 groups ahead)
  static constexpr uint32_t TMEM_COLS = 512;
  // Epilogue layout inside the drained ring: FP32 sums [BM][ACC_LD], then the
  // tile's LoRA-A rows [BM][MID_LD] (at most four fused parts of rank 32).
  static constexpr int ACC_LD = BN + 4, MID_LD = 132, MID_MAX = 128;
  static constexpr int MID_OFF = BM * ACC_LD * 4;
  static_assert(MID_OFF + BM * MID_LD * 4 <= RING, "epilogue staging must fit in the ring");
  // LoRA-B of the tile, transposed: [R][BT_LD].
  static constexpr int BT_LD = BN + 4;
  static constexpr int BT_OFF = RING;
  static constexpr int CW = BN / 16, HW = CW / 2;  // epilogue: columns per thread, per half
  static_assert((2 * STAGES + 2 * NBUF + 3) * 8 + 8 <= 256, "barrier area");
  __host__ __device__ static constexpr int bt_bytes(int R) { return R * BT_LD * 4; }
  __host__ __device__ static constexpr int bar_off(int R) { return BT_OFF + bt_bytes(R); }
  __host__ __device__ static constexpr int plan_off(int R) { return bar_off(R) + 256; }  // LoraPlan (128 bytes)
  __host__ __device__ static constexpr int smem_bytes(int R) { return plan_off(R) + 128 + 1024; }
};

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 512;" ::: "memory");  // the 16 promotion warps
}

// Loads HW consecutive floats (HW = 2 or 4) from shared memory.
template <int HW>
__device__ __forceinline__ void lds_vec(const float* p, float (&v)[HW]) {
  if constexpr (HW == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x; v[1] = t.y;
  }
}

// LoRA-B on the tensor cores (fast mode, 128-column tiles): the tile's
// 16-column chunks grouped by LoRA part, so each part is one MMA of N = 16 x
// its chunk count. slot[c] is chunk c's position in that order; part p owns
// slots [run[p], run[p + 1]).
struct LoraPlan {
  int nparts;
  int pid[4];
  int slot[8];
  int run[5];
};
static_assert(sizeof(LoraPlan) <= 128, "plan area");
__device__ __forceinline__ LoraPlan lora_plan(const int* chunk_pid, int n0) {
  LoraPlan pl;
  int cp[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) cp[c] = chunk_pid[(n0 >> 4) + c];
  pl.nparts = 0;
  // Distinct parts in ascending order (at most four: the fused groups have <= 4).
  int last = -1;
  for (int k = 0; k < 4; ++k) {
    int best = 1 << 30;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (cp[c] > last && cp[c] < best) best = cp[c];
    if (best == (1 << 30)) break;
    pl.pid[pl.nparts++] = best;
    last = best;
  }
  int s = 0;
  for (int k = 0; k < pl.nparts; ++k) {
    pl.run[k] = s;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (cp[c] == pl.pid[k]) pl.slot[c] = s++;
  }
  pl.run[pl.nparts] = s;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    if (cp[c] > last) pl.slot[c] = 0;  // parts beyond four are not staged (not produced by the fused groups)
  return pl;
}

// DUMP: also write the raw int32 group dots to p.dots (parity checks only).
// map_lb / map_mid (LoRA-B rows [N][32] and LoRA-A rows [M][ld_mid], FP32,
// 128-byte swizzle) are read only by the tensor-core LoRA path.
template <int BN, int R, int EPI, bool EXACT, bool DUMP>
__global__ void __launch_bounds__(576, 1)
    gemm_i8_g64_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_lb, const __grid_constant__ CUtensorMap map_mid,
                       GemmArgs p) {
  using S = GemmShape<BN>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES, STAGE_BYTES = S::STAGE_BYTES, HALF = S::HALF;
  constexpr int NBUF = S::NBUF;
  // Tensor-core LoRA-B (3 x TF32): fast mode, rank 32, 128-column tiles. The
  // LoRA operands come through the stage ring as stages KS (B rows) and
  // KS + 1 + part (A rows); the producer warp splits each FP32 tile into its
  // TF32 part and the low-order remainder.
  constexpr bool TCL = R == 32 && !EXACT && !DUMP && BN == 128;
  constexpr int LT = 128 * 128;  // bytes of one FP32 LoRA operand tile (128 rows x 32)
  static_assert(!TCL || (2 * LT <= STAGE_BYTES && STAGES >= 5), "LoRA operands must fit the ring");
  static_assert(EPI != kEpiSwiGlu || BN == 128, "SwiGLU pairs need 128-column tiles");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base (128-byte swizzled tiles). Pointer arithmetic on the
  // __shared__ array, not an integer round trip, so that the compiler keeps
  // every access through smem in the shared state space (ld.shared / st.shared):
  // generic accesses would queue behind the global stores in the same path.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::bar_off(R));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;     // group accumulator b written by the MMAs
  uint64_t* tempty = tfull + NBUF;      // group accumulator b read by every promotion warp
  uint64_t* mma_done = tempty + NBUF;
  uint64_t* lora_ready = mma_done + 1;  // LoRA operands split into TF32 parts (producer warp)
  uint64_t* lora_done = lora_ready + 1;  // LoRA-B MMAs complete
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(lora_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* bt_smem = reinterpret_cast<float*>(smem + S::BT_OFF);
  LoraPlan* plan = reinterpret_cast<LoraPlan*>(smem + S::plan_off(R));

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const uint64_t budget = p.wait_ns ? p.wait_ns : 2000000000ull;  // every pipeline wait
  const int KS = p.K / BK / int(gridDim.z);  // this split's K stages
  const int ks0 = int(blockIdx.z) * KS;      // its first stage

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], S::EPI_WARPS);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], S::EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    mbar_init(lora_ready, 1);
    mbar_init(lora_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
    if constexpr (TCL) {
      prefetch_tensormap(&map_lb);
      prefetch_tensormap(&map_mid);
      *plan = lora_plan(p.chunk_pid, n0);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (R > 0 && !TCL) if (warp >= S::EPI_WARP0) {
    // This tile's LoRA-B rows [BN][R], transposed to [R][BT_LD].
    const float4* src = reinterpret_cast<const float4*>(p.lora_b + size_t(n0) * R);
    for (int i = threadIdx.x - S::EPI_WARP0 * 32; i < BN * R / 4; i += S::EPI_THREADS) {
      const float4 v = src[i];
      const int n = i / (R / 4), r = (i % (R / 4)) * 4;
      bt_smem[(r + 0) * S::BT_LD + n] = v.x;
      bt_smem[(r + 1) * S::BT_LD + n] = v.y;
      bt_smem[(r + 2) * S::BT_LD + n] = v.z;
      bt_smem[(r + 3) * S::BT_LD + n] = v.w;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Set-up above touched only shared memory, TMEM and weights.
  if (!p.late_dep) griddep_wait();
  griddep_launch();

  if (warp == 0) {
    int issued = 0;
    if (lane == 0) {
      // ---------------- TMA producer
      for (int ks = 0; ks < KS; ++ks) {
        const int s = ks % STAGES, use = ks / STAGES;
        if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, p.status, 100 + s, abort_flag, budget)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES + 2 * BN * 4 + 2 * BM * 4);
        tma_load_2d(st, &map_a, &full[s], (ks0 + ks) * BK, m0);
        tma_load_2d(st + S::A_BYTES, &map_b, &full[s], (ks0 + ks) * BK, n0);
        for (int j = 0; j < 2; ++j) {
          const int g = 2 * (ks0 + ks) + j;
          bulk_load(st + S::WS_OFF + j * BN * 4, p.ws + size_t(g) * p.N + n0, BN * 4, &full[s]);
          bulk_load(st + S::XS_OFF + j * BM * 4, p.xs + size_t(g) * p.ldxs + m0, BM * 4, &full[s]);
        }
        issued = ks + 1;
      }
      if constexpr (TCL) {
        // LoRA operand stages: KS = this tile's LoRA-B rows, chunk by chunk into
        // their part-sorted slots; KS + 1 + k = the LoRA-A rows of part k.
        if (issued == KS) {
          if (p.late_dep) griddep_wait();  // lora_mid comes from the previous kernel
          for (int j = 0; j <= plan->nparts; ++j) {
            const int ls = KS + j, s = ls % STAGES, use = ls / STAGES;
            if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, p.status, 120 + s, abort_flag, budget)) break;
            uint8_t* st = smem + s * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], LT);
            if (j == 0) {
#pragma unroll
              for (int c = 0; c < 8; ++c) tma_load_2d(st + plan->slot[c] * 2048, &map_lb, &full[s], 0, n0 + 16 * c);
            } else {
              tma_load_2d(st, &map_mid, &full[s], plan->pid[j - 1] * 32, m0);
            }
            issued = ls + 1;
          }
        }
      }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);
    if constexpr (TCL) {
      // The whole warp splits each LoRA operand tile into its TF32 part (low
      // 13 mantissa bits cleared, in place) and the remainder (at +LT), while
      // the promotion warps finish the main loop; the MMA issuer then runs
      // hi·hi + hi·lo + lo·hi. Rows past M are zero (TMA fill).
      bool ready = issued == KS + 1 + plan->nparts;
      for (int j = 0; j <= plan->nparts && ready; ++j) {
        const int ls = KS + j, s = ls % STAGES;
        ready = mbar_wait_bounded(&full[s], (ls / STAGES) & 1, p.status, 140 + s, abort_flag, budget);
        if (!ready) break;
        float4* t = reinterpret_cast<float4*>(smem + s * STAGE_BYTES);
#pragma unroll 4
        for (int i = lane; i < LT / 16; i += 32) {
          const float4 v = t[i];
          float4 h;
          h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
          h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
          h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
          h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
          t[i] = h;
          t[i + LT / 16] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && ready) mbar_arrive(lora_ready);
    }
    if (lane == 0 && *abort_flag) {
      // Let this CTA's copies in flight land before the CTA exits.
      for (int ks = (issued > STAGES ? issued - STAGES : 0); ks < issued; ++ks)
        mbar_wait_bounded(&full[ks % STAGES], (ks / STAGES) & 1, p.status, 190, nullptr, 100000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      bool run = true;
      for (int ks = 0; ks < KS && run; ++ks) {
        const int s = ks % STAGES;
        if (!mbar_wait_bounded(&full[s], (ks / STAGES) & 1, p.status, 200 + s, abort_flag, budget)) break;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          // Group g goes to accumulator g % NBUF once every promotion warp
          // has read that accumulator's previous group (phase g / NBUF).
          const int g = 2 * ks + j, b = g % NBUF;
          if (!mbar_wait_bounded(&tempty[b], (g / NBUF) & 1, p.status, 210 + b, abort_flag, budget)) {
            run = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * STAGE_BYTES) + j * 64;
          const uint32_t b_addr = a_addr + S::A_BYTES;
          const uint32_t d = tmem_base + uint32_t(b * BN);
          // The group's first MMA overwrites the accumulator, the second adds.
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_i8(d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), idesc, kk);
          if (g + 1 != p.test_skip_commit) mma_commit(&tfull[b]);
        }
      }
      if constexpr (TCL) {
        // delta = mid · Bᵀ in 3 x TF32 (hi·hi + hi·lo + lo·hi) into the group
        // accumulator that the main loop's group 2 KS would have used.
        const int gd = 2 * KS, bd = gd % NBUF;
        if (run && !*abort_flag &&
            mbar_wait_bounded(&tempty[bd], (gd / NBUF) & 1, p.status, 230, abort_flag, budget) &&
            mbar_wait_bounded(lora_ready, 0, p.status, 231, abort_flag, budget)) {
          tc_fence_after();
          const LoraPlan& pl = *plan;
          const uint32_t d = tmem_base + uint32_t(bd * BN);
          const uint32_t b_hi = smem_addr(smem + (KS % STAGES) * STAGE_BYTES);
          for (int k = 0; k < pl.nparts; ++k) {
            const int s0 = pl.run[k], s1 = pl.run[k + 1];
            if (s1 == s0) continue;
            const uint32_t idesc = idesc_tf32(BM, uint32_t(16 * (s1 - s0)));
            const uint32_t a_hi = smem_addr(smem + ((KS + 1 + k) % STAGES) * STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t ah = a_hi + kk * 32, al = ah + LT;
              const uint32_t bh = b_hi + s0 * 2048 + kk * 32, bl = bh + LT;
              const uint32_t dd = d + uint32_t(16 * s0);
              mma_tf32(dd, smem_desc_sw128(ah), smem_desc_sw128(bh), idesc, kk > 0);
              mma_tf32(dd, smem_desc_sw128(ah), smem_desc_sw128(bl), idesc, 1);
              mma_tf32(dd, smem_desc_sw128(al), smem_desc_sw128(bh), idesc, 1);
            }
          }
          mma_commit(lora_done);
        }
      }
      // All MMAs of this thread have completed once mma_done flips.
      mma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status, 220, nullptr);
    }
  } else if (warp >= S::EPI_WARP0) {
    // ---------------- promotion (warps 2..17)
    const int q = warp & 3;                          // TMEM lane quarter this warp may read
    const int half = (warp - S::EPI_WARP0) >> 2;     // which quarter of the tile's columns
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(half * HALF);
    // Exact int32 -> float conversion: adding the bits of 1.5 * 2^23
    // (0x4B400000) to the dot (|dot| <= 64 * 128 * 128 < 2^22) gives the bits of
    // the float 1.5 * 2^23 + dot, so one subtraction of 1.5 * 2^23 is left.
    constexpr uint32_t kOffsetBits = 0x4B400000u;
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < NBUF; ++b) mbar_arrive(&tempty[b]);  // every accumulator starts free
    }
    float2 acc[HALF / 2];
#pragma unroll
    for (int j = 0; j < HALF / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    // Per group: load this warp's HALF columns (HALF / 16 chunks of 16), hand
    // the accumulator back to the MMA issuer, then scale in registers. With
    // one chunk per group (64-column tiles) both groups of a stage share one
    // TMEM load wait.
    constexpr int CPG = HALF / 16;
    constexpr int GB = CPG == 1 ? 2 : 1;  // groups per TMEM load wait
    bool ok = true;
    for (int ks = 0; ks < KS && ok; ++ks) {
      const int s = ks % STAGES;
      ok = mbar_wait_bounded(&full[s], (ks / STAGES) & 1, p.status, 300 + s, abort_flag, budget);
      if (!ok) break;
      const uint8_t* st = smem + s * STAGE_BYTES;
      const float* xsp = reinterpret_cast<const float*>(st + S::XS_OFF);
      const float* wsp = reinterpret_cast<const float*>(st + S::WS_OFF) + half * HALF;
#pragma unroll
      for (int j0 = 0; j0 < 2; j0 += GB) {
#pragma unroll
        for (int jj = 0; jj < GB && ok; ++jj) {
          const int g = 2 * ks + j0 + jj, b = g % NBUF;
          ok = mbar_wait_bounded(&tfull[b], (g / NBUF) & 1, p.status, 310 + b, abort_flag, budget);
        }
        if (!ok) break;
        tc_fence_after();
        // [group of the batch][chunk]: two 16-column loads per wait either way.
        static_assert(GB * CPG == 2, "two loads per TMEM wait");
        uint32_t d[2][16];
        const uint32_t a0 = lane_addr + uint32_t(((2 * ks + j0) % NBUF) * BN);
        tmem_ld16x2_sync(a0, GB == 2 ? lane_addr + uint32_t(((2 * ks + j0 + 1) % NBUF) * BN) : a0 + 16u, d[0], d[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int jj = 0; jj < GB; ++jj) mbar_arrive(&tempty[(2 * ks + j0 + jj) % NBUF]);
        }
#pragma unroll
        for (int jj = 0; jj < GB; ++jj) {
          const int j = j0 + jj, g = 2 * ks + j;
          const float xs = xsp[j * BM + row];
          // FMA mode folds the conversion into the row scale: with xs rounded
          // to 22 significant bits, 1.5 * 2^23 * xs' = 3 * 2^22 * xs' is exact,
          // so fma(1.5 * 2^23 + dot, xs', -1.5 * 2^23 * xs') = dot * xs'
          // rounded once; the column scale then enters by one more fma. Two
          // FP32 operations per element instead of three (xs' differs from xs
          // by at most 2^-22 relative).
          const float xsr = __uint_as_float((__float_as_uint(xs) + 2u) & ~3u);
          const float2 xs2 = make_float2(xsr, xsr);
          const float cxs = __fmul_rn(-12582912.0f, xsr);
          const float2 cxs2 = make_float2(cxs, cxs);
#pragma unroll
          for (int c = 0; c < CPG; ++c) {
            const uint32_t(&cur)[16] = d[jj * CPG + c];
            if (DUMP && m < p.M) {
              int4* dd = reinterpret_cast<int4*>(p.dots + (size_t(g) * p.M + m) * p.N + n0 + half * HALF + c * 16);
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4)
                dd[j4] = make_int4(int(cur[j4 * 4]), int(cur[j4 * 4 + 1]), int(cur[j4 * 4 + 2]), int(cur[j4 * 4 + 3]));
            }
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
              const float4 w4 = reinterpret_cast<const float4*>(wsp + j * BN + c * 16)[j4];
              const float2 wlo = make_float2(w4.x, w4.y), whi = make_float2(w4.z, w4.w);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int k = j4 * 4 + e * 2;
                float2 fd =
                    make_float2(__uint_as_float(cur[k] + kOffsetBits), __uint_as_float(cur[k + 1] + kOffsetBits));
                float2& a2 = acc[(c * 16 + k) / 2];
                const float2 w2 = e ? whi : wlo;
                if (EXACT) {
                  // Reference order with scalar IEEE operations (src/int8.rs:58):
                  // sum + float(dot) * (xs * ws), rounded after every step.
                  a2.x = __fadd_rn(a2.x, __fmul_rn(__fadd_rn(fd.x, -12582912.0f), __fmul_rn(xs, w2.x)));
                  a2.y = __fadd_rn(a2.y, __fmul_rn(__fadd_rn(fd.y, -12582912.0f), __fmul_rn(xs, w2.y)));
                } else {
                  a2 = fma2_rn(fma2_rn(fd, xs2, cxs2), w2, a2);
                }
              }
            }
          }
        }
      }
      if (!ok) break;
      // The stage's scales were read through the generic proxy and the next
      // TMA into the stage writes through the async proxy: without the proxy
      // fence the mbarrier release does not order the two, and a refill can
      // land before reads still queued in the load path (seen when global
      // stores sit ahead of them) have been performed.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // scales and operands of the stage are consumed
    }
    // ---------------- split-K: the last split of the tile adds the partials
    bool last = true;
    if (gridDim.z > 1) {
      const size_t slab = size_t(p.M) * p.N;
      volatile int* split_flag = reinterpret_cast<volatile int*>(smem + S::plan_off(R) + 96);
      if (m < p.M) {
        float4* d4 = reinterpret_cast<float4*>(p.split_ws + blockIdx.z * slab + size_t(m) * p.N + n0 + half * HALF);
#pragma unroll
        for (int j = 0; j < HALF / 4; ++j)
          d4[j] = make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
      }
      __threadfence();
      epi_bar_sync();
      if (threadIdx.x == S::EPI_WARP0 * 32) {
        int* cnt = p.split_cnt + blockIdx.y * gridDim.x + blockIdx.x;
        const int is_last = atomicAdd(cnt, 1) == int(gridDim.z) - 1;
        if (is_last) *cnt = 0;  // ready for the next launch
        *split_flag = is_last;
      }
      epi_bar_sync();
      last = *split_flag != 0;
      if (last) {
        __threadfence();
        if (m < p.M) {
#pragma unroll 1
          for (int z = 0; z < int(gridDim.z); ++z) {
            const float4* s4 =
                reinterpret_cast<const float4*>(p.split_ws + z * slab + size_t(m) * p.N + n0 + half * HALF);
#pragma unroll
            for (int j = 0; j < HALF / 4; ++j) {
              const float4 v = __ldcg(s4 + j);
              if (z == 0) {
                acc[2 * j] = make_float2(v.x, v.y);
                acc[2 * j + 1] = make_float2(v.z, v.w);
              } else {
                acc[2 * j] = make_float2(__fadd_rn(acc[2 * j].x, v.x), __fadd_rn(acc[2 * j].y, v.y));
                acc[2 * j + 1] = make_float2(__fadd_rn(acc[2 * j + 1].x, v.z), __fadd_rn(acc[2 * j + 1].y, v.w));
              }
            }
          }
        }
      }
    }
    // ---------------- epilogue
    if (p.late_dep) griddep_wait();  // lora_mid and the output buffer
    const int et = threadIdx.x - S::EPI_WARP0 * 32;  // 0 .. 511
    if constexpr (TCL) {
      const LoraPlan& pl = *plan;
      ok = ok && mbar_wait_bounded(lora_done, 0, p.status, 330, abort_flag, budget);
      if (ok) {
        // This thread's 32 columns: two 16-column chunks, at their part-sorted
        // slots of the delta accumulator.
        tc_fence_after();
        const uint32_t dcol = uint32_t(((2 * KS) % NBUF) * BN);
        const int c0 = (half * HALF) >> 4;
        static_assert(HALF == 32, "tensor-core LoRA-B: two 16-column chunks per thread");
        const uint32_t dbase = tmem_base + (uint32_t(q * 32) << 16) + dcol;
        uint32_t dv[2][16];
        tmem_ld16x2_sync(dbase + uint32_t(16 * pl.slot[c0]), dbase + uint32_t(16 * pl.slot[c0 + 1]), dv[0], dv[1]);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float2& a2 = acc[cc * 8 + e];
            a2.x = __fmaf_rn(p.lora_scale, __uint_as_float(dv[cc][2 * e]), __fadd_rn(a2.x, 0.0f));
            a2.y = __fmaf_rn(p.lora_scale, __uint_as_float(dv[cc][2 * e + 1]), __fadd_rn(a2.y, 0.0f));
          }
        }
      }
    }
    epi_bar_sync();  // every promotion warp has left the loop: the ring is free
    float* accs = reinterpret_cast<float*>(smem);
    float* mids = reinterpret_cast<float*>(smem + S::MID_OFF);
    {
      float4* dst = reinterpret_cast<float4*>(accs + size_t(row) * S::ACC_LD + half * HALF);
#pragma unroll
      for (int j = 0; j < HALF / 4; ++j) {
        // Bias-free projections add 0.0 as the reference does (src/tensor.rs:437);
        // the tensor-core LoRA path has already added it (and the delta).
        if constexpr (TCL)
          dst[j] = make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
        else
          dst[j] = make_float4(__fadd_rn(acc[2 * j].x, 0.0f), __fadd_rn(acc[2 * j].y, 0.0f),
                               __fadd_rn(acc[2 * j + 1].x, 0.0f), __fadd_rn(acc[2 * j + 1].y, 0.0f));
      }
    }
    constexpr int MAXP = R > 0 ? S::MID_MAX / R : 1;  // LoRA parts one tile may span
    int pmin = 0;
    if constexpr (R > 0 && !TCL) {
      // LoRA-A rows of the parts this tile's columns use, zero past row M.
      int lo = 1 << 30, hi = 0;
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        const int v = p.chunk_pid[(n0 >> 4) + c];
        lo = min(lo, v);
        hi = max(hi, v);
      }
      hi = min(hi, lo + MAXP - 1);
      pmin = lo;
      const int nc4 = (hi - lo + 1) * (R / 4);
      for (int i = et; i < BM * nc4; i += S::EPI_THREADS) {
        const int r = i / nc4, c4 = i % nc4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (m0 + r < p.M)
          v = *reinterpret_cast<const float4*>(p.lora_mid + size_t(m0 + r) * p.ld_mid + lo * R + c4 * 4);
        *reinterpret_cast<float4*>(mids + r * S::MID_LD + c4 * 4) = v;
      }
    }
    epi_bar_sync();
    if (*abort_flag || !last) {
      // nothing is written after a failed wait, nor by a split that is not the tile's last
    } else if constexpr (R == 0 || TCL) {
      // The staged sums are final: row-contiguous copies, one float4 per
      // thread and step (a warp covers 512 contiguous bytes of output).
      if constexpr (EPI == kEpiSwiGlu) {
        // Output column 16 k + t = silu(gate column 32 k + t) * (up column 32 k + 16 + t).
        constexpr int O4 = BN / 8;
        for (int i = et; i < BM * O4; i += S::EPI_THREADS) {
          const int r = i / O4, o4 = i % O4, mm = m0 + r;
          if (mm >= p.M) continue;
          const float* src = accs + r * S::ACC_LD + 32 * (o4 >> 2) + 4 * (o4 & 3);
          const float4 gt = *reinterpret_cast<const float4*>(src);
          const float4 up = *reinterpret_cast<const float4*>(src + 16);
          *reinterpret_cast<float4*>(p.out + size_t(mm) * p.ldo + (n0 >> 1) + 4 * o4) =
              make_float4(silu_f(gt.x) * up.x, silu_f(gt.y) * up.y, silu_f(gt.z) * up.z, silu_f(gt.w) * up.w);
        }
      } else {
        constexpr int C4 = BN / 4;
        for (int i = et; i < BM * C4; i += S::EPI_THREADS) {
          const int r = i / C4, c4 = i % C4, mm = m0 + r;
          if (mm >= p.M) continue;
          float4 v = *reinterpret_cast<const float4*>(accs + r * S::ACC_LD + 4 * c4);
          float4* o = reinterpret_cast<float4*>(p.out + size_t(mm) * p.ldo + n0 + 4 * c4);
          if constexpr (EPI == kEpiAdd) {
            const float4 old = *o;
            v = make_float4(__fadd_rn(old.x, v.x), __fadd_rn(old.y, v.y), __fadd_rn(old.z, v.z), __fadd_rn(old.w, v.w));
          }
          *o = v;
        }
      }
    } else {
      // Each thread finishes rows r0..r0+3 of two HW-column halves: adjacent
      // (WRITE/ADD) or a gate chunk and its up chunk 16 columns on (SWIGLU),
      // after the register-tiled LoRA-B product of those columns.
      constexpr int HW = S::HW;
      const int cg = et & 15, r0 = (et >> 4) * 4;
      int col[2], ocol;
      if constexpr (EPI == kEpiSwiGlu) {
        col[0] = 32 * (cg >> 2) + 4 * (cg & 3);
        col[1] = col[0] + 16;
        ocol = (n0 >> 1) + 16 * (cg >> 2) + 4 * (cg & 3);
      } else {
        col[0] = cg * S::CW;
        col[1] = col[0] + HW;
        ocol = n0 + col[0];
      }
      // v: the FP32 sums, read half by half after that half's LoRA-B product.
      float v[4][2][HW];
      {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int part = min(max(p.chunk_pid[(n0 + col[h]) >> 4] - pmin, 0), MAXP - 1);
          const float* mrow = mids + r0 * S::MID_LD + part * R;
          const float* brow = bt_smem + col[h];
          if constexpr (EXACT) {
            // dot_scores order (src/tensor.rs:6-25): lane l sums ranks l, l+8,
            // l+16, l+24 from 0.0; the lanes are added in order from -0.0.
            float tot[4][HW];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int c = 0; c < HW; ++c) tot[i][c] = -0.0f;
#pragma unroll 1
            for (int l = 0; l < 8; ++l) {
              float lan[4][HW];
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < HW; ++c) lan[i][c] = 0.0f;
#pragma unroll
              for (int jj = 0; jj < R / 8; ++jj) {
                const int r = l + 8 * jj;
                float b[HW];
                lds_vec<HW>(brow + r * S::BT_LD, b);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float x = mrow[i * S::MID_LD + r];
#pragma unroll
                  for (int c = 0; c < HW; ++c) lan[i][c] = __fadd_rn(lan[i][c], __fmul_rn(x, b[c]));
                }
              }
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < HW; ++c) tot[i][c] = __fadd_rn(tot[i][c], lan[i][c]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              lds_vec<HW>(accs + (r0 + i) * S::ACC_LD + col[h], v[i][h]);
#pragma unroll
              for (int c = 0; c < HW; ++c)
                v[i][h][c] = __fadd_rn(v[i][h][c], __fmul_rn(p.lora_scale, __fadd_rn(tot[i][c], 0.0f)));
            }
          } else {
            float dl[4][HW];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int c = 0; c < HW; ++c) dl[i][c] = 0.0f;
#pragma unroll 1
            for (int r4 = 0; r4 < R / 4; ++r4) {
              float b[4][HW];
#pragma unroll
              for (int e = 0; e < 4; ++e) lds_vec<HW>(brow + (r4 * 4 + e) * S::BT_LD, b[e]);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 x = *reinterpret_cast<const float4*>(mrow + i * S::MID_LD + r4 * 4);
#pragma unroll
                for (int c = 0; c < HW; ++c) {
                  dl[i][c] = __fmaf_rn(x.x, b[0][c], dl[i][c]);
                  dl[i][c] = __fmaf_rn(x.y, b[1][c], dl[i][c]);
                  dl[i][c] = __fmaf_rn(x.z, b[2][c], dl[i][c]);
                  dl[i][c] = __fmaf_rn(x.w, b[3][c], dl[i][c]);
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              lds_vec<HW>(accs + (r0 + i) * S::ACC_LD + col[h], v[i][h]);
#pragma unroll
              for (int c = 0; c < HW; ++c) v[i][h][c] = __fmaf_rn(p.lora_scale, dl[i][c], v[i][h][c]);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int mm = m0 + r0 + i;
        if (mm >= p.M) continue;
        float* o = p.out + size_t(mm) * p.ldo + ocol;
        if constexpr (EPI == kEpiSwiGlu) {
          *reinterpret_cast<float4*>(o) = make_float4(silu_f(v[i][0][0]) * v[i][1][0], silu_f(v[i][0][1]) * v[i][1][1],
                                                      silu_f(v[i][0][2]) * v[i][1][2], silu_f(v[i][0][3]) * v[i][1][3]);
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float w[HW];
#pragma unroll
            for (int c = 0; c < HW; ++c) w[c] = v[i][h][c];
            if constexpr (EPI == kEpiAdd) {
              float old[HW];
              if constexpr (HW == 4) {
                const float4 t = *reinterpret_cast<const float4*>(o + h * HW);
                old[0] = t.x; old[1] = t.y; old[2] = t.z; old[3] = t.w;
              } else {
                const float2 t = *reinterpret_cast<const float2*>(o + h * HW);
                old[0] = t.x; old[1] = t.y;
              }
#pragma unroll
              for (int c = 0; c < HW; ++c) w[c] = __fadd_rn(old[c], w[c]);
            }
            if constexpr (HW == 4)
              *reinterpret_cast<float4*>(o + h * HW) = make_float4(w[0], w[1], w[2], w[3]);
            else
              *reinterpret_cast<float2*>(o + h * HW) = make_float2(w[0], w[1]);
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
