// Chunked gated delta rule (the engine's fast mode; dk = dv = 128).
//
// The reference runs the recurrence token by token (Recurrence::head,
// src/qwen.rs:813-875):  S <- g_t S ;  d_t = b_t (v_t - S^T k_t) ;
// S <- S + k_t d_t^T ;  o_t = S^T q_t.  Over a chunk of C tokens starting
// from state S0, with G_t = prod_{s<=t} g_s (log-space cumulative sums), the
// same quantities are
//   D = U - W S0,   U = T diag(b) V,   W = T diag(b G) K,
//   T = (I + L)^-1, L[t][s] = b_t (G_t / G_s) k_t.k_s  (s < t),
//   O = diag(G) Q S0 + (M o Q K^T) D,   M[t][s] = G_t / G_s (s <= t),
//   S_C = G_C S0 + K^T diag(G_C / G) D,
// so only the S0-dependent products are sequential across chunks.
//
// delta_chunk_prep_kernel (one CTA per sequence x head x chunk, all chunks in
// parallel) builds T, U, W, the masked Q K^T and the decay vectors;
// delta_chunk_scan_kernel (one CTA per sequence x head x 32 value columns)
// carries the state slice through the chunks. FP32 throughout.
#include "launch.h"

namespace dg {

namespace {

constexpr int CK = 64, DK = 128;
// Scan CTAs: SC value columns on 8 * SC threads (each thread the same tile).
// 16 columns (128 threads) keep one sequence's scan on 8 CTAs per head, the
// shorter latency per chunk; 32 columns (256 threads) halve the CTAs and the
// W / K staging traffic per column, which pays when many sequences fill the
// GPU anyway, or when other work runs beside the scan (measured: 64
// sequences x 4096 tokens 38.9 -> 34.0 ms; one 512-token sequence 8.45 ->
// 8.72 ms per 24-layer forward; config 5 on two lanes +1 %).

// Per-chunk products written by the prep kernel.
struct ChunkOut {
  float W[CK][DK];
  float U[CK][DK];
  float QK[CK][CK];
  float gam[CK];    // G_t
  float rem[CK];    // G_C / G_t
  float gC;         // G_C
  float pad[3];
};

// Per-chunk values of the sequential pass, read by the output pass.
struct ChunkState {
  float S[DK][DK];  // state at the chunk start (value columns j0.. of each slice)
  float D[CK][DK];  // U - W S0
};

// Shared memory holds K and Q, and V once Q is no longer needed (V is loaded
// by the warps the triangular solve leaves idle), so two CTAs fit on an SM
// and one CTA's solve overlaps the other's products.
__global__ void __launch_bounds__(256, 2) delta_chunk_prep_kernel(DeltaArgs a, ChunkOut* __restrict__ outs,
                                                               int chunks) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) float sm[];
  float* Ks = sm;                   // [CK][DK + 1]
  float* Qs = Ks + CK * (DK + 1);   // [CK][DK + 1]
  float* Vs = Qs;                   // [CK][DK + 1]: V after the Q K^T products
  float* L = Qs + CK * (DK + 1);    // [CK][CK + 1]
  float* T = L + CK * (CK + 1);     // [CK][CK + 1]
  float* lg = T + CK * (CK + 1);    // [CK] cumulative log decay
  float* bt = lg + CK;              // [CK]
  float* gm = bt + CK;              // [CK] G_t = exp(lg)
  float* Xs = gm + CK;              // [CK / 16 - 1][16][16] block-row products
  const int tid = threadIdx.x;
  const int c = blockIdx.x % chunks, h = (blockIdx.x / chunks) % a.value_heads;
  const size_t bi = blockIdx.x / (chunks * a.value_heads);
  const int kh = h / (a.value_heads / a.key_heads);
  const int t0 = c * CK, tn = min(CK, a.n - t0);
  ChunkOut& o = outs[(bi * a.value_heads + h) * chunks + c];
  const float* qb = a.q + bi * a.bs_qkv + kh * DK;
  const float* kb = a.k + bi * a.bs_qkv + kh * DK;
  const float* vb = a.v + bi * a.bs_qkv + h * a.dv;
  for (int i = tid; i < CK * (DK / 4); i += 256) {
    const int t = i / (DK / 4), d = (i % (DK / 4)) * 4;
    float4 q4 = make_float4(0, 0, 0, 0), k4 = q4;
    if (t < tn) {
      q4 = *reinterpret_cast<const float4*>(qb + size_t(t0 + t) * a.ld_qk + d);
      k4 = *reinterpret_cast<const float4*>(kb + size_t(t0 + t) * a.ld_qk + d);
    }
    float* qd = Qs + t * (DK + 1) + d;
    float* kd = Ks + t * (DK + 1) + d;
    qd[0] = q4.x; qd[1] = q4.y; qd[2] = q4.z; qd[3] = q4.w;
    kd[0] = k4.x; kd[1] = k4.y; kd[2] = k4.z; kd[3] = k4.w;
  }
  if (tid < 32) {
    // Cumulative log decay over the chunk (two tokens per lane, then a scan).
    float g0 = 0.0f, g1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
    const int ta = 2 * tid, tb = 2 * tid + 1;
    const float* gd = a.decay + bi * a.bs_gb + h;
    const float* bd = a.beta + bi * a.bs_gb + h;
    if (ta < tn) {
      g0 = gd[size_t(t0 + ta) * a.ld_gb];
      b0 = bd[size_t(t0 + ta) * a.ld_gb];
    }
    if (tb < tn) {
      g1 = gd[size_t(t0 + tb) * a.ld_gb];
      b1 = bd[size_t(t0 + tb) * a.ld_gb];
    }
    if (!a.log_decay) {
      g0 = ta < tn ? logf(g0) : 0.0f;
      g1 = tb < tn ? logf(g1) : 0.0f;
    }
    float pair = g0 + g1, incl = pair;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float v = __shfl_up_sync(0xffffffffu, incl, off);
      if (tid >= off) incl += v;
    }
    const float excl = incl - pair;
    lg[ta] = excl + g0;
    lg[tb] = incl;
    gm[ta] = expf(excl + g0);
    gm[tb] = expf(incl);
    bt[ta] = b0;
    bt[tb] = b1;
  }
  __syncthreads();
  // K K^T and Q K^T over the lower triangle, a 4 x 4 block of (t, s) per
  // thread: L (strictly lower, scaled by b_t G_t/G_s) and the masked Q K^T.
  {
    const int bt4 = (tid / 16) * 4, bs4 = (tid % 16) * 4;
    if (bs4 <= bt4 + 3) {
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) kk[a][b] = qk[a][b] = 0.0f;
#pragma unroll 4
      for (int d = 0; d < DK; ++d) {
        float kt[4], qt[4], ks[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          kt[a] = Ks[(bt4 + a) * (DK + 1) + d];
          qt[a] = Qs[(bt4 + a) * (DK + 1) + d];
          ks[a] = Ks[(bs4 + a) * (DK + 1) + d];
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            kk[a][b] = __fmaf_rn(kt[a], ks[b], kk[a][b]);
            qk[a][b] = __fmaf_rn(qt[a], ks[b], qk[a][b]);
          }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int t = bt4 + a, s = bs4 + b;
          float l = 0.0f, q = 0.0f;
          if (s <= t && t < tn) {
            const float ratio = expf(lg[t] - lg[s]);
            q = qk[a][b] * ratio;
            l = s < t ? bt[t] * ratio * kk[a][b] : 0.0f;
          }
          L[t * (CK + 1) + s] = l;
          o.QK[t][s] = q;
        }
    } else {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          L[(bt4 + a) * (CK + 1) + bs4 + b] = 0.0f;
          o.QK[bt4 + a][bs4 + b] = 0.0f;
        }
    }
  }
  // T = (I + L)^-1 (unit lower triangular), blocked by 16. The diagonal
  // blocks by forward substitution, one warp each (lane = column, so every
  // lane reads only the column it writes):
  //   T[t][s] = -sum_{u=s}^{t-1} L[t][u] T[u][s] (s < t), T[t][t] = 1;
  // then the block rows in order, all blocks of a row at once:
  //   X_ij = sum_{k=j}^{i-1} L_ik T_kj,   T_ij = -T_ii X_ij   (j < i).
  __syncthreads();
  {
    constexpr int NB = CK / 16;
    const int warp = tid / 32, lane = tid % 32;
    for (int i = tid; i < CK * CK; i += 256) {
      const int t = i / CK, s = i % CK;
      if (s / 16 != t / 16) T[t * (CK + 1) + s] = 0.0f;
    }
    if (warp < NB && lane < 16) {
      const int b0 = warp * 16, s = b0 + lane;
      for (int t = b0; t < b0 + 16; ++t) {
        float acc = 0.0f;
        for (int u = s; u < t; ++u) acc = __fmaf_rn(L[t * (CK + 1) + u], T[u * (CK + 1) + s], acc);
        T[t * (CK + 1) + s] = s < t ? -acc : (s == t ? 1.0f : 0.0f);
      }
    } else if (warp >= NB) {
      // The other warps bring V into Q's buffer (Q K^T is done).
      for (int i = tid - NB * 32; i < CK * (DK / 4); i += 256 - NB * 32) {
        const int t = i / (DK / 4), d = (i % (DK / 4)) * 4;
        float4 v4 = make_float4(0, 0, 0, 0);
        if (t < tn) v4 = *reinterpret_cast<const float4*>(vb + size_t(t0 + t) * a.ld_v + d);
        float* vd = Vs + t * (DK + 1) + d;
        vd[0] = v4.x; vd[1] = v4.y; vd[2] = v4.z; vd[3] = v4.w;
      }
    }
    __syncthreads();
    float* X = Xs;  // [NB - 1][16][16]
    for (int bi_ = 1; bi_ < NB; ++bi_) {
      for (int e = tid; e < bi_ * 256; e += 256) {
        const int j = e / 256, r = (e / 16) % 16, cc = e % 16;
        const int t = bi_ * 16 + r, s = j * 16 + cc;
        float acc = 0.0f;
        for (int u = j * 16; u < bi_ * 16; ++u) acc = __fmaf_rn(L[t * (CK + 1) + u], T[u * (CK + 1) + s], acc);
        X[e] = acc;
      }
      __syncthreads();
      for (int e = tid; e < bi_ * 256; e += 256) {
        const int j = e / 256, r = (e / 16) % 16, cc = e % 16;
        const int t = bi_ * 16 + r;
        float acc = 0.0f;
        for (int u = 0; u <= r; ++u) acc = __fmaf_rn(T[t * (CK + 1) + bi_ * 16 + u], X[j * 256 + u * 16 + cc], acc);
        T[t * (CK + 1) + j * 16 + cc] = -acc;
      }
      __syncthreads();
    }
  }
  // U = T diag(b) V and W = T diag(b G) K: a 4-row x 8-column block per thread.
  {
    const int t4 = (tid / 16) * 4, d8 = (tid % 16) * 8;
    float u[4][8], w[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int e = 0; e < 8; ++e) u[a][e] = w[a][e] = 0.0f;
    for (int s = 0; s <= t4 + 3; ++s) {
      float tb[4], tg[4], vv[8], kv[8];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        tb[a] = T[(t4 + a) * (CK + 1) + s] * bt[s];  // zero above the diagonal
        tg[a] = tb[a] * gm[s];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        vv[e] = Vs[s * (DK + 1) + d8 + e];
        kv[e] = Ks[s * (DK + 1) + d8 + e];
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          u[a][e] = __fmaf_rn(tb[a], vv[e], u[a][e]);
          w[a][e] = __fmaf_rn(tg[a], kv[e], w[a][e]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float4* uo = reinterpret_cast<float4*>(&o.U[t4 + a][d8]);
      float4* wo = reinterpret_cast<float4*>(&o.W[t4 + a][d8]);
      uo[0] = make_float4(u[a][0], u[a][1], u[a][2], u[a][3]);
      uo[1] = make_float4(u[a][4], u[a][5], u[a][6], u[a][7]);
      wo[0] = make_float4(w[a][0], w[a][1], w[a][2], w[a][3]);
      wo[1] = make_float4(w[a][4], w[a][5], w[a][6], w[a][7]);
    }
  }
  if (tid < CK) {
    const float last = lg[max(tn - 1, 0)];
    o.gam[tid] = tid < tn ? gm[tid] : 0.0f;
    o.rem[tid] = tid < tn ? expf(last - lg[tid]) : 0.0f;
    if (tid == 0) o.gC = expf(last);
  }
}

// Sequential pass over the chunks for one sequence, head and SC value
// columns: D = U - W S0 and S_C = G_C S0 + K^T diag(G_C / G) D. The state
// slice S[128][SC] stays in shared memory; chunk c + 1's W, K, U slice and
// decay are copied in (cp.async) while chunk c is computed. Each chunk's
// starting state and D go to `states` for the output pass.
constexpr int SCAN_LD = DK + 4;  // padded row stride, keeps 16-byte alignment
template <int SC>
struct ScanStage {
  float W[CK][SCAN_LD];
  float K[CK][SCAN_LD];
  float U[CK][SC];
  float rem[CK];
};

__device__ __forceinline__ void cp16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}

// NT threads, register tiles: with CQ = SC / 4 column quads and
// NG = NT / CQ row groups, thread (g, q) (g = tid / CQ, q = tid % CQ) owns
// in D = U - W S0 the rows g + NG r (r < 64 / NG) and in the state update the
// rows 4g + (r % 4) + 64 (r / 4) (r < 128 / NG), each at columns
// 4q .. 4q + 3. Every output keeps the single
// FMA chain, in the same order, of a one-output-per-thread formulation, so
// the results do not depend on the tiling; the tiles cut the shared-memory
// operand traffic per FMA.
template <int NT, int SC>
__global__ void __launch_bounds__(NT) delta_chunk_scan_kernel(DeltaArgs a, const ChunkOut* __restrict__ outs,
                                                              ChunkState* __restrict__ states, int chunks) {
  constexpr int CQ = SC / 4, SCAN_THREADS = NT, NG = NT / CQ, RD = CK / NG, RS = DK / NG;
  static_assert(RD >= 1 && RS % 4 == 0 && (RS == 4 || NG == 16), "tile shape");
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) float sm[];
  float* S = sm;                                            // [DK][SC]
  float* D = S + DK * SC;                                   // [CK][SC]
  ScanStage<SC>* stg = reinterpret_cast<ScanStage<SC>*>(D + CK * SC);  // [2]
  const int tid = threadIdx.x;
  const int groups = a.dv / SC;
  const int slice = blockIdx.x % groups, h = (blockIdx.x / groups) % a.value_heads;
  const size_t bi = blockIdx.x / (groups * a.value_heads);
  const int kh = h / (a.value_heads / a.key_heads), j0 = slice * SC;
  const float* kb = a.k + bi * a.bs_qkv + kh * DK;
  float* Sg = a.state + bi * a.bs_state + size_t(h) * DK * a.dv;
  const size_t head = bi * a.value_heads + h;
  auto stage = [&](int c, ScanStage<SC>& st) {
    const ChunkOut& co = outs[head * chunks + c];
    const int t0 = c * CK, tn = min(CK, a.n - t0);
    for (int i = tid; i < CK * (DK / 4); i += SCAN_THREADS) {
      const int t = i / (DK / 4), d = (i % (DK / 4)) * 4;
      cp16(&st.W[t][d], &co.W[t][d], 16);
      // K rows past the sequence are zero-filled (never read from memory).
      cp16(&st.K[t][d], t < tn ? kb + size_t(t0 + t) * a.ld_qk + d : kb, t < tn ? 16 : 0);
    }
    for (int i = tid; i < CK * (SC / 4); i += SCAN_THREADS) {
      const int t = i / (SC / 4), j4 = (i % (SC / 4)) * 4;
      cp16(&st.U[t][j4], &co.U[t][j0 + j4], 16);
    }
    if (tid < CK / 4) cp16(&st.rem[tid * 4], &co.rem[tid * 4], 16);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int e = tid; e < DK * SC; e += SCAN_THREADS) S[e] = Sg[size_t(e / SC) * a.dv + j0 + e % SC];
  stage(0, stg[0]);
  const int g = tid / CQ, jc = (tid % CQ) * 4;
  for (int c = 0; c < chunks; ++c) {
    const ScanStage<SC>& st = stg[c & 1];
    ChunkState& cs = states[head * chunks + c];
    const int t0 = c * CK, tn = min(CK, a.n - t0);
    if (c + 1 < chunks) {
      stage(c + 1, stg[(c + 1) & 1]);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    // The state this chunk starts from, for the output pass.
    for (int e = tid; e < DK * (SC / 4); e += SCAN_THREADS) {
      const int i = e / (SC / 4), j4 = (e % (SC / 4)) * 4;
      *reinterpret_cast<float4*>(&cs.S[i][j0 + j4]) = *reinterpret_cast<const float4*>(S + i * SC + j4);
    }
    // D = U - W S0: rows g + NG r, columns jc .. jc + 3.
    {
      float ws[RD][4];
#pragma unroll
      for (int r = 0; r < RD; ++r)
#pragma unroll
        for (int e = 0; e < 4; ++e) ws[r][e] = 0.0f;
#pragma unroll 2
      for (int i = 0; i < DK; i += 4) {
        float4 w4[RD];
#pragma unroll
        for (int r = 0; r < RD; ++r) w4[r] = *reinterpret_cast<const float4*>(&st.W[g + NG * r][i]);
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) {
          const float4 s4 = *reinterpret_cast<const float4*>(S + (i + ii) * SC + jc);
#pragma unroll
          for (int r = 0; r < RD; ++r) {
            const float wv = ii == 0 ? w4[r].x : ii == 1 ? w4[r].y : ii == 2 ? w4[r].z : w4[r].w;
            ws[r][0] = __fmaf_rn(wv, s4.x, ws[r][0]);
            ws[r][1] = __fmaf_rn(wv, s4.y, ws[r][1]);
            ws[r][2] = __fmaf_rn(wv, s4.z, ws[r][2]);
            ws[r][3] = __fmaf_rn(wv, s4.w, ws[r][3]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RD; ++r) {
        const int t = g + NG * r;
        const float4 u4 = *reinterpret_cast<const float4*>(&st.U[t][jc]);
        const bool live = t < tn;
        const float4 d4 = make_float4(live ? u4.x - ws[r][0] : 0.0f, live ? u4.y - ws[r][1] : 0.0f,
                                      live ? u4.z - ws[r][2] : 0.0f, live ? u4.w - ws[r][3] : 0.0f);
        *reinterpret_cast<float4*>(D + t * SC + jc) = d4;
        *reinterpret_cast<float4*>(&cs.D[t][j0 + jc]) = d4;
      }
    }
    __syncthreads();
    // S_C = G_C S0 + K^T diag(G_C / G) D: rows 4g + (r % 4) + 64 (r / 4).
    {
      const float gC = outs[head * chunks + c].gC;
      float acc[RS][4];
#pragma unroll
      for (int r = 0; r < RS; ++r) {
        const int i = 4 * g + (r % 4) + 64 * (r / 4);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[r][e] = gC * S[i * SC + jc + e];
      }
#pragma unroll 4
      for (int s2 = 0; s2 < CK; ++s2) {
        const float rs = st.rem[s2];
        float kv[RS];
#pragma unroll
        for (int r4 = 0; r4 < RS / 4; ++r4) {
          const float4 k4 = *reinterpret_cast<const float4*>(&st.K[s2][4 * g + 64 * r4]);
          kv[4 * r4] = k4.x;
          kv[4 * r4 + 1] = k4.y;
          kv[4 * r4 + 2] = k4.z;
          kv[4 * r4 + 3] = k4.w;
        }
        const float4 d4 = *reinterpret_cast<const float4*>(D + s2 * SC + jc);
#pragma unroll
        for (int r = 0; r < RS; ++r) {
          const float kr = kv[r] * rs;
          acc[r][0] = __fmaf_rn(kr, d4.x, acc[r][0]);
          acc[r][1] = __fmaf_rn(kr, d4.y, acc[r][1]);
          acc[r][2] = __fmaf_rn(kr, d4.z, acc[r][2]);
          acc[r][3] = __fmaf_rn(kr, d4.w, acc[r][3]);
        }
      }
      __syncthreads();  // every thread has read the old S (and this stage)
#pragma unroll
      for (int r = 0; r < RS; ++r) {
        const int i = 4 * g + (r % 4) + 64 * (r / 4);
        *reinterpret_cast<float4*>(S + i * SC + jc) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
      }
    }
    __syncthreads();
  }
  for (int e = tid; e < DK * SC; e += SCAN_THREADS) Sg[size_t(e / SC) * a.dv + j0 + e % SC] = S[e];
}

// O = diag(G) Q S0 + (M o Q K^T) D for one chunk, head and 64 value columns,
// all chunks in parallel once the scan has produced every S0 and D.
// Thread -> 4 rows x 4 columns (columns strided by 16: conflict-free loads).
constexpr int OUT_COLS = 64, OQ_LD = DK + 4, OS_LD = OUT_COLS + 4, OK_LD = CK + 4;
__global__ void __launch_bounds__(256) delta_chunk_out_kernel(DeltaArgs a, const ChunkOut* __restrict__ outs,
                                                              const ChunkState* __restrict__ states, int chunks) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;                    // [CK][OQ_LD]
  float* Ss = Qs + CK * OQ_LD;       // [DK][OS_LD]
  float* QKs = Ss + DK * OS_LD;      // [CK][OK_LD]
  float* Ds = QKs + CK * OK_LD;      // [CK][OS_LD]
  const int tid = threadIdx.x;
  const int halves = a.dv / OUT_COLS;
  const int part = blockIdx.x % halves, c = (blockIdx.x / halves) % chunks;
  const int h = (blockIdx.x / (halves * chunks)) % a.value_heads;
  const size_t bi = blockIdx.x / (halves * chunks * a.value_heads);
  const int kh = h / (a.value_heads / a.key_heads), j0 = part * OUT_COLS;
  const int t0 = c * CK, tn = min(CK, a.n - t0);
  const size_t head = bi * a.value_heads + h;
  const ChunkOut& co = outs[head * chunks + c];
  const ChunkState& cs = states[head * chunks + c];
  const float* qb = a.q + bi * a.bs_qkv + kh * DK;
  for (int i = tid; i < CK * (DK / 4); i += 256) {
    const int t = i / (DK / 4), d = (i % (DK / 4)) * 4;
    cp16(Qs + t * OQ_LD + d, t < tn ? qb + size_t(t0 + t) * a.ld_qk + d : qb, t < tn ? 16 : 0);
  }
  for (int i = tid; i < DK * (OUT_COLS / 4); i += 256) {
    const int r = i / (OUT_COLS / 4), j4 = (i % (OUT_COLS / 4)) * 4;
    cp16(Ss + r * OS_LD + j4, &cs.S[r][j0 + j4], 16);
  }
  for (int i = tid; i < CK * (CK / 4); i += 256) {
    const int t = i / (CK / 4), s4 = (i % (CK / 4)) * 4;
    cp16(QKs + t * OK_LD + s4, &co.QK[t][s4], 16);
    cp16(Ds + t * OS_LD + s4, &cs.D[t][j0 + s4], 16);  // OUT_COLS == CK
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int rg = tid / 16, cg = tid % 16, r0 = rg * 4;
  float acc[4][4], y[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = y[i][e] = 0.0f;
#pragma unroll 2
  for (int k = 0; k < DK; k += 4) {
    float4 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = *reinterpret_cast<const float4*>(Qs + (r0 + i) * OQ_LD + k);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float sv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) sv[e] = Ss[(k + kk) * OS_LD + cg + 16 * e];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qv = kk == 0 ? q[i].x : kk == 1 ? q[i].y : kk == 2 ? q[i].z : q[i].w;
#pragma unroll
        for (int e = 0; e < 4; ++e) y[i][e] = __fmaf_rn(qv, sv[e], y[i][e]);
      }
    }
  }
#pragma unroll 2
  for (int s = 0; s < CK; s += 4) {
    float4 m[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = *reinterpret_cast<const float4*>(QKs + (r0 + i) * OK_LD + s);
#pragma unroll
    for (int ss = 0; ss < 4; ++ss) {
      float dv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) dv[e] = Ds[(s + ss) * OS_LD + cg + 16 * e];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float mv = ss == 0 ? m[i].x : ss == 1 ? m[i].y : ss == 2 ? m[i].z : m[i].w;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = __fmaf_rn(mv, dv[e], acc[i][e]);
      }
    }
  }
  float* ob = a.o + bi * a.bs_o + h * a.dv + j0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = r0 + i;
    if (t >= tn) continue;
    const float g = co.gam[t];
#pragma unroll
    for (int e = 0; e < 4; ++e) ob[size_t(t0 + t) * a.ldo + cg + 16 * e] = __fmaf_rn(g, y[i][e], acc[i][e]);
  }
}

}  // namespace

size_t delta_chunk_workspace_bytes(int batch, int heads, int n) {
  const int chunks = (n + CK - 1) / CK;
  return size_t(batch) * heads * chunks * (sizeof(ChunkOut) + sizeof(ChunkState));
}

void launch_delta_chunked(const DeltaArgs& a, int batch, void* workspace, size_t workspace_bytes, cudaStream_t s,
                          bool wide) {
  if (a.n <= 0 || batch <= 0) return;
  if (a.dv != DK || a.value_heads % a.key_heads)
    throw CudaError("delta_chunked: needs dk = dv = 128");
  const int chunks = (a.n + CK - 1) / CK;
  if (workspace_bytes < delta_chunk_workspace_bytes(batch, a.value_heads, a.n))
    throw CudaError("delta_chunked: workspace too small");
  if (a.ld_qk % 4 || a.ld_v % 4 || a.ldo % 4 || reinterpret_cast<uintptr_t>(workspace) % 16 ||
      reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.k) % 16)
    throw CudaError("delta_chunked: rows must be 16-byte aligned");
  const size_t units = size_t(batch) * a.value_heads * chunks;
  ChunkOut* outs = static_cast<ChunkOut*>(workspace);
  ChunkState* states = reinterpret_cast<ChunkState*>(outs + units);
  const int prep_smem = (2 * CK * (DK + 1) + 2 * CK * (CK + 1) + 3 * CK + (CK / 16 - 1) * 256) * sizeof(float);
  auto scan_smem = [](int sc, int stage_bytes) { return (DK * sc + CK * sc) * int(sizeof(float)) + 2 * stage_bytes; };
  const int scan16_smem = scan_smem(16, sizeof(ScanStage<16>)), scan32_smem = scan_smem(32, sizeof(ScanStage<32>));
  const int out_smem = (CK * OQ_LD + DK * OS_LD + CK * OK_LD + CK * OS_LD) * sizeof(float);
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [&] {
    DG_CUDA(cudaFuncSetAttribute(delta_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem));
    DG_CUDA(cudaFuncSetAttribute(delta_chunk_scan_kernel<128, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 scan16_smem));
    DG_CUDA(cudaFuncSetAttribute(delta_chunk_scan_kernel<256, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 scan32_smem));
    DG_CUDA(cudaFuncSetAttribute(delta_chunk_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, out_smem));
  });
  launch_pdl(delta_chunk_prep_kernel, dim3(int(units)), dim3(256), prep_smem, s, a, outs, chunks);
  DG_CUDA(cudaGetLastError());
  // Wide slices once they make at least two waves of scan CTAs, or when
  // asked for (other lanes' kernels fill the SMs the scan leaves free).
  if (wide || size_t(batch) * a.value_heads * (a.dv / 32) >= 2 * 148)
    launch_pdl(delta_chunk_scan_kernel<256, 32>, dim3(batch * a.value_heads * (a.dv / 32)), dim3(256), scan32_smem, s,
               a, outs, states, chunks);
  else
    launch_pdl(delta_chunk_scan_kernel<128, 16>, dim3(batch * a.value_heads * (a.dv / 16)), dim3(128), scan16_smem, s,
               a, outs, states, chunks);
  DG_CUDA(cudaGetLastError());
  launch_pdl(delta_chunk_out_kernel, dim3(int(units) * (a.dv / OUT_COLS)), dim3(256), out_smem, s, a, outs, states, chunks);
  DG_CUDA(cudaGetLastError());
}

}  // namespace dg

