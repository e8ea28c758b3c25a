// Gated GQA attention with partial RoPE and the shared-prefix KV cache, the
// final norm, and the pointer head (src/qwen.rs:530-643, src/lib.rs:106-131).
#include <cfloat>

#include <cooperative_groups.h>

#include "launch.h"

namespace cg = cooperative_groups;

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

// Full::forward's pre-attention steps (src/qwen.rs:542-566): split q|gate per
// head, centred RMSNorm of q and k per head (eps), partial RoPE on pairs
// (i, i + half) from the table rope[pos][i] = (sin, cos), and append the
// normalised, rotated k and the raw v at position start + t. One warp per
// vector (heads q vectors + kv_heads k vectors + kv_heads v vectors per token).
// Segmented forwards (seg_len > 0: rows are consecutive sequences of seg_len
// tokens, each continuing the same `start` positions) put row t at position
// start + t % seg_len and its k and v at row t of kcache / vcache, the
// segment-local buffers the attention reads next to the shared prefix.
__global__ void qk_norm_rope_kernel(const float* __restrict__ qkv, int ldq, int heads, int kv_heads, int d,
                                    const float* __restrict__ qn, const float* __restrict__ kn, float eps,
                                    const float* __restrict__ rope, int half, int start, float* __restrict__ q_out,
                                    float* __restrict__ kcache, float* __restrict__ vcache, int seg_len) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float buf[];  // [warps][d]
  const int t = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  float* x = buf + warp * d;
  const float* row = qkv + size_t(t) * ldq;
  const int pos = start + (seg_len ? t % seg_len : t), kvrow = seg_len ? t : pos, kw = kv_heads * d;
  for (int v = warp; v < heads + 2 * kv_heads; v += nw) {
    const float* src;
    const float* g = nullptr;
    float* dst;
    if (v < heads) {
      src = row + size_t(v) * 2 * d;
      g = qn;
      dst = q_out + (size_t(t) * heads + v) * d;
    } else if (v < heads + kv_heads) {
      const int kh = v - heads;
      src = row + size_t(heads) * 2 * d + kh * d;
      g = kn;
      dst = kcache + size_t(kvrow) * kw + kh * d;
    } else {
      const int kh = v - heads - kv_heads;
      src = row + size_t(heads) * 2 * d + kw + kh * d;
      dst = vcache + size_t(kvrow) * kw + kh * d;
    }
    float ss = 0.0f;
    for (int i = lane; i < d; i += 32) {
      const float a = src[i];
      x[i] = a;
      ss = __fmaf_rn(a, a, ss);
    }
    __syncwarp();
    if (g) {
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / float(d) + eps);
      for (int i = lane; i < d; i += 32) x[i] = x[i] * (inv * (1.0f + g[i]));
      __syncwarp();
      const float* ang = rope + size_t(pos) * half * 2;
      for (int i = lane; i < half; i += 32) {
        const float sn = ang[2 * i], cs = ang[2 * i + 1];
        const float a = x[i], b = x[i + half];
        x[i] = a * cs - b * sn;
        x[i + half] = b * cs + a * sn;
      }
      __syncwarp();
    }
    for (int i = lane; i < d; i += 32) dst[i] = x[i];
    __syncwarp();
  }
}

// Flash-style causal attention for head_dim 256, FP32 throughout. CTA: 16
// query rows of one head (4 warps x 4 rows); key blocks of 32 in shared memory
// (K transposed so lane = key reads conflict-free); online softmax; output
// multiplied by sigmoid(gate) (src/qwen.rs:581-583).
constexpr int AD = 256, ABQ = 16, ABK = 32;
__global__ void __launch_bounds__(128) attention256_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                           const float* __restrict__ vc,
                                                           const float* __restrict__ gate_src, int ld_gate, int n,
                                                           int offset, int heads, int kv_heads,
                                                           float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float sm[];
  float* Qs = sm;                       // [ABQ][AD]
  float* Kt = Qs + ABQ * AD;            // [AD][ABK + 1]
  float* Vs = Kt + AD * (ABK + 1);      // [ABK][AD]
  const int h = blockIdx.y, kh = h / (heads / kv_heads), t0 = blockIdx.x * ABQ;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kw = kv_heads * AD;
  const float scale = 1.0f / sqrtf(float(AD));
  for (int i = threadIdx.x; i < ABQ * AD; i += 128) {
    const int r = i / AD, c = i % AD, t = t0 + r;
    Qs[i] = t < n ? q[(size_t(t) * heads + h) * AD + c] : 0.0f;
  }
  float o[4][AD / 32];
  float mrow[4], lrow[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    mrow[r] = -INFINITY;
    lrow[r] = 0.0f;
#pragma unroll
    for (int e = 0; e < AD / 32; ++e) o[r][e] = 0.0f;
  }
  const int L = offset + n;
  const int last_key = min(L - 1, offset + t0 + ABQ - 1);
  for (int kb = 0; kb <= last_key; kb += ABK) {
    __syncthreads();
    // 32 keys x 256 dims = 2048 float4 per matrix, 16 per thread: issue all
    // loads of a batch before any shared-memory store so their latency overlaps.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float4 kr[8], vr[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = (half * 8 + u) * 128 + threadIdx.x;
        const int key = i / (AD / 4), c = (i % (AD / 4)) * 4, s = kb + key;
        if (s < L) {
          kr[u] = __ldg(reinterpret_cast<const float4*>(kc + size_t(s) * kw + kh * AD + c));
          vr[u] = __ldg(reinterpret_cast<const float4*>(vc + size_t(s) * kw + kh * AD + c));
        } else {
          kr[u] = vr[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = (half * 8 + u) * 128 + threadIdx.x;
        const int key = i / (AD / 4), c = (i % (AD / 4)) * 4;
        Kt[(c + 0) * (ABK + 1) + key] = kr[u].x;
        Kt[(c + 1) * (ABK + 1) + key] = kr[u].y;
        Kt[(c + 2) * (ABK + 1) + key] = kr[u].z;
        Kt[(c + 3) * (ABK + 1) + key] = kr[u].w;
        *reinterpret_cast<float4*>(&Vs[key * AD + c]) = vr[u];
      }
    }
    __syncthreads();
    float sc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) sc[r] = 0.0f;
    const float* qrow = Qs + (warp * 4) * AD;
#pragma unroll 8
    for (int c = 0; c < AD; ++c) {
      const float kv = Kt[c * (ABK + 1) + lane];
#pragma unroll
      for (int r = 0; r < 4; ++r) sc[r] = __fmaf_rn(qrow[r * AD + c], kv, sc[r]);
    }
    const int key = kb + lane;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = t0 + warp * 4 + r;
      float s = sc[r] * scale;
      if (key > offset + t || key >= L) s = -INFINITY;
      const float mx = warp_max(s);
      const float mnew = fmaxf(mrow[r], mx);
      const float p = s == -INFINITY ? 0.0f : expf(s - mnew);
      const float corr = mrow[r] == -INFINITY ? 0.0f : expf(mrow[r] - mnew);
      lrow[r] = lrow[r] * corr + warp_sum(p);
      mrow[r] = mnew;
#pragma unroll
      for (int e = 0; e < AD / 32; ++e) o[r][e] = o[r][e] * corr;
      sc[r] = p;
    }
#pragma unroll 4
    for (int k2 = 0; k2 < ABK; ++k2) {
      float pk[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) pk[r] = __shfl_sync(0xffffffffu, sc[r], k2);
#pragma unroll
      for (int e = 0; e < AD / 32; ++e) {
        const float v = Vs[k2 * AD + lane + 32 * e];
#pragma unroll
        for (int r = 0; r < 4; ++r) o[r][e] = __fmaf_rn(pk[r], v, o[r][e]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = t0 + warp * 4 + r;
    if (t >= n) continue;
    const float inv = 1.0f / lrow[r];
#pragma unroll
    for (int e = 0; e < AD / 32; ++e) {
      const int c = lane + 32 * e;
      const float g = gate_src[size_t(t) * ld_gate + size_t(h) * 2 * AD + AD + c];
      out[size_t(t) * heads * AD + h * AD + c] = (o[r][e] * inv) * sigmoid_f(g);
    }
  }
}

// Flash-style causal attention for head_dim 256, FP32, register-tiled, with
// the key blocks of each 32-row query block dealt round-robin to a cluster of
// NS CTAs (2, 4 or 8).
// Each CTA stages key blocks of 32 in shared memory with cp.async (the next
// block's K is copied in during this block's softmax and P·V, its V during the
// next Q·Kᵀ). Thread (rg, kg) = (tid / 16, tid % 16) owns rows 2rg, 2rg + 1:
// scores against keys kg and kg + 16 of a block, outputs in columns
// 4 kg + 64 j .. + 3. Online softmax per row across its 16 threads. CTA 1 of
// the pair leaves its unnormalised (m, l, o) in shared memory; CTA 0 reads them
// through distributed shared memory, merges, divides and multiplies by
// sigmoid(gate) (src/qwen.rs:581-583). Heavy (late) query blocks go first.
// With NS > 2 every CTA but the first publishes, and CTA 0 merges the NS
// partial states in rank order (for NS = 2 the same expression as a pair).
constexpr int TQ = 32, TK = 32, TLD = AD + 4, PLD = TQ + 4;
constexpr int ATT_SMEM = (TQ * TLD + TK * TLD + TK * AD + TK * PLD + 2 * TQ) * 4;

__device__ __forceinline__ void att_cp16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void att_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void att_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

//
// Segmented forwards (seg_len > 0): the rows are nseg consecutive sequences of
// seg_len tokens, each continuing the same `offset` prefix positions. Keys
// below `offset` come from kc / vc (the shared prefix), the rest from the
// sequence's own rows of kc_own / vc_own; query block b of the grid is block
// b / nseg (latest first) of sequence b % nseg. A sequence's key blocks are
// the same absolute positions as in a forward of that sequence alone, so each
// row's arithmetic is the same.
template <int NS>
__global__ void __cluster_dims__(NS, 1, 1) __launch_bounds__(256)
    attention256_split_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                              const float* __restrict__ gate_src, int ld_gate, int n, int offset, int heads,
                              int kv_heads, float* __restrict__ out, int seg_len, int nseg,
                              const float* __restrict__ kc_own, const float* __restrict__ vc_own) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;               // [TQ][TLD]
  float* Ks = Qs + TQ * TLD;    // [TK][TLD]; at the end CTA 1's o [TQ][TLD]
  float* Vs = Ks + TK * TLD;    // [TK][AD]
  float* PT = Vs + TK * AD;     // [TK][PLD]: probabilities, key-major
  float* ML = PT + TK * PLD;    // [2][TQ]: CTA 1's running max and sum
  cg::cluster_group cluster = cg::this_cluster();
  const int part = int(cluster.block_rank());
  if (seg_len) n = seg_len;  // rows of this block's sequence
  const int nrb = (n + TQ - 1) / TQ, b = int(blockIdx.x / NS);
  const int seg = seg_len ? b % nseg : 0, row0 = seg * n;  // the sequence's first row in q, gate and out
  const int rb = nrb - 1 - (seg_len ? b / nseg : b), h = blockIdx.y, kh = h / (heads / kv_heads);
  const int t0 = rb * TQ, tid = threadIdx.x, rg = tid / 16, kg = tid % 16;
  const int kw = kv_heads * AD, L = offset + n;
  const int last_key = min(L - 1, offset + t0 + TQ - 1), nkb = last_key / TK + 1;
  // CTA `part` takes key blocks part, part + NS, ...: every query row sees the
  // same split and merge whatever block it sits in, so for one NS a prefix
  // continuation reproduces the full forward bit for bit.
  const int kb_begin = part, kb_end = nkb;
  const float scale = 1.0f / sqrtf(float(AD));
  auto load_rows = [&](float* dst, int ld, const float* src, const float* own, int k0) {
    for (int i = tid; i < TK * (AD / 4); i += 256) {
      const int r = i / (AD / 4), c = (i % (AD / 4)) * 4, s = k0 + r;
      const float* p = src;
      if (s < L) p = (!seg_len || s < offset) ? src + size_t(s) * kw + kh * AD + c
                                              : own + size_t(row0 + s - offset) * kw + kh * AD + c;
      att_cp16(dst + r * ld + c, p, s < L);
    }
  };
  for (int i = tid; i < TQ * (AD / 4); i += 256) {
    const int r = i / (AD / 4), c = (i % (AD / 4)) * 4, t = t0 + r;
    att_cp16(Qs + r * TLD + c, t < n ? q + (size_t(row0 + t) * heads + h) * AD + c : q, t < n);
  }
  if (kb_begin < kb_end) {
    load_rows(Ks, TLD, kc, kc_own, kb_begin * TK);
    att_commit();
    load_rows(Vs, AD, vc, vc_own, kb_begin * TK);
  }
  att_commit();
  float o[2][16], mrow[2], lrow[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) o[i][e] = 0.0f;
  }
  for (int kb = kb_begin; kb < kb_end; kb += NS) {
    const int k0 = kb * TK;
    att_wait<1>();  // this block's K (and Q) have landed
    __syncthreads();
    float sc[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) sc[i][0] = sc[i][1] = 0.0f;
#pragma unroll 4
    for (int c = 0; c < AD; c += 4) {
      float4 qv[2], kv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (2 * rg + i) * TLD + c);
#pragma unroll
      for (int j = 0; j < 2; ++j) kv[j] = *reinterpret_cast<const float4*>(Ks + (kg + 16 * j) * TLD + c);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          sc[i][j] = __fmaf_rn(qv[i].x, kv[j].x, sc[i][j]);
          sc[i][j] = __fmaf_rn(qv[i].y, kv[j].y, sc[i][j]);
          sc[i][j] = __fmaf_rn(qv[i].z, kv[j].z, sc[i][j]);
          sc[i][j] = __fmaf_rn(qv[i].w, kv[j].w, sc[i][j]);
        }
    }
    __syncthreads();  // every thread is done with Ks
    if (kb + NS < kb_end) {
      load_rows(Ks, TLD, kc, kc_own, k0 + NS * TK);
      att_commit();
      att_wait<1>();  // this block's V has landed
    } else {
      att_wait<0>();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = t0 + 2 * rg + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = k0 + kg + 16 * j;
        float s = sc[i][j] * scale;
        if (key > offset + t || key >= L) s = -INFINITY;
        sc[i][j] = s;
        mx = fmaxf(mx, s);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(mrow[i], mx);
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float p = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - mnew);
        PT[(kg + 16 * j) * PLD + 2 * rg + i] = p;
        psum += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      const float corr = mrow[i] == -INFINITY ? 0.0f : expf(mrow[i] - mnew);
      lrow[i] = lrow[i] * corr + psum;
      mrow[i] = mnew;
#pragma unroll
      for (int e = 0; e < 16; ++e) o[i][e] *= corr;
    }
    __syncthreads();  // PT and this block's V are visible
    const int nk = min(TK, last_key + 1 - k0);
#pragma unroll 4
    for (int s = 0; s < nk; ++s) {
      const float2 p = *reinterpret_cast<const float2*>(PT + s * PLD + 2 * rg);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(Vs + s * AD + 4 * kg + 64 * j);
        o[0][4 * j + 0] = __fmaf_rn(p.x, v.x, o[0][4 * j + 0]);
        o[0][4 * j + 1] = __fmaf_rn(p.x, v.y, o[0][4 * j + 1]);
        o[0][4 * j + 2] = __fmaf_rn(p.x, v.z, o[0][4 * j + 2]);
        o[0][4 * j + 3] = __fmaf_rn(p.x, v.w, o[0][4 * j + 3]);
        o[1][4 * j + 0] = __fmaf_rn(p.y, v.x, o[1][4 * j + 0]);
        o[1][4 * j + 1] = __fmaf_rn(p.y, v.y, o[1][4 * j + 1]);
        o[1][4 * j + 2] = __fmaf_rn(p.y, v.z, o[1][4 * j + 2]);
        o[1][4 * j + 3] = __fmaf_rn(p.y, v.w, o[1][4 * j + 3]);
      }
    }
    __syncthreads();  // every thread is done with Vs and PT
    if (kb + NS < kb_end) {
      load_rows(Vs, AD, vc, vc_own, k0 + NS * TK);
      att_commit();
    }
  }
  att_wait<0>();
  // Merge the key parts: CTAs 1 .. NS-1 publish, CTA 0 combines and stores.
  if (part != 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float* dst = Ks + (2 * rg + i) * TLD;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4*>(dst + 4 * kg + 64 * j) =
            make_float4(o[i][4 * j], o[i][4 * j + 1], o[i][4 * j + 2], o[i][4 * j + 3]);
      if (kg == 0) {
        ML[2 * rg + i] = mrow[i];
        ML[TQ + 2 * rg + i] = lrow[i];
      }
    }
  }
  cluster.sync();
  if (part == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = t0 + 2 * rg + i;
      float mm = mrow[i];
#pragma unroll
      for (int r = 1; r < NS; ++r) mm = fmaxf(mm, cluster.map_shared_rank(ML, r)[2 * rg + i]);
      const float a0 = mrow[i] == -INFINITY ? 0.0f : expf(mrow[i] - mm);
      float lsum = lrow[i] * a0;
#pragma unroll
      for (int j = 0; j < 16; ++j) o[i][j] = o[i][j] * a0;
#pragma unroll
      for (int r = 1; r < NS; ++r) {
        const float* rML = cluster.map_shared_rank(ML, r);
        const float mr = rML[2 * rg + i], lr = rML[TQ + 2 * rg + i];
        const float ar = mr == -INFINITY ? 0.0f : expf(mr - mm);
        lsum = lsum + lr * ar;
        const float* orow = cluster.map_shared_rank(Ks, r) + (2 * rg + i) * TLD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 rv = *reinterpret_cast<const float4*>(orow + 4 * kg + 64 * j);
          o[i][4 * j + 0] = o[i][4 * j + 0] + rv.x * ar;
          o[i][4 * j + 1] = o[i][4 * j + 1] + rv.y * ar;
          o[i][4 * j + 2] = o[i][4 * j + 2] + rv.z * ar;
          o[i][4 * j + 3] = o[i][4 * j + 3] + rv.w * ar;
        }
      }
      const float inv = 1.0f / lsum;
      if (t >= n) continue;
      const float* g = gate_src + size_t(row0 + t) * ld_gate + size_t(h) * 2 * AD + AD;
      float* dst = out + (size_t(row0 + t) * heads + h) * AD;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 4 * kg + 64 * j;
        float4 r;
        r.x = (o[i][4 * j + 0] * inv) * sigmoid_f(g[c + 0]);
        r.y = (o[i][4 * j + 1] * inv) * sigmoid_f(g[c + 1]);
        r.z = (o[i][4 * j + 2] * inv) * sigmoid_f(g[c + 2]);
        r.w = (o[i][4 * j + 3] * inv) * sigmoid_f(g[c + 3]);
        *reinterpret_cast<float4*>(dst + c) = r;
      }
    }
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until CTA 0 has read it
}

// Generic causal attention (any head_dim): one thread per (token, head),
// reference order (causal_attention, src/qwen.rs:610-629) with the scores
// recomputed per pass instead of buffered.
__global__ void attention_generic_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                         const float* __restrict__ vc, const float* __restrict__ gate_src, int ld_gate,
                                         int n, int offset, int heads, int kv_heads, int d, float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int id = blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n * heads) return;
  const int t = id / heads, h = id % heads, kh = h / (heads / kv_heads), kw = kv_heads * d;
  const float scale = 1.0f / sqrtf(float(d));
  const float* qr = q + (size_t(t) * heads + h) * d;
  auto score = [&](int s) {
    const float* kr = kc + size_t(s) * kw + kh * d;
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int full = (d / 8) * 8;
    for (int i = 0; i < full; ++i) lanes[i & 7] = lanes[i & 7] + qr[i] * kr[i];
    float sum = -0.0f;
    for (int i = 0; i < 8; ++i) sum = sum + lanes[i];
    for (int i = full; i < d; ++i) sum = sum + qr[i] * kr[i];
    return sum * scale;
  };
  float mx = -INFINITY;
  for (int s = 0; s <= offset + t; ++s) mx = fmaxf(mx, score(s));
  float total = 0.0f;
  for (int s = 0; s <= offset + t; ++s) total = total + expf(score(s) - mx);
  float* dst = out + size_t(t) * heads * d + h * d;
  for (int i = 0; i < d; ++i) dst[i] = 0.0f;
  for (int s = 0; s <= offset + t; ++s) {
    float p = expf(score(s) - mx);
    if (total > 0.0f) p = p / total;
    const float* vr = vc + size_t(s) * kw + kh * d;
    for (int i = 0; i < d; ++i) dst[i] = dst[i] + p * vr[i];
  }
  for (int i = 0; i < d; ++i)
    dst[i] = dst[i] * sigmoid_f(gate_src[size_t(t) * ld_gate + size_t(h) * 2 * d + d + i]);
}

// rms (centred) in place, src/qwen.rs:495, plus the non-finite hidden-state
// check of src/qwen.rs:496-498. One 256-thread CTA per row.
__global__ void final_norm_kernel(float* __restrict__ x, int K, const float* __restrict__ g, float eps,
                                  DeviceStatus* st) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[8];
  __shared__ int bad;
  float* r = x + size_t(blockIdx.x) * K;
  if (threadIdx.x == 0) bad = 0;
  float ss = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) ss = __fmaf_rn(r[k], r[k], ss);
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  float tot = threadIdx.x < 8 ? red[threadIdx.x] : 0.0f;
  if (threadIdx.x < 32) tot = warp_sum(tot);
  __syncthreads();
  if (threadIdx.x == 0) red[0] = tot;
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / float(K) + eps);
  int local_bad = 0;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = r[k] * (inv * (1.0f + g[k]));
    r[k] = v;
    local_bad |= !isfinite(v);
  }
  if (local_bad) bad = 1;
  __syncthreads();
  if (threadIdx.x == 0 && bad) report(st, kNonFinite, 3);
}

// Head::normalize, src/lib.rs:106-115: mean, biased variance, eps 1e-5.
__global__ void head_norm_kernel(const float* __restrict__ hidden, int K, const int* __restrict__ rows,
                                 const float* __restrict__ w, const float* __restrict__ b, float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  __shared__ float red[8];
  __shared__ float bc;
  const float* x = hidden + size_t(rows[blockIdx.x]) * K;
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    __syncthreads();
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.0f;
      t = warp_sum(t);
      if (threadIdx.x == 0) bc = t;
    }
    __syncthreads();
    return bc;
  };
  float s = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) s += x[k];
  const float mean = block_sum(s) / float(K);
  float v2 = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float d = x[k] - mean;
    v2 = __fmaf_rn(d, d, v2);
  }
  const float var = block_sum(v2) / float(K);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (int k = threadIdx.x; k < K; k += 256)
    out[size_t(blockIdx.x) * K + k] = (x[k] - mean) * inv * w[k] + b[k];
}

// logits[i] = dot_scores(q + bq, k_i + bk) * scale (src/lib.rs:120-128: the
// head projections add their bias to the dot, then the query-key dot).
__global__ void head_dot_kernel(const float* __restrict__ q, const float* __restrict__ k, int n_keys, int dim,
                                float scale, const float* __restrict__ bq, const float* __restrict__ bk,
                                float* __restrict__ logits) {
  griddep_wait();
  griddep_launch();
  // One warp per key; lane l < 8 runs the reference's lane l (indices l, l+8, ...).
  const int i = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
  if (i >= n_keys) return;
  const float* kr = k + size_t(i) * dim;
  auto qv = [&](int j) { return bq ? q[j] + bq[j] : q[j]; };
  auto kv = [&](int j) { return bk ? kr[j] + bk[j] : kr[j]; };
  const int full = (dim / 8) * 8;
  float chain = 0.0f;
  if (lane < 8) {
#pragma unroll 8
    for (int j = lane; j < full; j += 8) chain = chain + qv(j) * kv(j);
  }
  float s = -0.0f;
#pragma unroll
  for (int l = 0; l < 8; ++l) s = s + __shfl_sync(0xffffffffu, chain, l);
  if (lane == 0) {
    for (int j = full; j < dim; ++j) s = s + qv(j) * kv(j);
    logits[i] = s * scale;
  }
}

}  // namespace

void launch_qk_norm_rope(const float* qkv, int ldq, int n, int heads, int kv_heads, int d, const float* qn,
                         const float* kn, float eps, const float* rope, int half, int start, float* q_out,
                         float* kcache, float* vcache, cudaStream_t s, int seg_len) {
  if (n <= 0) return;
  if (seg_len < 0 || (seg_len && n % seg_len)) throw CudaError("qk_norm_rope: rows must be whole segments");
  launch_pdl(qk_norm_rope_kernel, dim3(n), dim3(256), 8 * d * sizeof(float), s, qkv, ldq, heads, kv_heads, d, qn, kn, eps, rope, half,
                                                            start, q_out, kcache, vcache, seg_len);
  DG_CUDA(cudaGetLastError());
}

template <int NS>
void launch_attention_split(const float* q, const float* kcache, const float* vcache, const float* gate_src,
                            int ld_gate, int n, int offset, int heads, int kv_heads, float* out, cudaStream_t s,
                            int seg_len, const float* kc_own, const float* vc_own) {
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    DG_CUDA(cudaFuncSetAttribute(attention256_split_kernel<NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ATT_SMEM));
  });
  const int nl = seg_len ? seg_len : n, nseg = seg_len ? n / seg_len : 1;
  dim3 grid(NS * nseg * ((nl + TQ - 1) / TQ), heads);  // clusters of NS along x
  launch_pdl(attention256_split_kernel<NS>, dim3(grid), dim3(256), ATT_SMEM, s, q, kcache, vcache, gate_src, ld_gate,
             n, offset, heads, kv_heads, out, seg_len, nseg, kc_own, vc_own);
}

// Cluster size of the split kernel. Reference order keeps pairs, so that a
// prefix continuation (few query rows after a long prefix) splits its keys as
// the full forward does and reproduces it bit for bit. Otherwise the cluster
// grows (4, then 8) while the grid has fewer than two CTAs per SM and every
// CTA keeps at least two key blocks: a 64-token question after a 3584-token
// prefix is 2 query blocks x 8 heads, 32 CTAs in pairs.
int attention_split_ways(int n, int offset, int heads, bool exact, int nseg) {
  if (exact) return 2;
  const int nrb = nseg * ((n + TQ - 1) / TQ), nkb = (offset + n + TK - 1) / TK;
  int ns = 2;
  while (ns < 8 && ns * nrb * heads < 2 * 148 && nkb / (2 * ns) >= 2) ns *= 2;
  return ns;
}

void launch_attention(const float* q, const float* kcache, const float* vcache, const float* gate_src, int ld_gate,
                      int n, int offset, int heads, int kv_heads, int d, float* out, bool exact, cudaStream_t s,
                      int seg_len, const float* kc_own, const float* vc_own) {
  if (n <= 0) return;
  const bool aligned = reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(kcache) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(vcache) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(kc_own) % 16 == 0 && reinterpret_cast<uintptr_t>(vc_own) % 16 == 0;
  if (seg_len) {
    // Segmented forwards have only the head_dim-256 kernel.
    if (seg_len < 0 || n % seg_len || d != AD || !aligned || !kc_own || !vc_own)
      throw CudaError("attention: segmented rows need head_dim 256, aligned buffers and whole segments");
  }
  if (d == AD && aligned) {
    const int nl = seg_len ? seg_len : n, nseg = seg_len ? n / seg_len : 1;
    const int ns = attention_split_ways(nl, offset, heads, exact, nseg);
    if (ns == 8)
      launch_attention_split<8>(q, kcache, vcache, gate_src, ld_gate, n, offset, heads, kv_heads, out, s, seg_len, kc_own,
                                vc_own);
    else if (ns == 4)
      launch_attention_split<4>(q, kcache, vcache, gate_src, ld_gate, n, offset, heads, kv_heads, out, s, seg_len, kc_own,
                                vc_own);
    else
      launch_attention_split<2>(q, kcache, vcache, gate_src, ld_gate, n, offset, heads, kv_heads, out, s, seg_len, kc_own,
                                vc_own);
  } else if (d == AD) {
    const int smem = (ABQ * AD + AD * (ABK + 1) + ABK * AD) * sizeof(float);
    static std::atomic<uint64_t> configured{0};
    once_per_device(configured, [&] {
      DG_CUDA(cudaFuncSetAttribute(attention256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    });
    dim3 grid((n + ABQ - 1) / ABQ, heads);
    launch_pdl(attention256_kernel, dim3(grid), dim3(128), smem, s, q, kcache, vcache, gate_src, ld_gate, n, offset, heads, kv_heads, out);
  } else {
    const int threads = n * heads;
    launch_pdl(attention_generic_kernel, dim3((threads + 127) / 128), dim3(128), 0, s, q, kcache, vcache, gate_src, ld_gate, n, offset,
                                                                   heads, kv_heads, d, out);
  }
  DG_CUDA(cudaGetLastError());
}

void launch_final_norm(float* x, int M, int K, const float* gamma, float eps, DeviceStatus* st, cudaStream_t s) {
  if (M <= 0) return;
  launch_pdl(final_norm_kernel, dim3(M), dim3(256), 0, s, x, K, gamma, eps, st);
  DG_CUDA(cudaGetLastError());
}

void launch_head_norm(const float* hidden, int K, const int* rows, int n_rows, const float* w, const float* b,
                      float* out, cudaStream_t s) {
  if (n_rows <= 0) return;
  launch_pdl(head_norm_kernel, dim3(n_rows), dim3(256), 0, s, hidden, K, rows, w, b, out);
  DG_CUDA(cudaGetLastError());
}

void launch_head_dot(const float* q, const float* k, int n_keys, int dim, float scale, const float* bq,
                     const float* bk, float* logits, cudaStream_t s) {
  if (n_keys <= 0) return;
  launch_pdl(head_dot_kernel, dim3((n_keys + 3) / 4), dim3(128), 0, s, q, k, n_keys, dim, scale, bq, bk, logits);
  DG_CUDA(cudaGetLastError());
}

}  // namespace dg
