// Shared device helpers for the decider GPU library (sm_100a only).
//
// Compiled with -fmad=false: a*b+c rounds twice unless a kernel asks for a
// fused multiply-add explicitly (fmaf / __fmaf_rn), so the reference-order
// paths reproduce the CPU engine's FP32 rounding.
#pragma once
#include <cfloat>

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "decider GPU kernels target sm_100a only"
#endif

namespace dg {

// ---------------------------------------------------------------- status word
// Device-side failures never trap: kernels record a code in a status word the
// host reads after each forward pass.
enum StatusCode : uint32_t {
  kOk = 0,
  kNonFinite = 1,      // non-finite activation met while quantizing or at the end
  kWaitTimeout = 2,    // a bounded mbarrier wait expired (pipeline stalled)
  kBadToken = 3,       // token id outside the vocabulary
};

struct DeviceStatus {
  uint32_t code;      // first error code (atomicCAS from 0)
  uint32_t where;     // kernel-specific location of the failure
  uint32_t nonfinite; // count of non-finite detections
  uint32_t pad;
};

__device__ __forceinline__ void report(DeviceStatus* st, uint32_t code, uint32_t where) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0u, code) == 0u) st->where = where;
  if (code == kNonFinite) atomicAdd(&st->nonfinite, 1u);
}

// Epilogue::store variants, src/tensor.rs:86-100.
enum EpiKind { kEpiWrite = 0, kEpiAdd = 1, kEpiSwiGlu = 2 };

// ---------------------------------------------------------------- host errors
struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
#define DG_CUDA(expr)                                                                   \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess)                                                              \
      throw ::dg::CudaError(std::string(#expr) + ": " + cudaGetErrorString(_e));        \
  } while (0)

// Runs `configure` once per device for one call site: kernel attributes such
// as the dynamic shared-memory limit belong to the device's context, so each
// device a process launches on needs its own call. `done` is the call site's
// bit set of configured device ordinals (0-63).
template <class F>
inline void once_per_device(std::atomic<uint64_t>& done, F&& configure) {
  int d = 0;
  DG_CUDA(cudaGetDevice(&d));
  const uint64_t bit = uint64_t(1) << (d & 63);
  if (done.load(std::memory_order_acquire) & bit) return;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (done.load(std::memory_order_relaxed) & bit) return;
  configure();
  done.fetch_or(bit, std::memory_order_release);
}

// Count of kernel launches issued by this library (host side), reported by
// the C ABI so callers can see that device code ran.
uint64_t launch_count();
void note_launches(uint64_t n);
void note_launch();

// Programmatic dependent launch. Every kernel is launched with programmatic
// stream serialization (launch_pdl), so its CTAs may start while the previous
// kernel in the stream is still finishing: each kernel calls griddep_wait()
// before its first global access that can depend on earlier kernels (reads
// of their outputs, or writes to buffers they may still read); set-up that
// touches only shared memory, TMEM or read-only weights may come first.
// griddep_launch() then lets the next kernel's CTAs be scheduled.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
bool pdl_enabled();  // DG_PDL=1 sets the attribute (default: plain stream order)
// launch_k(pdl, ...): the attribute chosen per launch; launch_pdl: by DG_PDL.
template <typename... KArgs, typename... Args>
void launch_k(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DG_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  note_launch();  // every kernel of the library goes through here
}
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  launch_k(pdl_enabled(), kernel, grid, block, smem, s, std::forward<Args>(args)...);
}


// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (after recording
// kWaitTimeout) once `budget_ns` of global time has passed, so a stalled
// pipeline ends the kernel instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, DeviceStatus* st,
                                                  uint32_t where, volatile int* abort_flag,
                                                  uint64_t budget_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (abort_flag && *abort_flag) return false;
      if (global_timer_ns() - t0 > budget_ns) {
        report(st, kWaitTimeout, where);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// TMA: 2-D tiled load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, FP32 operands read as TF32, FP32 accumulate.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA, tensor core) before a barrier hands them over.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Arrive on `bar` once all previously issued tcgen05 MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// TMEM -> registers, 32 lanes x 16 columns of 32-bit data (thread t gets lane
// base + t), completed inside the statement: the load and its
// tcgen05.wait::ld form one asm block, so the destination registers exist
// for the compiler only once the asynchronous load has landed, and it can
// never spill or copy them while the load is in flight.
__device__ __forceinline__ void tmem_ld16_sync(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// Two such loads in flight together (one wait).
__device__ __forceinline__ void tmem_ld16x2_sync(uint32_t a0, uint32_t a1, uint32_t (&r0)[16], uint32_t (&r1)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r0[0]), "=r"(r0[1]), "=r"(r0[2]), "=r"(r0[3]), "=r"(r0[4]), "=r"(r0[5]), "=r"(r0[6]), "=r"(r0[7]), "=r"(r0[8]), "=r"(r0[9]), "=r"(r0[10]), "=r"(r0[11]), "=r"(r0[12]), "=r"(r0[13]), "=r"(r0[14]), "=r"(r0[15]),
        "=r"(r1[0]), "=r"(r1[1]), "=r"(r1[2]), "=r"(r1[3]), "=r"(r1[4]), "=r"(r1[5]), "=r"(r1[6]), "=r"(r1[7]), "=r"(r1[8]), "=r"(r1[9]), "=r"(r1[10]), "=r"(r1[11]), "=r"(r1[12]), "=r"(r1[13]), "=r"(r1[14]), "=r"(r1[15])
      : "r"(a0), "r"(a1)
      : "memory");
}
// 32 lanes x 16 columns, every word set to v.
__device__ __forceinline__ void tmem_fill_32x32b_x16(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 bytes, 8-row
// groups 1024 bytes apart. `addr` is the byte address of the operand start.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFF) >> 4);       // start address, bits [0,14)
  d |= uint64_t(1) << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;             // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                     // descriptor version for tcgen05
  d |= uint64_t(2) << 61;                     // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: signed A and B, S32 accumulator,
// both operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format S32
         | (1u << 7)          // A signed 8-bit
         | (1u << 10)         // B signed 8-bit
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}
// Instruction descriptor for kind::tf32: TF32 A and B, F32 accumulator,
// both operands K-major, M x N tile (M = 128: N % 16 == 0, 16 <= N <= 256).
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n) {
  return (1u << 4)            // D format F32
         | (2u << 7)          // A TF32
         | (2u << 10)         // B TF32
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------- packed f32x2
// Two FP32 lanes per instruction. The explicit .rn rounding keeps mul and add
// separate (never contracted into a fused multiply-add), lane by lane IEEE.
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "add.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 x, y, w, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 w, {%6, %7};\n\t"
      "fma.rn.f32x2 z, x, y, w;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

// Group-64 quantisation of the four values a lane holds; the 16 lanes of a
// half-warp hold one 64-wide group (same formula as quantize_group_warp).
__device__ __forceinline__ void quantize_vec4_halfwarp(float4 v, int8_t* q_out, float* scale_out, bool leader,
                                                       bool* bad) {
  float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  *bad |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
  const float scale = mx == 0.0f ? 1.0f : fmaxf(mx / 127.0f, FLT_MIN);
  char4 q;
  q.x = int8_t(fminf(fmaxf(roundf(v.x / scale), -127.0f), 127.0f));
  q.y = int8_t(fminf(fmaxf(roundf(v.y / scale), -127.0f), 127.0f));
  q.z = int8_t(fminf(fmaxf(roundf(v.z / scale), -127.0f), 127.0f));
  q.w = int8_t(fminf(fmaxf(roundf(v.w / scale), -127.0f), 127.0f));
  *reinterpret_cast<char4*>(q_out) = q;
  if (leader) *scale_out = scale;
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
// Exact int32 -> float for |v| < 2^22 (every 64-product group dot qualifies).
__device__ __forceinline__ float i32_to_f32_small(int32_t v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

}  // namespace dg
