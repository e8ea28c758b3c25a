// Dense INT8 tensor-core ceiling of this GPU, measured (a measurement aid with
// no counterpart in the reference): every SM runs one CTA whose elected
// thread issues back-to-back tcgen05.mma.kind::i8 of 128 x 256 x 32 from
// shared memory into two alternating TMEM accumulators. Nothing else runs,
// so the rate is the tensor pipe's own; the projection's roofline fraction
// is read against it next to twice the measured dense bf16 figure.
#include "launch.h"

namespace dg {

namespace {
constexpr int kPeakM = 128, kPeakN = 256;
constexpr int kPeakA = kPeakM * 128, kPeakB = kPeakN * 128;  // 128-byte K rows, 128-byte swizzle
// More dynamic shared memory than two CTAs fit in, so each SM runs one.
constexpr int kPeakSmem = 160 * 1024;
}  // namespace

__global__ void __launch_bounds__(128, 1) tc_peak_i8_kernel(int iters, DeviceStatus* st) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + kPeakA + kPeakB);
  uint32_t* holder = reinterpret_cast<uint32_t*>(done + 1);
  // Small operand values: the accumulators never approach the int32 range.
  for (int i = threadIdx.x; i < (kPeakA + kPeakB) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = 0x01010101u * uint32_t((i & 3) + 1);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_i8(kPeakM, kPeakN);
    const uint32_t a = smem_addr(smem), b = a + kPeakA;
    for (int it = 0; it < iters; ++it) {
      const uint32_t d = tmem + uint32_t((it & 1) * kPeakN);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_i8(d, smem_desc_sw128(a + kk * 32), smem_desc_sw128(b + kk * 32), idesc, kk > 0 ? 1u : 0u);
    }
    mma_commit(done);
    // Bounded (10 s): on expiry the status word records it and the CTA still
    // frees its TMEM below.
    mbar_wait_bounded(done, 0, st, 900, nullptr, 10000000000ull);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

double measure_i8_peak(int device, int iters, float* ms_out) {
  if (iters <= 0 || iters > (1 << 22)) throw CudaError("i8 peak: iterations out of range");
  DG_CUDA(cudaSetDevice(device));
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    DG_CUDA(cudaFuncSetAttribute(tc_peak_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem));
  });
  int sms = 0;
  DG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  cudaStream_t s = nullptr;
  DG_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  DeviceStatus* st = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms = 0.0f;
  DeviceStatus h{};
  cudaError_t err = cudaMallocAsync(reinterpret_cast<void**>(&st), sizeof(DeviceStatus), s);
  if (err == cudaSuccess) err = cudaMemsetAsync(st, 0, sizeof(DeviceStatus), s);
  if (err == cudaSuccess) err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  if (err == cudaSuccess) {
    // One short launch first (clocks up, code loaded), then the timed one.
    launch_k(false, tc_peak_i8_kernel, dim3(sms), dim3(128), kPeakSmem, s, std::max(1, iters / 8), st);
    err = cudaEventRecord(e0, s);
    if (err == cudaSuccess) launch_k(false, tc_peak_i8_kernel, dim3(sms), dim3(128), kPeakSmem, s, iters, st);
    if (err == cudaSuccess) err = cudaEventRecord(e1, s);
    if (err == cudaSuccess) err = cudaMemcpyAsync(&h, st, sizeof(h), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  }
  if (st) cudaFreeAsync(st, s);
  cudaStreamSynchronize(s);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  DG_CUDA(err);
  if (h.code) throw CudaError("i8 peak: device status " + std::to_string(h.code));
  if (ms_out) *ms_out = ms;
  const double ops = 2.0 * kPeakM * kPeakN * 32 * 4 * double(iters) * sms;
  return ops / (double(ms) * 1e-3) / 1e12;
}

}  // namespace dg
