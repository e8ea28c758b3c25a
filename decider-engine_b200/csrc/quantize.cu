// Weight quantisation on the device: Data::quantize (src/weights.rs:98-146)
// of an F32 [rows][width] tensor, in groups of 64 along the width.
//
// Per (row, group): mx = the largest |w| of the group, scale = 1 when mx is
// 0, else max(mx / bound, FLT_MIN) (bound 127 for 8 bits, 7 for 4 bits), and
// code = clamp(round(w / scale), -bound, bound), rounding half away from
// zero. The divisions are IEEE (__fdiv_rn) and roundf rounds like the
// reference's f32::round, so every scale and code equals the host's bit for
// bit; a maximum does not depend on the order it is taken in.
//
// Two passes, both coalesced: weight_scales_kernel (one warp per row and
// group: two values per lane, a shuffle maximum) writes the scales, then
// one thread per output byte writes the codes, reading its group's scale:
// 8 bits one byte per value; 4 bits two values per byte, value i of the
// flattened tensor in the low nibble of byte i / 2 when i is even and in the
// high nibble when odd, each as code + 8 (the reference's packing, which runs
// across row ends when the width is odd).
//
// The 8-bit form can write a fused projection's layout directly: row j goes
// to output row (j / rb) * rs + ro + j % rb, at q_row bytes per output row,
// and the scale of (row, group) to scales[out_row * s_row + group * s_group].
#include <cfloat>

#include "common.cuh"
#include "launch.h"

namespace dg {
namespace {

__device__ __forceinline__ size_t quant_out_row(long j, const QuantLayout& L) {
  return size_t(j / L.rb) * size_t(L.rs) + size_t(L.ro) + size_t(j % L.rb);
}

__global__ void __launch_bounds__(256) weight_scales_kernel(const float* __restrict__ w, long rows, int width,
                                                            float bound, float* __restrict__ scales, QuantLayout L) {
  const long warp = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = (width + 63) / 64;
  if (warp >= rows * groups) return;
  const long r = warp / groups;
  const int g = int(warp % groups), lo = g * 64, n = min(64, width - lo);
  const float* v = w + size_t(r) * width + lo;
  float mx = 0.0f;
  if (lane < n) mx = fabsf(v[lane]);
  if (lane + 32 < n) mx = fmaxf(mx, fabsf(v[lane + 32]));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) {
    const float scale = mx == 0.0f ? 1.0f : fmaxf(__fdiv_rn(mx, bound), FLT_MIN);
    scales[quant_out_row(r, L) * L.s_row + size_t(g) * L.s_group] = scale;
  }
}

__device__ __forceinline__ float quant_code(float v, float scale, float bound) {
  const float x = roundf(__fdiv_rn(v, scale));
  return fminf(fmaxf(x, -bound), bound);
}

__global__ void __launch_bounds__(256) weight_codes_i8_kernel(const float* __restrict__ w, long rows, int width,
                                                              const float* __restrict__ scales,
                                                              uint8_t* __restrict__ q, QuantLayout L) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * width) return;
  const long r = i / width;
  const int c = int(i % width);
  const size_t orow = quant_out_row(r, L);
  const float scale = scales[orow * L.s_row + size_t(c / 64) * L.s_group];
  q[orow * L.q_row + c] = uint8_t(int8_t(int(quant_code(w[i], scale, 127.0f))));
}

__global__ void __launch_bounds__(256) weight_codes_i4_kernel(const float* __restrict__ w, long el, int width,
                                                              const float* __restrict__ scales,
                                                              uint8_t* __restrict__ q) {
  const long b = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= (el + 1) / 2) return;
  const int groups = (width + 63) / 64;
  uint32_t out = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const long i = 2 * b + h;
    if (i < el) {
      const long r = i / width;
      const int c = int(i % width);
      const int code = int(quant_code(w[i], scales[size_t(r) * groups + c / 64], 7.0f));
      out |= uint32_t(uint8_t(code + 8)) << (4 * h);
    }
  }
  q[b] = uint8_t(out);
}

// The reference's reading of a quantised row (Data::row): q as f32 times its
// group's scale, one IEEE multiply (8 bits: the signed byte; 4 bits: the
// nibble minus 8).
__global__ void __launch_bounds__(256) weight_dequant_kernel(const uint8_t* __restrict__ q,
                                                             const float* __restrict__ scales, long el, int width,
                                                             int bits, float* __restrict__ out) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= el) return;
  const long r = i / width;
  const int c = int(i % width), groups = (width + 63) / 64;
  const float code = bits == 8 ? float(int8_t(q[i])) : float(int((q[i / 2] >> (4 * (i % 2))) & 15)) - 8.0f;
  out[i] = __fmul_rn(code, scales[size_t(r) * groups + c / 64]);
}

}  // namespace

void dequantize_weights_device(const uint8_t* q, const float* scales, size_t rows, size_t width, int bits,
                               float* out, cudaStream_t s) {
  if (width == 0 || width > size_t(INT32_MAX) || rows > size_t(INT32_MAX)) throw CudaError("dequantize: bad width");
  if (bits != 8 && bits != 4) throw CudaError("dequantize: bits must be 8 or 4");
  const long el = long(rows) * long(width);
  if (el == 0) return;
  weight_dequant_kernel<<<unsigned((el + 255) / 256), 256, 0, s>>>(q, scales, el, int(width), bits, out);
  DG_CUDA(cudaGetLastError());
}

QuantLayout quant_plain_layout(size_t rows, size_t width) {
  QuantLayout L;
  L.q_row = width;
  L.s_row = (width + 63) / 64;
  L.s_group = 1;
  L.rb = int(std::max<size_t>(rows, 1));
  L.rs = 0;
  L.ro = 0;
  return L;
}

void quantize_weights_device(const float* w, size_t rows, size_t width, int bits, uint8_t* q, float* scales,
                             const QuantLayout* layout, cudaStream_t s) {
  if (width == 0 || width > size_t(INT32_MAX) || rows > size_t(INT32_MAX))
    throw CudaError("quantize: bad width");
  if (bits != 8 && bits != 4) throw CudaError("quantize: bits must be 8 or 4");
  if (rows == 0) return;
  const QuantLayout L = layout ? *layout : quant_plain_layout(rows, width);
  if (L.rb <= 0) throw CudaError("quantize: bad row map");
  if (bits == 4 && layout) throw CudaError("quantize: 4-bit values are written in the plain layout only");
  const long r = long(rows), wd = long(width), groups = (wd + 63) / 64;
  const long warps = r * groups;
  weight_scales_kernel<<<unsigned((warps * 32 + 255) / 256), 256, 0, s>>>(w, r, int(wd), bits == 8 ? 127.0f : 7.0f,
                                                                          scales, L);
  DG_CUDA(cudaGetLastError());
  if (bits == 8) {
    weight_codes_i8_kernel<<<unsigned((r * wd + 255) / 256), 256, 0, s>>>(w, r, int(wd), scales, q, L);
  } else {
    const long bytes = (r * wd + 1) / 2;
    weight_codes_i4_kernel<<<unsigned((bytes + 255) / 256), 256, 0, s>>>(w, r * wd, int(wd), scales, q);
  }
  DG_CUDA(cudaGetLastError());
}

}  // namespace dg
