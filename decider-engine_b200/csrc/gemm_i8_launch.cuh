// Per-tile-width launchers of the tcgen05 INT8 projection.
#pragma once
#include "gemm_i8.cuh"
#include "launch.h"

namespace dg {

// Tensor maps of one launch: activations, weights, and (tensor-core LoRA
// path) LoRA-B rows and LoRA-A rows.
struct GemmMaps {
  const CUtensorMap* a;
  const CUtensorMap* b;
  const CUtensorMap* lb;
  const CUtensorMap* mid;
};

void launch_gemm_i8_bn128(const GemmMaps& m, const GemmArgs& args, int rank, int epi, bool exact, cudaStream_t s);
void launch_gemm_i8_bn64(const GemmMaps& m, const GemmArgs& args, int rank, int epi, bool exact, cudaStream_t s);

template <int BN, int R, int EPI, bool EXACT, bool DUMP>
void launch_gemm_kernel(const GemmMaps& m, const GemmArgs& args, cudaStream_t s) {
  auto kern = gemm_i8_g64_kernel<BN, R, EPI, EXACT, DUMP>;
  const int smem = GemmShape<BN>::smem_bytes(R);
  static std::atomic<uint64_t> configured{0};  // per instantiation
  once_per_device(configured, [&] { DG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)); });
  dim3 grid((args.M + 127) / 128, args.N / BN, args.splits > 1 ? args.splits : 1);
  launch_k(args.late_dep != 0 || pdl_enabled(), kern, dim3(grid), dim3(GemmShape<BN>::NUM_THREADS), smem, s, *m.a,
           *m.b, *m.lb, *m.mid, args);
  DG_CUDA(cudaGetLastError());
}

// The group-dot dump exists only for reference-order WRITE projections.
template <int BN, int R, int EPI, bool EXACT>
void launch_gemm_impl(const GemmMaps& m, const GemmArgs& args, cudaStream_t s) {
  if constexpr (EPI == kEpiWrite && EXACT) {
    if (args.dots) return launch_gemm_kernel<BN, R, EPI, EXACT, true>(m, args, s);
  } else {
    if (args.dots) throw CudaError("gemm_i8: group-dot dump needs the reference-order WRITE epilogue");
  }
  launch_gemm_kernel<BN, R, EPI, EXACT, false>(m, args, s);
}

}  // namespace dg
