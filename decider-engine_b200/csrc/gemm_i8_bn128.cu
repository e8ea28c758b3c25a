// Instantiations of the tcgen05 INT8 projection with 128-column tiles.
#include "gemm_i8_launch.cuh"

namespace dg {

void launch_gemm_i8_bn128(const GemmMaps& m, const GemmArgs& args, int rank, int epi, bool exact, cudaStream_t s) {
#define DG_GEMM_CASE(R_, E_, X_) \
  if (rank == R_ && epi == E_ && exact == X_) return launch_gemm_impl<128, R_, E_, X_>(m, args, s);
  DG_GEMM_CASE(32, kEpiWrite, true) DG_GEMM_CASE(32, kEpiAdd, true)
  DG_GEMM_CASE(32, kEpiWrite, false) DG_GEMM_CASE(32, kEpiAdd, false)
  DG_GEMM_CASE(0, kEpiWrite, true) DG_GEMM_CASE(0, kEpiWrite, false)
  DG_GEMM_CASE(32, kEpiSwiGlu, true) DG_GEMM_CASE(32, kEpiSwiGlu, false)
#undef DG_GEMM_CASE
  throw CudaError("gemm_i8: unsupported rank/epilogue combination for this tile width");
}

}  // namespace dg
