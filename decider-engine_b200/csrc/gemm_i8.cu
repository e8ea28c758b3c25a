// Tensor maps, tile-width choice and launch of the tcgen05 INT8 projection.
// The kernel instantiations live in gemm_i8_bn128.cu and gemm_i8_bn64.cu.
#include <cstdlib>
#include <mutex>

#include "gemm_i8_launch.cuh"

namespace dg {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) throw CudaError("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Row-major int8 matrix [outer][inner] (inner contiguous), 128-byte swizzled boxes.
void make_tmap_i8_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                     uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || inner % 16)
    throw CudaError("TMA operand must be 16-byte aligned with a 16-byte multiple row stride");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}

// Row-major FP32 matrix [rows][ld] (ld >= cols), boxes of box_rows rows x 32
// columns (128 bytes, the swizzle span), 128-byte swizzled.
static void make_tmap_f32_rows(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                               uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * 4) % 16 || cols < 32)
    throw CudaError("TMA operand must be 16-byte aligned with a 16-byte multiple row stride");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {32, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                           elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}

void make_weight_maps(WeightMaps* maps, const void* wq, int k, int n, const float* lora_b, int rank) {
  make_tmap_i8_2d(&maps->bn128, wq, uint64_t(k), uint64_t(n), 128, 128);
  make_tmap_i8_2d(&maps->bn64, wq, uint64_t(k), uint64_t(n), 128, 64);
  maps->has_lb = lora_b != nullptr && rank == 32;
  if (maps->has_lb) make_tmap_f32_rows(&maps->lb, lora_b, 32, uint64_t(n), 32, 16);
}

// Cost model: a CTA's time grows with its tile width plus a fixed share
// (pipeline fill, activation tiles, epilogue set-up) worth about 64 columns;
// the grid takes ceil(ctas / 148) waves. SwiGLU pairs 16 gate with 16 up
// columns per 32, which the epilogue finishes in 128-column tiles only.
// DG_GEMM_TILE_N (64 or 128) forces the width where the shape allows it, for
// tuning on new parts.
int gemm_i8_choose_bn(int M, int N, int epi) {
  if (const char* f = std::getenv("DG_GEMM_TILE_N")) {
    const int bn = std::atoi(f);
    if ((bn == 64 || bn == 128) && N % bn == 0 && !(epi == kEpiSwiGlu && bn == 64)) return bn;
  }
  const int mt = (M + 127) / 128;
  int best = 128;
  long best_cost = -1;
  for (int bn : {128, 64}) {
    if (N % bn || (epi == kEpiSwiGlu && bn == 64)) continue;
    const long ctas = long(mt) * (N / bn), waves = (ctas + 147) / 148;
    const long cost = waves * (bn + 64);
    if (best_cost < 0 || cost < best_cost) best = bn, best_cost = cost;
  }
  return best;
}

// Split-K for grids of less than one wave (few token rows): FMA mode only
// (reference order sums the groups strictly in order), with a workspace, no
// group-dot dump. The largest split of 2-4 that divides the K stages, keeps
// at least four stages per split and the grid within one wave of 148 SMs.
int gemm_i8_choose_splits(const GemmArgs& args, int bn, bool exact) {
  if (exact || !args.split_ws || !args.split_cnt || args.dots) return 1;
  const int tiles = ((args.M + 127) / 128) * (args.N / bn), ks = args.K / 128;
  if (tiles > kGemmSplitTiles) return 1;
  for (int sp = 4; sp >= 2; --sp)
    if (ks % sp == 0 && ks / sp >= 4 && tiles * sp <= 148 &&
        size_t(sp) * size_t(args.M) * size_t(args.N) <= args.split_ws_floats)
      return sp;
  return 1;
}

void launch_gemm_i8(const CUtensorMap& a, const WeightMaps& w, const GemmArgs& args, int rank, int epi,
                    bool exact, cudaStream_t s) {
  if (args.M <= 0) return;
  if (args.N % 256 || args.K % 128 || args.K <= 0)
    throw CudaError("gemm_i8: N must be a multiple of 256 and K a positive multiple of 128");
  if (args.ldxs % 128 || args.ldxs < ((args.M + 127) / 128) * 128)
    throw CudaError("gemm_i8: activation-scale stride must cover whole 128-row tiles");
  if (rank != 0 && rank != 32) throw CudaError("gemm_i8: LoRA rank must be 0 or 32");
  if (rank && (args.ld_mid % 4 || !args.lora_mid || !args.lora_b || !args.chunk_pid))
    throw CudaError("gemm_i8: bad LoRA operands");
  if (epi == kEpiSwiGlu ? (args.ldo % 4) : (args.ldo % 4 || args.ldo < args.N))
    throw CudaError("gemm_i8: output stride must be a multiple of 4 covering the tile");
  const int bn = gemm_i8_choose_bn(args.M, args.N, epi);
  // The tensor-core LoRA path (fast mode, rank 32, 128-column tiles) reads the
  // LoRA rows through tensor maps.
  CUtensorMap none{}, mid{};
  const CUtensorMap* lb = &none;
  const CUtensorMap* mp = &none;
  if (rank == 32 && !exact && bn == 128) {
    if (!w.has_lb) throw CudaError("gemm_i8: the LoRA-B tensor map is missing");
    if (args.ld_mid < 32) throw CudaError("gemm_i8: LoRA-A rows narrower than one part");
    make_tmap_f32_rows(&mid, args.lora_mid, uint64_t(args.ld_mid), uint64_t(args.M), uint64_t(args.ld_mid), 128);
    lb = &w.lb;
    mp = &mid;
  }
  const GemmMaps m{&a, bn == 64 ? &w.bn64 : &w.bn128, lb, mp};
  GemmArgs g = args;
  g.splits = gemm_i8_choose_splits(g, bn, exact);
  if (bn == 64)
    launch_gemm_i8_bn64(m, g, rank, epi, exact, s);
  else
    launch_gemm_i8_bn128(m, g, rank, epi, exact, s);
}

}  // namespace dg
