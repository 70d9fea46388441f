// Prefill linears on the tensor cores: y = x·Wᵀ (+ residual) for m > 8 token
// rows, as CUTLASS sm100 "FastFP32" GEMMs: TMA loads fp32 tiles, a transform
// warp group splits each value into three bf16 parts, and tcgen05 MMAs
// accumulate the significant cross products in TMEM (fp32), which gives
// products close to fp32 accuracy at tensor-core rates.  The epilogue writes
// D = A·Bᵀ or D = A·Bᵀ + C (the block's residual, src/model.rs:546-558).
//
// Shapes as a GEMM: M = token rows (x, row-major, K contiguous), N = weight
// rows (W, row-major [N][K] = column-major K×N), K = cols; D row-major [M][N].
#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/epilogue/thread/linear_combination.h"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

using namespace cute;

using ElementA = float;
using ElementB = float;
using ElementC = float;
using ElementD = float;
using ElementAcc = float;
using LayoutA = cutlass::layout::RowMajor;     // x: [M][K]
using LayoutB = cutlass::layout::ColumnMajor;  // W: [N][K]
using LayoutC = cutlass::layout::RowMajor;     // residual / output: [M][N]
using LayoutD = cutlass::layout::RowMajor;
constexpr int kAlign = 4;  // 16 bytes of fp32

using ArchTag = cutlass::arch::Sm100;
using OpClass = cutlass::arch::OpClassTensorOp;
#ifndef SLM_TC_TILE_N
#define SLM_TC_TILE_N 64
#endif
#ifndef SLM_TC_TILE_K
#define SLM_TC_TILE_K 32
#endif
// 64 × 64 × 32 tiles: measured on prefill (4096 ids, R = 4) 134.8k tok/s against 131.0k with
// 128 × 64, 129.0k with 64 × 128, 130.7k with a K tile of 64, 122.6k with 64 × 32.
#ifndef SLM_TC_TILE_M
#define SLM_TC_TILE_M 64
#endif
using TileShape = Shape<Int<SLM_TC_TILE_M>, Int<SLM_TC_TILE_N>, Int<SLM_TC_TILE_K>>;
// The split A operand kept in shared memory (the "Smem" schedule) measured
// 4% faster on the prefill chunks than the TMEM-resident form.
#ifndef SLM_TC_SCHEDULE
#define SLM_TC_SCHEDULE cutlass::gemm::KernelTmaWarpSpecialized1SmFastFP32SmemSm100
#endif
using ClusterShape = Shape<_1, _1, _1>;

using CollectiveEpilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    ArchTag, OpClass, TileShape, ClusterShape, cutlass::epilogue::collective::EpilogueTileAuto, ElementAcc, ElementAcc,
    ElementC, LayoutC, kAlign, ElementD, LayoutD, kAlign, cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;

using CollectiveMainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    ArchTag, OpClass, ElementA, LayoutA, kAlign, ElementB, LayoutB, kAlign, ElementAcc, TileShape, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
        sizeof(typename CollectiveEpilogue::SharedStorage))>,
    SLM_TC_SCHEDULE>::CollectiveOp;

// Stream-K tile scheduling: the 768-wide outputs of a 256-token chunk make only
// 2 × 12 output tiles, so the K loop is shared out over the idle SMs (with the
// deterministic reduction of the partial tiles).
using GemmKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, CollectiveMainloop,
                                                        CollectiveEpilogue, cutlass::gemm::StreamKScheduler>;
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<GemmKernel>;

using StrideA = typename Gemm::GemmKernel::StrideA;
using StrideB = typename Gemm::GemmKernel::StrideB;
using StrideC = typename Gemm::GemmKernel::StrideC;
using StrideD = typename Gemm::GemmKernel::StrideD;

}  // namespace

bool tc_linear_ok(const LinearArgs& a) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return a.m > 8 && a.epi != EPI_SILU && a.cols % 4 == 0 && a.rows % 4 == 0 && a.ldx == a.cols &&
         a.ldy == a.rows && (a.epi != EPI_ADD || a.ldres == a.rows) && al(a.w) && al(a.x) && al(a.y) &&
         (a.epi != EPI_ADD || al(a.res));
}

size_t tc_linear_workspace(const LinearArgs& a) {
  typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {a.m, a.rows, a.cols, 1},
                                {a.x, cutlass::make_cute_packed_stride(StrideA{}, make_shape(a.m, a.cols, 1)), a.w,
                                 cutlass::make_cute_packed_stride(StrideB{}, make_shape(a.rows, a.cols, 1))},
                                {{1.0f, 0.0f},
                                 a.res,
                                 cutlass::make_cute_packed_stride(StrideC{}, make_shape(a.m, a.rows, 1)),
                                 a.y,
                                 cutlass::make_cute_packed_stride(StrideD{}, make_shape(a.m, a.rows, 1))}};
  return Gemm::get_workspace_size(args);
}

// Runs the GEMM; `workspace` holds tc_linear_workspace(a) bytes (may be null when 0).
void tc_linear(const LinearArgs& a, void* workspace, cudaStream_t st) {
  const float beta = a.epi == EPI_ADD ? 1.0f : 0.0f;
  const float* c = a.epi == EPI_ADD ? a.res : a.y;
  typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {a.m, a.rows, a.cols, 1},
                                {a.x, cutlass::make_cute_packed_stride(StrideA{}, make_shape(a.m, a.cols, 1)), a.w,
                                 cutlass::make_cute_packed_stride(StrideB{}, make_shape(a.rows, a.cols, 1))},
                                {{1.0f, beta},
                                 c,
                                 cutlass::make_cute_packed_stride(StrideC{}, make_shape(a.m, a.rows, 1)),
                                 a.y,
                                 cutlass::make_cute_packed_stride(StrideD{}, make_shape(a.m, a.rows, 1))}};
  Gemm gemm;
  cutlass::Status s = gemm.can_implement(args);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_INVALID, "tensor-core linear: shape not supported");
  s = gemm.initialize(args, workspace, st);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_CUDA, "tensor-core linear: initialize failed");
  s = gemm.run(st);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_CUDA, "tensor-core linear: launch failed");
  SLM_LAUNCHED("tc_linear");
}

}  // namespace slm
