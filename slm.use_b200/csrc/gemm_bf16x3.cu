// Prefill linears (m > 64 token rows) as one bf16 tensor-core GEMM carrying
// fp32 accuracy: y = x·Wᵀ (+ residual), the reference's Ops::linear
// (src/ops.rs:118, src/cpu.rs:111-130).
//
// Every fp32 value v is split into three bf16 parts, v = v0 + v1 + v2 (each
// the bf16 rounding of what the previous parts leave), which together carry
// the 24-bit significand.  The product keeps the six part products whose
// weights are at least 2^-16 of the whole, Σ_{i+j≤2} x_i·w_jᵀ; the three
// dropped ones are ~2^-24 relative, fp32 rounding level.  Laid out along K,
//   A = [x0 | x1 | x2 | x0 | x1 | x0]   (m × 6K, split per call, bf16)
//   B = [w0 | w0 | w0 | w1 | w1 | w2]   (N × 6K, split once at model load)
// so one plain bf16 GEMM with fp32 accumulation computes the sum: a CUTLASS
// sm100 kernel (TMA loads, tcgen05.mma into TMEM, 64 × 64 tiles, persistent tile scheduler) whose epilogue
// adds the residual (β = 1) for the block's x += h.
#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/epilogue/thread/linear_combination.h"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

using namespace cute;

using ElementAB = cutlass::bfloat16_t;
using ElementC = float;
using ElementD = float;
using ElementAcc = float;
using LayoutA = cutlass::layout::RowMajor;     // A: [M][6K]
using LayoutB = cutlass::layout::ColumnMajor;  // B: [N][6K]
using LayoutC = cutlass::layout::RowMajor;     // residual / output: [M][N]
using LayoutD = cutlass::layout::RowMajor;
constexpr int kAlignAB = 8;  // 16 bytes of bf16
constexpr int kAlignCD = 4;  // 16 bytes of fp32

using ArchTag = cutlass::arch::Sm100;
using OpClass = cutlass::arch::OpClassTensorOp;
// 64 × 64 output tiles: a 256-token chunk's qkv projection makes 144 of them,
// about one per SM, so no K split is needed.  Measured on prefill (4096 ids,
// R = 4): 130.5k tok/s, against 127.6k with 128 × 64 tiles and stream-K
// (which was 4% faster than 128 × 128), 129.0k with 64 × 64 and stream-K,
// 126.9k with 64 × 128.
#ifndef SLM_B3_TILE_M
#define SLM_B3_TILE_M 64
#endif
#ifndef SLM_B3_TILE_N
#define SLM_B3_TILE_N 64
#endif
using TileShape = Shape<Int<SLM_B3_TILE_M>, Int<SLM_B3_TILE_N>, _64>;
using ClusterShape = Shape<_1, _1, _1>;  // no cluster: plain (non-multicast) TMA loads

using CollectiveEpilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    ArchTag, OpClass, TileShape, ClusterShape, cutlass::epilogue::collective::EpilogueTileAuto, ElementAcc, ElementAcc,
    ElementC, LayoutC, kAlignCD, ElementD, LayoutD, kAlignCD, cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;

using CollectiveMainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    ArchTag, OpClass, ElementAB, LayoutA, kAlignAB, ElementAB, LayoutB, kAlignAB, ElementAcc, TileShape, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
        sizeof(typename CollectiveEpilogue::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;

using GemmKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, CollectiveMainloop,
                                                        CollectiveEpilogue, void>;  // default persistent scheduler
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<GemmKernel>;

using StrideA = typename Gemm::GemmKernel::StrideA;
using StrideB = typename Gemm::GemmKernel::StrideB;
using StrideC = typename Gemm::GemmKernel::StrideC;
using StrideD = typename Gemm::GemmKernel::StrideD;

// v = p0 + p1 + p2, each the bf16 rounding (to nearest) of what is left.
__device__ __forceinline__ void split3(float v, __nv_bfloat16* p) {
  const __nv_bfloat16 a = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(a);
  const __nv_bfloat16 b = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(b);
  p[0] = a, p[1] = b, p[2] = __float2bfloat16_rn(r2);
}

// Weights: out[r] = [w0 | w0 | w0 | w1 | w1 | w2] (6·cols bf16 per row).
__global__ void k_split_w(const float* __restrict__ w, size_t rows, size_t cols, __nv_bfloat16* __restrict__ out) {
  for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < rows * cols; t += (size_t)gridDim.x * blockDim.x) {
    const size_t r = t / cols, c = t % cols;
    __nv_bfloat16 p[3];
    split3(w[t], p);
    __nv_bfloat16* o = out + r * 6 * cols + c;
    o[0] = p[0], o[cols] = p[0], o[2 * cols] = p[0], o[3 * cols] = p[1], o[4 * cols] = p[1], o[5 * cols] = p[2];
  }
}

// Activations: out[i] = [x0 | x1 | x2 | x0 | x1 | x0].
__global__ void k_split_x(const float* __restrict__ x, int ldx, size_t m, size_t cols,
                          __nv_bfloat16* __restrict__ out) {
  for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < m * cols; t += (size_t)gridDim.x * blockDim.x) {
    const size_t i = t / cols, c = t % cols;
    __nv_bfloat16 p[3];
    split3(x[i * ldx + c], p);
    __nv_bfloat16* o = out + i * 6 * cols + c;
    o[0] = p[0], o[cols] = p[1], o[2 * cols] = p[2], o[3 * cols] = p[0], o[4 * cols] = p[1], o[5 * cols] = p[0];
  }
}

// RMSNorm of each group (src/cpu.rs:187-207, as k_rms) that also writes the
// bf16x3 planes of its output, the A operand of the wide linears that read it.
__global__ void k_rms_split(float* __restrict__ y, __nv_bfloat16* __restrict__ planes, const float* __restrict__ x,
                            const float* __restrict__ w, size_t size, float eps) {
  __shared__ float red[32];
  const float* in = x + (size_t)blockIdx.x * size;
  float s = 0.0f;
  for (size_t e = threadIdx.x; e < size; e += blockDim.x) s = fmaf(in[e], in[e], s);
  s = block_sum(s, red);
  const float r = 1.0f / sqrtf(s / (float)size + eps);
  float* out = y + (size_t)blockIdx.x * size;
  __nv_bfloat16* o = planes + (size_t)blockIdx.x * 6 * size;
  for (size_t e = threadIdx.x; e < size; e += blockDim.x) {
    const float v = in[e] * r * w[e];
    out[e] = v;
    __nv_bfloat16 p[3];
    split3(v, p);
    o[e] = p[0], o[size + e] = p[1], o[2 * size + e] = p[2], o[3 * size + e] = p[0], o[4 * size + e] = p[1],
    o[5 * size + e] = p[0];
  }
}

typename Gemm::Arguments make_args(const LinearArgs& a, const void* aplanes) {
  const int K6 = 6 * a.cols;
  const float beta = a.epi == EPI_ADD ? 1.0f : 0.0f;
  const float* c = a.epi == EPI_ADD ? a.res : a.y;
  return typename Gemm::Arguments{
      cutlass::gemm::GemmUniversalMode::kGemm,
      {a.m, a.rows, K6, 1},
      {static_cast<const ElementAB*>(aplanes), cutlass::make_cute_packed_stride(StrideA{}, make_shape(a.m, K6, 1)),
       static_cast<const ElementAB*>(a.wplanes), cutlass::make_cute_packed_stride(StrideB{}, make_shape(a.rows, K6, 1))},
      {{1.0f, beta},
       c,
       cutlass::make_cute_packed_stride(StrideC{}, make_shape(a.m, a.rows, 1)),
       a.y,
       cutlass::make_cute_packed_stride(StrideD{}, make_shape(a.m, a.rows, 1))}};
}

}  // namespace

size_t b3_planes_bytes(size_t rows, size_t cols) { return rows * cols * 6 * sizeof(__nv_bfloat16); }

void b3_split_weights(const float* w, size_t rows, size_t cols, void* planes, cudaStream_t st) {
  const size_t n = rows * cols;
  const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 16);
  k_split_w<<<grid, 256, 0, st>>>(w, rows, cols, static_cast<__nv_bfloat16*>(planes));
  SLM_LAUNCHED("k_split_w");
}

#ifndef SLM_B3_MIN_ROWS
#define SLM_B3_MIN_ROWS 2048  // narrower outputs stay on the FastFP32 kernel
#endif
#ifndef SLM_B3_MIN_COLS
#define SLM_B3_MIN_COLS 1000000000  // deep inputs (the down projection) stay on FastFP32 unless set
#endif
#ifndef SLM_B3_MIN_M
#define SLM_B3_MIN_M 65  // fewer token rows go to the skinny SIMT kernel
#endif

bool b3_linear_ok(const LinearArgs& a) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return a.wplanes && a.m >= SLM_B3_MIN_M && (a.rows >= SLM_B3_MIN_ROWS || a.cols >= SLM_B3_MIN_COLS) &&
         a.epi != EPI_SILU && a.cols % 8 == 0 &&
         a.rows % 4 == 0 && a.ldy == a.rows &&
         (a.epi != EPI_ADD || a.ldres == a.rows) && al(a.wplanes) && al(a.y) && (a.epi != EPI_ADD || al(a.res));
}

// Workspace: the activation planes (m × 6K bf16, 256-byte aligned) then the
// GEMM's own workspace.
size_t b3_linear_workspace(const LinearArgs& a) {
  const size_t planes = ((size_t)a.m * 6 * a.cols * sizeof(__nv_bfloat16) + 255) / 256 * 256;
  return planes + Gemm::get_workspace_size(make_args(a, nullptr));
}

void b3_rms_split(float* y, void* planes, const float* x, const float* w, size_t groups, size_t size, float eps,
                  cudaStream_t st) {
  if (!groups) return;
  k_rms_split<<<(unsigned)groups, 256, 0, st>>>(y, static_cast<__nv_bfloat16*>(planes), x, w, size, eps);
  SLM_LAUNCHED("k_rms_split");
}

void b3_linear(const LinearArgs& a, void* ws, cudaStream_t st) {
  const size_t pb = ((size_t)a.m * 6 * a.cols * sizeof(__nv_bfloat16) + 255) / 256 * 256;
  const void* planes = a.xplanes;
  if (!planes) {  // split the activations here
    const size_t n = (size_t)a.m * a.cols;
    k_split_x<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(
        a.x, a.ldx, a.m, a.cols, static_cast<__nv_bfloat16*>(ws));
    SLM_LAUNCHED("k_split_x");
    planes = ws;
  }
  auto args = make_args(a, planes);
  Gemm gemm;
  cutlass::Status s = gemm.can_implement(args);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_INVALID, "bf16x3 linear: shape not supported");
  s = gemm.initialize(args, static_cast<char*>(ws) + pb, st);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_CUDA, "bf16x3 linear: initialize failed");
  s = gemm.run(st);
  if (s != cutlass::Status::kSuccess) fail(SLM_ERR_CUDA, "bf16x3 linear: launch failed");
  SLM_LAUNCHED("b3_linear");
}

}  // namespace slm
