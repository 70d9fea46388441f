// Linear layers y[i] = W·x[i] (reference Ops::linear, src/ops.rs:116-126; CPU
// arithmetic src/cpu.rs:111-130) for the two regimes of the token loop:
//
//  * m ≤ 8 (decode, small chunks): a bandwidth-bound GEMV.  x sits in shared
//    memory, each warp streams one weight row (or a gate/amp row pair) with
//    16-byte non-allocating loads, so every weight byte is read from HBM once
//    and used for all m tokens.
//  * m > 8 (prefill chunks, m ≤ 256): a tiled FP32 SIMT GEMM, 64×64 output
//    tiles, 16-deep k slices double-buffered through registers.
//
// Both take the same fused epilogues (common.cuh: Epi): plain store, residual
// add (the block's x += h, src/model.rs:546-558) and the MLP's gate/amp pairing
// with silu (src/model.rs:552-555), so no separate add/columns/silu launches.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

constexpr int GEMV_WARPS = 8;

template <int M, int EPI>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
    k_gemv(const float* __restrict__ W, int rows, int cols, const float* __restrict__ x, int ldx, int m,
           float* y, int ldy, const float* res, int ldres) {
  extern __shared__ float4 xs4[];  // [M][cols / 4]
  const int c4 = cols >> 2;
  for (int t = threadIdx.x; t < M * c4; t += blockDim.x) {
    int i = t / c4, c = t - i * c4;
    xs4[t] = i < m ? reinterpret_cast<const float4*>(x + (size_t)i * ldx)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int out_rows = EPI == EPI_SILU ? rows / 2 : rows;
  const int r = blockIdx.x * GEMV_WARPS + warp;
  if (r >= out_rows) return;
  const float4* w0 = reinterpret_cast<const float4*>(W + (size_t)r * cols);
  const float4* w1 = reinterpret_cast<const float4*>(W + (size_t)(r + out_rows) * cols);
  float a0[M], a1[M];
#pragma unroll
  for (int i = 0; i < M; i++) a0[i] = a1[i] = 0.0f;
#pragma unroll 4
  for (int c = lane; c < c4; c += 32) {
    float4 wv = ld_stream(w0 + c);
    float4 wu = EPI == EPI_SILU ? ld_stream(w1 + c) : wv;
#pragma unroll
    for (int i = 0; i < M; i++) {
      float4 xv = xs4[i * c4 + c];
      a0[i] = dot4(wv, xv, a0[i]);
      if (EPI == EPI_SILU) a1[i] = dot4(wu, xv, a1[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < M; i++) {
    a0[i] = warp_sum(a0[i]);
    if (EPI == EPI_SILU) a1[i] = warp_sum(a1[i]);
  }
  if (lane < M && lane < m) {
    // Each of the first m lanes writes one token's output (registers indexed
    // with a compile-time loop to stay out of local memory).
#pragma unroll
    for (int i = 0; i < M; i++) {
      if (i == lane) {
        float v = a0[i];
        if (EPI == EPI_ADD) v = res[(size_t)i * ldres + r] + v;
        if (EPI == EPI_SILU) v = silu_mul(a0[i], a1[i]);
        y[(size_t)i * ldy + r] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// GEMV, m ≤ 8, by row blocks, for narrow outputs (the 768-wide o, down and
// inject projections, the decay): 32 outputs per CTA, 4 per warp (with
// EPI_SILU their gate and amp rows), so x is staged in shared memory once per
// 32 outputs and a warp keeps 4 (or 8) rows of 16-byte loads in flight.  K is
// split so that about one CTA per SM streams weights: each slice
// writes its partial sums, and the last CTA of a row block to finish (counted
// on that block's counter, which it puts back to zero) adds the slices in
// slice order and applies the epilogue.
// ---------------------------------------------------------------------------

constexpr int GR_RPW = 4, GR_ROWS = 8 * GR_RPW;

template <int M, int EPI>
__global__ void __launch_bounds__(256)
    k_gemv_rows(const float* __restrict__ W, int rows, int cols, const float* __restrict__ x, int ldx, int m,
                float* y, int ldy, const float* res, int ldres, int kper, float* __restrict__ part,
                unsigned* __restrict__ cnt) {
  extern __shared__ float4 xs4[];  // [M][kper / 4]
  const int out_rows = EPI == EPI_SILU ? rows / 2 : rows;
  const int s = blockIdx.y, k0 = s * kper, c4 = min(kper, cols - k0) >> 2, kp4 = kper >> 2;
  for (int t = threadIdx.x; t < M * c4; t += blockDim.x) {
    const int i = t / c4, c = t - i * c4;
    xs4[i * kp4 + c] = i < m ? reinterpret_cast<const float4*>(x + (size_t)i * ldx + k0)[c]
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = blockIdx.x * GR_ROWS + warp * GR_RPW;
  const float4* w0[GR_RPW];
  const float4* w1[GR_RPW];
#pragma unroll
  for (int j = 0; j < GR_RPW; j++) {
    const int o = min(o0 + j, out_rows - 1);  // rows past the end load a valid row; their sums are dropped
    w0[j] = reinterpret_cast<const float4*>(W + (size_t)o * cols + k0);
    w1[j] = reinterpret_cast<const float4*>(W + (size_t)(EPI == EPI_SILU ? o + out_rows : o) * cols + k0);
  }
  float a0[GR_RPW][M], a1[GR_RPW][M];
#pragma unroll
  for (int j = 0; j < GR_RPW; j++)
#pragma unroll
    for (int i = 0; i < M; i++) a0[j][i] = a1[j][i] = 0.0f;
#pragma unroll 2
  for (int c = lane; c < c4; c += 32) {
    float4 wv[GR_RPW], wu[GR_RPW];
#pragma unroll
    for (int j = 0; j < GR_RPW; j++) {
      wv[j] = ld_stream(w0[j] + c);
      if (EPI == EPI_SILU) wu[j] = ld_stream(w1[j] + c);
    }
#pragma unroll
    for (int i = 0; i < M; i++) {
      const float4 xv = xs4[i * kp4 + c];
#pragma unroll
      for (int j = 0; j < GR_RPW; j++) {
        a0[j][i] = dot4(wv[j], xv, a0[j][i]);
        if (EPI == EPI_SILU) a1[j][i] = dot4(wu[j], xv, a1[j][i]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < GR_RPW; j++)
#pragma unroll
    for (int i = 0; i < M; i++) {
      a0[j][i] = warp_sum(a0[j][i]);
      if (EPI == EPI_SILU) a1[j][i] = warp_sum(a1[j][i]);
    }
  const bool split = gridDim.y > 1;
  const size_t prow = (size_t)out_rows * (EPI == EPI_SILU ? 2 : 1);  // a slice's partial row per token
  // Lane j·M + i holds output o0 + j of token i (compile-time register selection).
#pragma unroll
  for (int j = 0; j < GR_RPW; j++)
#pragma unroll
    for (int i = 0; i < M; i++) {
      const int o = o0 + j;
      if (lane != j * M + i || i >= m || o >= out_rows) continue;
      if (split) {
        float* p = part + ((size_t)s * M + i) * prow;
        p[o] = a0[j][i];
        if (EPI == EPI_SILU) p[out_rows + o] = a1[j][i];
      } else {
        float v = a0[j][i];
        if (EPI == EPI_ADD) v = res[(size_t)i * ldres + o] + v;
        if (EPI == EPI_SILU) v = silu_mul(a0[j][i], a1[j][i]);
        y[(size_t)i * ldy + o] = v;
      }
    }
  if (!split) return;
  __shared__ int last;
  __threadfence();  // this slice's partials, before its count
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* c = cnt + blockIdx.x;
    last = atomicAdd(c, 1u) == gridDim.y - 1;
    if (last) *c = 0;  // every slice has counted
  }
  __syncthreads();
  if (!last) return;
  __threadfence();  // the other slices' partials
  const int i = threadIdx.x / GR_ROWS, o = blockIdx.x * GR_ROWS + threadIdx.x % GR_ROWS;
  if (i >= m || o >= out_rows) return;
  const float* p0 = part + (size_t)i * prow + o;
  const size_t sstride = (size_t)M * prow;
  float g = 0.0f, u = 0.0f;
  for (int s0 = 0; s0 < (int)gridDim.y; s0 += 4) {  // four slices' loads in flight, added in slice order
    float gv[4], uv[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int s2 = s0 + q < (int)gridDim.y ? s0 + q : s0;
      gv[q] = __ldcg(p0 + s2 * sstride);
      uv[q] = EPI == EPI_SILU ? __ldcg(p0 + s2 * sstride + out_rows) : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (s0 + q < (int)gridDim.y) g += gv[q], u += uv[q];
  }
  float v = g;
  if (EPI == EPI_ADD) v = res[(size_t)i * ldres + o] + v;
  if (EPI == EPI_SILU) v = silu_mul(g, u);
  y[(size_t)i * ldy + o] = v;
}

// K per slice (multiple of 128 columns, at least 256) and the slice count for
// the row-block GEMV: about one CTA per SM over all row blocks.
void gemv_plan(const LinearArgs& a, int* kper, int* slices) {
  const int out_rows = a.epi == EPI_SILU ? a.rows / 2 : a.rows;
  const int blocks = (out_rows + GR_ROWS - 1) / GR_ROWS;
  int want = std::max(1, 148 / blocks);
  want = std::min(want, std::max(1, a.cols / 256));
  int per = (a.cols + want - 1) / want;
  per = (per + 127) / 128 * 128;
  *kper = std::min(per, a.cols);
  *slices = (a.cols + *kper - 1) / *kper;
}

// ---------------------------------------------------------------------------
// GEMM, m > 8.  Output tile 64 tokens × 64 outputs, 256 threads, 4×4 each.
// With EPI_SILU a tile covers 32 output pairs: weight rows [32 gate | 32 amp].
// ---------------------------------------------------------------------------

constexpr int TM = 64, TN = 64, TK = 16, PAD = 4;

template <int EPI>
__global__ void __launch_bounds__(256)
    k_gemm(const float* __restrict__ W, int rows, int cols, const float* __restrict__ X, int ldx, int m,
           float* Y, int ldy, const float* res, int ldres) {
  __shared__ __align__(16) float As[2][TK][TM + PAD];
  __shared__ __align__(16) float Bs[2][TK][TN + PAD];
  const int tid = threadIdx.x;
  const int out_rows = EPI == EPI_SILU ? rows / 2 : rows;
  const int i0 = blockIdx.y * TM;
  // Loader mapping: one float4 of A and one of B per thread per k slice.
  const int lrow = tid >> 2, lk = (tid & 3) * 4;
  const int a_row = i0 + lrow;
  int b_row;
  if (EPI == EPI_SILU) {
    int pair0 = blockIdx.x * (TN / 2);
    b_row = lrow < TN / 2 ? pair0 + lrow : out_rows + pair0 + (lrow - TN / 2);
    if ((lrow < TN / 2 ? pair0 + lrow : pair0 + lrow - TN / 2) >= out_rows) b_row = -1;
  } else {
    b_row = blockIdx.x * TN + lrow;
    if (b_row >= rows) b_row = -1;
  }
  const float* a_ptr = a_row < m ? X + (size_t)a_row * ldx : nullptr;
  const float* b_ptr = b_row >= 0 ? W + (size_t)b_row * cols : nullptr;

  auto load = [&](int k0, float4& av, float4& bv) {
    int k = k0 + lk;
    av = (a_ptr && k < cols) ? *reinterpret_cast<const float4*>(a_ptr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    bv = (b_ptr && k < cols) ? ld_stream(reinterpret_cast<const float4*>(b_ptr + k))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  auto stash = [&](int buf, float4 av, float4 bv) {
    As[buf][lk + 0][lrow] = av.x;
    As[buf][lk + 1][lrow] = av.y;
    As[buf][lk + 2][lrow] = av.z;
    As[buf][lk + 3][lrow] = av.w;
    Bs[buf][lk + 0][lrow] = bv.x;
    Bs[buf][lk + 1][lrow] = bv.y;
    Bs[buf][lk + 2][lrow] = bv.z;
    Bs[buf][lk + 3][lrow] = bv.w;
  };

  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) acc[a][b] = 0.0f;

  float4 av, bv;
  load(0, av, bv);
  stash(0, av, bv);
  __syncthreads();
  const int nk = (cols + TK - 1) / TK;
  for (int kt = 0; kt < nk; kt++) {
    const int buf = kt & 1;
    const bool more = kt + 1 < nk;
    if (more) load((kt + 1) * TK, av, bv);
#pragma unroll
    for (int k = 0; k < TK; k++) {
      float4 a = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      float b[4];
      if (EPI == EPI_SILU) {
        float2 g = *reinterpret_cast<const float2*>(&Bs[buf][k][tx * 2]);
        float2 u = *reinterpret_cast<const float2*>(&Bs[buf][k][TN / 2 + tx * 2]);
        b[0] = g.x, b[1] = g.y, b[2] = u.x, b[3] = u.y;
      } else {
        float4 t = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
        b[0] = t.x, b[1] = t.y, b[2] = t.z, b[3] = t.w;
      }
      float av4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int ii = 0; ii < 4; ii++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) acc[ii][jj] = fmaf(av4[ii], b[jj], acc[ii][jj]);
    }
    if (more) stash(buf ^ 1, av, bv);
    __syncthreads();
  }

#pragma unroll
  for (int ii = 0; ii < 4; ii++) {
    int i = i0 + ty * 4 + ii;
    if (i >= m) continue;
    float* yrow = Y + (size_t)i * ldy;
    if (EPI == EPI_SILU) {
#pragma unroll
      for (int jj = 0; jj < 2; jj++) {
        int j = blockIdx.x * (TN / 2) + tx * 2 + jj;
        if (j < out_rows) yrow[j] = silu_mul(acc[ii][jj], acc[ii][jj + 2]);
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        int j = blockIdx.x * TN + tx * 4 + jj;
        if (j < rows) {
          float v = acc[ii][jj];
          if (EPI == EPI_ADD) v = res[(size_t)i * ldres + j] + v;
          yrow[j] = v;
        }
      }
    }
  }
}

// Any-shape fallback for the op-level API (cols not a multiple of 4 or
// unaligned operands): one warp per output, scalar loads.
__global__ void k_linear_scalar(const float* __restrict__ W, int rows, int cols, const float* __restrict__ x,
                                int ldx, int m, float* y, int ldy) {
  size_t t = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (t >= (size_t)m * rows) return;
  int i = (int)(t / rows), r = (int)(t % rows);
  const float* wr = W + (size_t)r * cols;
  const float* xr = x + (size_t)i * ldx;
  float s = 0.0f;
  for (int c = lane; c < cols; c += 32) s = fmaf(wr[c], xr[c], s);
  s = warp_sum(s);
  if (lane == 0) y[(size_t)i * ldy + r] = s;
}

template <int M, int EPI>
void launch_gemv(const LinearArgs& a, cudaStream_t st) {
  int out_rows = EPI == EPI_SILU ? a.rows / 2 : a.rows;
  // Narrow outputs of 4 to 8 token rows split over K (measured: the
  // 768-wide o and down projections of an 8-row batch, 20.4 → 10–13 µs);
  // wide outputs, and one or two rows, stay on the one-row-per-warp kernel
  // below, which measured as fast or faster there.
  int kper = 0, slices = 0;
  if (a.cols % 128 == 0 && M >= 4) gemv_plan(a, &kper, &slices);
  const size_t need = slices > 1 ? (size_t)slices * M * out_rows * (EPI == EPI_SILU ? 2 : 1) * sizeof(float) : 0;
  if (slices > 1 && a.cnt && need <= a.ws_bytes && (out_rows + GR_ROWS - 1) / GR_ROWS <= kGemvCounters) {
    const size_t smem = (size_t)M * kper * sizeof(float);
    k_gemv_rows<M, EPI><<<dim3(cdiv(out_rows, GR_ROWS), slices), 256, smem, st>>>(
        a.w, a.rows, a.cols, a.x, a.ldx, a.m, a.y, a.ldy, a.res, a.ldres, kper, static_cast<float*>(a.ws), a.cnt);
    SLM_LAUNCHED("k_gemv_rows");
    return;
  }
  size_t smem = (size_t)M * a.cols * sizeof(float);
  k_gemv<M, EPI><<<cdiv(out_rows, GEMV_WARPS), GEMV_WARPS * 32, smem, st>>>(a.w, a.rows, a.cols, a.x, a.ldx, a.m,
                                                                           a.y, a.ldy, a.res, a.ldres);
  SLM_LAUNCHED("k_gemv");
}

template <int EPI>
void dispatch(const LinearArgs& a, cudaStream_t st) {
  if (a.m <= 1)
    launch_gemv<1, EPI>(a, st);
  else if (a.m <= 2)
    launch_gemv<2, EPI>(a, st);
  else if (a.m <= 4)
    launch_gemv<4, EPI>(a, st);
  else if (a.m <= 8)
    launch_gemv<8, EPI>(a, st);
  else {
    int out_rows = EPI == EPI_SILU ? a.rows / 2 : a.rows;
    int tn = EPI == EPI_SILU ? TN / 2 : TN;
    dim3 grid(cdiv(out_rows, tn), cdiv(a.m, TM));
    k_gemm<EPI><<<grid, 256, 0, st>>>(a.w, a.rows, a.cols, a.x, a.ldx, a.m, a.y, a.ldy, a.res, a.ldres);
    SLM_LAUNCHED("k_gemm");
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int M>
void prepare_m() {
  SLM_CUDA(cudaFuncSetAttribute(k_gemv<M, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  SLM_CUDA(cudaFuncSetAttribute(k_gemv<M, EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  SLM_CUDA(cudaFuncSetAttribute(k_gemv<M, EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  SLM_CUDA(cudaFuncSetAttribute(k_gemv_rows<M, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  SLM_CUDA(cudaFuncSetAttribute(k_gemv_rows<M, EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  SLM_CUDA(cudaFuncSetAttribute(k_gemv_rows<M, EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

}  // namespace

size_t gemv_workspace(const LinearArgs& a) {
  if (a.m < 3 || a.m > 8 || a.cols % 128 != 0 || a.rows == 0) return 0;
  int kper = 0, slices = 0;
  gemv_plan(a, &kper, &slices);
  const int M = a.m <= 1 ? 1 : a.m <= 2 ? 2 : a.m <= 4 ? 4 : 8;
  const size_t out_rows = a.epi == EPI_SILU ? a.rows / 2 : a.rows;
  return slices > 1 ? (size_t)slices * M * out_rows * (a.epi == EPI_SILU ? 2 : 1) * sizeof(float) : 0;
}

// Per device, before any launch or graph capture: opt the GEMV kernels into
// more than 48 KB of dynamic shared memory (x of up to 8 rows × 6400 floats).
void linear_prepare() {
  prepare_m<1>();
  prepare_m<2>();
  prepare_m<4>();
  prepare_m<8>();
  skinny_prepare();
}

void linear(const LinearArgs& a, cudaStream_t st) {
  if (a.m == 0 || a.rows == 0) return;
  bool vec = a.cols % 4 == 0 && a.ldx % 4 == 0 && aligned16(a.w) && aligned16(a.x) &&
             (size_t)8 * a.cols * sizeof(float) <= 200 * 1024;
  if (!vec) {
    SLM_REQUIRE(a.epi == EPI_STORE, "linear: fused epilogues need cols % 4 == 0 and aligned operands");
    size_t outs = (size_t)a.m * a.rows;
    k_linear_scalar<<<cdiv(outs, 8), 256, 0, st>>>(a.w, a.rows, a.cols, a.x, a.ldx, a.m, a.y, a.ldy);
    SLM_LAUNCHED("k_linear_scalar");
    return;
  }
  if (a.epi == EPI_SILU) SLM_REQUIRE(a.rows % 2 == 0, "linear: silu pairing needs an even row count");
  if (b3_linear_ok(a) && b3_linear_workspace(a) <= a.ws_bytes) {
    b3_linear(a, a.ws, st);
    return;
  }
  if (skinny_ok(a) && skinny_workspace(a) <= a.ws_bytes) {
    skinny_linear(a, a.ws, st);
    return;
  }
  if (a.m > 64 && tc_linear_ok(a)) {
    const size_t need = tc_linear_workspace(a);
    if (need <= a.ws_bytes) {
      tc_linear(a, a.ws, st);
      return;
    }
  }
  switch (a.epi) {
    case EPI_STORE: dispatch<EPI_STORE>(a, st); break;
    case EPI_ADD: dispatch<EPI_ADD>(a, st); break;
    case EPI_SILU: dispatch<EPI_SILU>(a, st); break;
    default: fail(SLM_ERR_INVALID, "linear: unknown epilogue");
  }
}

}  // namespace slm
