// Linears with a few token rows (8 < m ≤ 64: a batched decode step of
// independent sessions, short prompt chunks) and the narrow outputs of full
// prefill chunks (m ≤ 256, tiled 64 tokens at a time): y[i] = W·x[i]
// (+ residual), the reference's Ops::linear (src/ops.rs:118,
// src/cpu.rs:111-130) in fp32.
//
// At these sizes the weights (one read per call) and the launch dominate,
// and a tensor-core tile pipeline sits mostly idle, so this is a SIMT kernel
// shaped for bandwidth and occupancy: a CTA owns 64 weight rows × all tokens
// (padded to 32 or 64) over one slice of K; slices split K so that about two
// CTAs per SM are busy.  K tiles of 32 of W and x flow through a 4-stage
// cp.async pipeline in rows padded to 36 floats; thread (tr, tt) accumulates
// rows tr + 16·j (j < 4) × tokens tt + 8·u (u < TT/8), so the 16 weight rows
// a warp reads at once sit in 8 different bank groups (two addresses per
// group: conflict-free for 16-byte loads) and its two token rows in two.
// With one slice the epilogue writes y directly.  Otherwise every slice
// writes its partial product to the workspace and k_skinny_reduce, spread
// over all SMs, sums the slices in slice order (deterministic) and adds the
// residual.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

constexpr int RT = 64;  // weight rows per CTA
constexpr int KT = 32;  // K per stage
constexpr int LD = KT + 4;
#ifndef SLM_SKINNY_STAGES
#define SLM_SKINNY_STAGES 4
#endif
constexpr int STAGES = SLM_SKINNY_STAGES;
#ifndef SLM_SKINNY_MAX_M
#define SLM_SKINNY_MAX_M 64  // token rows (above 64 in tiles of 64; 256-token chunks measured faster on FastFP32)
#endif
#ifndef SLM_SKINNY_K_MAX
#define SLM_SKINNY_K_MAX 768  // linears with K at most this take the kernel for whole 256-token chunks too
#endif

template <int TT>
constexpr size_t smem_bytes() {
  return (size_t)STAGES * (RT + TT) * LD * sizeof(float);
}

__device__ __forceinline__ void cp16z(void* dst, const void* src, bool ok) {
  unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// grid (ceil(rows/64), slices, ceil(m/TT)); 128 threads.  Thread t: rows
// r0 + t%16 + 16·j, tokens z·TT + t/16 + 8·u.
template <int TT, int EPI>
__global__ void __launch_bounds__(128)
    k_skinny(const float* __restrict__ w, int rows, int cols, const float* __restrict__ x, int ldx, int m, int kper,
             float* __restrict__ y, int ldy, const float* __restrict__ res, int ldres, float* __restrict__ part) {
  constexpr int TPT = TT / 8;
  extern __shared__ __align__(16) float smem[];
  float (*Ws)[RT][LD] = reinterpret_cast<float (*)[RT][LD]>(smem);
  float (*Xs)[TT][LD] = reinterpret_cast<float (*)[TT][LD]>(smem + (size_t)STAGES * RT * LD);
  const int t = threadIdx.x, tr = t % 16, tt = t / 16;
  const int r0 = blockIdx.x * RT, s = blockIdx.y, i0 = blockIdx.z * TT;
  const int k0 = s * kper, k1 = min(cols, k0 + kper);
  const int stages = (k1 - k0) / KT;

  auto load = [&](int st, int buf) {
    const int kb = k0 + st * KT;
    for (int e = t; e < RT * (KT / 4); e += 128) {
      const int r = e / (KT / 4), c = (e % (KT / 4)) * 4;
      const bool ok = r0 + r < rows;
      cp16z(&Ws[buf][r][c], w + (size_t)(ok ? r0 + r : 0) * cols + kb + c, ok);
    }
    for (int e = t; e < TT * (KT / 4); e += 128) {
      const int i = e / (KT / 4), c = (e % (KT / 4)) * 4;
      const bool ok = i0 + i < m;
      cp16z(&Xs[buf][i][c], x + (size_t)(ok ? i0 + i : 0) * ldx + kb + c, ok);
    }
  };

  float acc[4][TPT];
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int u = 0; u < TPT; u++) acc[j][u] = 0.0f;

  // Prologue: STAGES-1 stages in flight (empty groups keep the count uniform).
#pragma unroll
  for (int p = 0; p < STAGES - 1; p++) {
    if (p < stages) load(p, p);
    commit();
  }
  for (int st = 0; st < stages; st++) {
    wait_group<STAGES - 2>();  // stage st has landed
    __syncthreads();           // … for every thread; and stage st-1's buffer is free
    const int nx = st + STAGES - 1;
    if (nx < stages) load(nx, nx % STAGES);
    commit();
    const int buf = st % STAGES;
#pragma unroll
    for (int kk = 0; kk < KT; kk += 4) {
      float4 wv[4], xv[TPT];
#pragma unroll
      for (int j = 0; j < 4; j++) wv[j] = *reinterpret_cast<const float4*>(&Ws[buf][tr + 16 * j][kk]);
#pragma unroll
      for (int u = 0; u < TPT; u++) xv[u] = *reinterpret_cast<const float4*>(&Xs[buf][tt + 8 * u][kk]);
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int u = 0; u < TPT; u++) acc[j][u] = dot4(wv[j], xv[u], acc[j][u]);
    }
  }
  wait_group<0>();

  auto out = [&](int i, int r, float v) {
    if (EPI == EPI_ADD)
      y[(size_t)i * ldy + r] = res[(size_t)i * ldres + r] + v;
    else
      y[(size_t)i * ldy + r] = v;
  };
  if (!part) {
#pragma unroll
    for (int u = 0; u < TPT; u++) {
      const int i = i0 + tt + 8 * u;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = r0 + tr + 16 * j;
        if (i < m && r < rows) out(i, r, acc[j][u]);
      }
    }
    return;
  }
#pragma unroll
  for (int u = 0; u < TPT; u++) {
    const int i = i0 + tt + 8 * u;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = r0 + tr + 16 * j;
      if (i < m && r < rows) part[((size_t)s * m + i) * rows + r] = acc[j][u];
    }
  }
}

// y[i][r] = (res[i][r] +) Σ_s part[s][i][r], slices in order.  A thread
// takes four consecutive r (rows % 4 == 0) and loads eight slices at a time
// before adding them, so its L2 reads overlap; the adds keep slice order.
template <int EPI>
__global__ void k_skinny_reduce(const float* __restrict__ part, int slices, int m, int rows, float* __restrict__ y,
                                int ldy, const float* __restrict__ res, int ldres) {
  const size_t n4 = (size_t)m * rows / 4, plane = (size_t)m * rows;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += (size_t)gridDim.x * blockDim.x) {
    const size_t i = 4 * e / rows, r = 4 * e % rows;
    const float4* p = reinterpret_cast<const float4*>(part + i * rows + r);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < slices; s0 += 8) {
      float4 q[8];
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (s0 + u < slices) q[u] = __ldcg(p + (s0 + u) * plane / 4);
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (s0 + u < slices) v.x += q[u].x, v.y += q[u].y, v.z += q[u].z, v.w += q[u].w;
    }
    float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      float a = o[k];
      if (EPI == EPI_ADD) a = res[i * ldres + r + k] + a;
      y[i * ldy + r + k] = a;
    }
  }
}

// The same sums for any row count, one output per thread.
template <int EPI>
__global__ void k_skinny_reduce1(const float* __restrict__ part, int slices, int m, int rows, float* __restrict__ y,
                                 int ldy, const float* __restrict__ res, int ldres) {
  const size_t n = (size_t)m * rows;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const size_t i = e / rows, r = e % rows;
    float v = 0.0f;
    for (int s = 0; s < slices; s++) v += part[((size_t)s * m + i) * rows + r];
    if (EPI == EPI_ADD) v = res[i * ldres + r] + v;
    y[i * ldy + r] = v;
  }
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// K per slice (a multiple of KT) and the slice count.
void plan(const LinearArgs& a, int* kper, int* slices) {
  const int tiles = (a.rows + RT - 1) / RT * ((a.m + 63) / 64), kt = a.cols / KT;
  int want = (2 * sm_count() + tiles - 1) / tiles;
  want = std::max(1, std::min(want, kt));
  const int per = (kt + want - 1) / want;
  *kper = per * KT;
  *slices = (kt + per - 1) / per;
}

template <int TT, int EPI>
void launch(const LinearArgs& a, int kper, int slices, float* part, cudaStream_t st) {
  dim3 grid((a.rows + RT - 1) / RT, slices, (a.m + TT - 1) / TT);
  k_skinny<TT, EPI><<<grid, 128, smem_bytes<TT>(), st>>>(a.w, a.rows, a.cols, a.x, a.ldx, a.m, kper, a.y, a.ldy,
                                                          a.res, a.ldres, part);
  SLM_LAUNCHED("k_skinny");
}

template <int TT, int EPI>
void allow_smem() {
  SLM_CUDA(cudaFuncSetAttribute(k_skinny<TT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes<TT>()));
}

}  // namespace

void skinny_prepare() {
  allow_smem<32, EPI_STORE>();
  allow_smem<32, EPI_ADD>();
  allow_smem<64, EPI_STORE>();
  allow_smem<64, EPI_ADD>();
}

bool skinny_ok(const LinearArgs& a) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  // Outputs of at most 128 rows (the GLA decay) and short K (the o and inject
  // projections of d 768) take it for whole chunks too: a tensor-core GEMM
  // launch costs ~20-30 µs for little work there.
  const int max_m = a.rows <= 128 || a.cols <= SLM_SKINNY_K_MAX ? 256 : SLM_SKINNY_MAX_M;
  return a.m > 8 && a.m <= max_m && (a.epi == EPI_STORE || a.epi == EPI_ADD) && a.cols % KT == 0 &&
         a.ldx % 4 == 0 &&
         al(a.w) && al(a.x);
}

size_t skinny_workspace(const LinearArgs& a) {
  int kper = 0, slices = 0;
  plan(a, &kper, &slices);
  return slices > 1 ? (size_t)slices * a.m * a.rows * sizeof(float) : 0;
}

void skinny_linear(const LinearArgs& a, void* ws, cudaStream_t st) {
  int kper = 0, slices = 0;
  plan(a, &kper, &slices);
  float* part = slices > 1 ? static_cast<float*>(ws) : nullptr;
  const bool add = a.epi == EPI_ADD;
  if (a.m <= 32) {
    add ? launch<32, EPI_ADD>(a, kper, slices, part, st) : launch<32, EPI_STORE>(a, kper, slices, part, st);
  } else {
    add ? launch<64, EPI_ADD>(a, kper, slices, part, st) : launch<64, EPI_STORE>(a, kper, slices, part, st);
  }
  if (part) {
    const size_t n = (size_t)a.m * a.rows;
    if (a.rows % 4 == 0) {  // float4 of the workspace: rows and m·rows are multiples of 4
      const unsigned grid = (unsigned)std::min<size_t>((n / 4 + 255) / 256, (size_t)8 * sm_count());
      if (add)
        k_skinny_reduce<EPI_ADD><<<grid, 256, 0, st>>>(part, slices, a.m, a.rows, a.y, a.ldy, a.res, a.ldres);
      else
        k_skinny_reduce<EPI_STORE><<<grid, 256, 0, st>>>(part, slices, a.m, a.rows, a.y, a.ldy, a.res, a.ldres);
      SLM_LAUNCHED("k_skinny_reduce");
    } else {
      const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)8 * sm_count());
      if (add)
        k_skinny_reduce1<EPI_ADD><<<grid, 256, 0, st>>>(part, slices, a.m, a.rows, a.y, a.ldy, a.res, a.ldres);
      else
        k_skinny_reduce1<EPI_STORE><<<grid, 256, 0, st>>>(part, slices, a.m, a.rows, a.y, a.ldy, a.res, a.ldres);
      SLM_LAUNCHED("k_skinny_reduce1");
    }
  }
}

}  // namespace slm
