// Gated linear attention, the recurrent state of the L layers (reference
// Ops::gla, src/ops.rs:191-205; CPU arithmetic src/cpu.rs:284-329), fused with
// what follows it in the L mixer (src/model.rs:463-485): the per-head RMSNorm
// (head_norm) and the silu gate.
//
// Per head, for each token in order:
//   d = 1 / (1 + e^(decay + bias))       (= exp(-softplus(decay + bias)))
//   S[a][b] = d·S[a][b] + k[a]·v[b]
//   y[b] = Σ_a q[a]·S[a][b]
//   out[b] = silu(g[b]) · (y[b] · r · w[b]),  r = 1/sqrt(mean(y²) + eps)
//
// One CTA per head.  Columns of S are independent; each is split over RQ
// adjacent lanes that keep DH/RQ of its rows in registers for the whole call,
// so the state crosses HBM once per call.  Tokens are staged TC at a time in
// shared memory (q, k, v, the decay factor); the sequential walk over them
// needs no barrier, only two shuffles per token to sum a column's y.  The
// head_norm and gate of the staged tokens then run in parallel, one warp per
// token.
#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

template <int DH>
struct GlaShape {
  static constexpr int RQ = DH >= 128 ? 2 : 4;  // lanes per column
  static constexpr int R = DH / RQ;             // rows of S per lane
  static constexpr int T = DH * RQ;             // threads
  static constexpr int TC = DH >= 128 ? 16 : 32;  // tokens staged per round
};

template <int DH>
__global__ void __launch_bounds__(GlaShape<DH>::T)
    k_gla(float* __restrict__ S, const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
          const float* __restrict__ v, int ldv, const float* __restrict__ gt, int ldg, const float* __restrict__ dec,
          int lddec, const float* __restrict__ bias, const float* __restrict__ hnw, float eps, int m, int heads,
          float* __restrict__ out, int ldo, int fuse) {
  using Sh = GlaShape<DH>;
  constexpr int RQ = Sh::RQ, R = Sh::R, T = Sh::T, TC = Sh::TC;
  __shared__ float qs[TC][DH], ks[TC][DH], vs[TC][DH], ys[TC][DH], ds[TC];
  const int h = blockIdx.x, t = threadIdx.x;
  const int b = t / RQ, rq = t % RQ, a0 = rq * R;
  const int lane = t & 31, warp = t >> 5;
  float col[R];
  float* Sh_ = S + (size_t)h * DH * DH;
#pragma unroll
  for (int j = 0; j < R; j++) col[j] = Sh_[(size_t)(a0 + j) * DH + b];
  const float bh = bias[h];

  for (int c0 = 0; c0 < m; c0 += TC) {
    const int n = min(TC, m - c0);
    for (int e = t; e < n * DH; e += T) {
      const int i = e / DH, x = e % DH;
      const size_t row = (size_t)(c0 + i);
      qs[i][x] = q[row * ldq + (size_t)h * DH + x];
      ks[i][x] = k[row * ldk + (size_t)h * DH + x];
      vs[i][x] = v[row * ldv + (size_t)h * DH + x];
    }
    for (int i = t; i < n; i += T) ds[i] = 1.0f / (1.0f + expf(dec[(size_t)(c0 + i) * lddec + h] + bh));
    __syncthreads();
    for (int i = 0; i < n; i++) {
      const float d = ds[i], vb = vs[i][b];
      float y = 0.0f;
#pragma unroll
      for (int j = 0; j < R; j++) {
        const float s = d * col[j] + ks[i][a0 + j] * vb;
        col[j] = s;
        y = fmaf(qs[i][a0 + j], s, y);
      }
#pragma unroll
      for (int o = 1; o < RQ; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
      if (rq == 0) ys[i][b] = y;
    }
    __syncthreads();
    // head_norm + gate (or the raw y), one warp per staged token.
    for (int i = warp; i < n; i += T / 32) {
      const size_t row = (size_t)(c0 + i);
      float ss = 0.0f;
      for (int x = lane; x < DH; x += 32) ss = fmaf(ys[i][x], ys[i][x], ss);
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss / (float)DH + eps);
      for (int x = lane; x < DH; x += 32) {
        const float y = ys[i][x];
        out[row * ldo + (size_t)h * DH + x] =
            fuse ? silu_mul(gt[row * ldg + (size_t)h * DH + x], y * r * hnw[x]) : y;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < R; j++) Sh_[(size_t)(a0 + j) * DH + b] = col[j];
}

template <int DH>
void launch(const GlaArgs& g, cudaStream_t st) {
  k_gla<DH><<<g.heads, GlaShape<DH>::T, 0, st>>>(g.S, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv, g.g, g.ldg, g.dec, g.lddec,
                                                 g.bias, g.hnw, g.eps, g.m, g.heads, g.out, g.ldo, g.fuse);
  SLM_LAUNCHED("k_gla");
}

}  // namespace

void gla(const GlaArgs& g, cudaStream_t st) {
  if (g.m == 0) return;
  switch (g.dh) {
    case 8: launch<8>(g, st); break;
    case 16: launch<16>(g, st); break;
    case 32: launch<32>(g, st); break;
    case 64: launch<64>(g, st); break;
    case 128: launch<128>(g, st); break;
    default: fail(SLM_ERR_INVALID, "gla: head size must be one of 8, 16, 32, 64, 128");
  }
}

}  // namespace slm
