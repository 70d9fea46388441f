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
// Columns of S are independent, so thread b keeps column S[·][b] in registers
// for the whole chunk; the state crosses HBM once per call (read at entry,
// written at exit).  One CTA per head; k and q of each token are shared
// through shared memory, double-buffered so one barrier per token suffices.
#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

template <int DH>
__global__ void __launch_bounds__(DH < 32 ? 32 : DH)
    k_gla(float* __restrict__ S, const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
          const float* __restrict__ v, int ldv, const float* __restrict__ gt, int ldg, const float* __restrict__ dec,
          int lddec, const float* __restrict__ bias, const float* __restrict__ hnw, float eps, int m, int heads,
          float* __restrict__ out, int ldo, int fuse) {
  constexpr int NW = (DH + 31) / 32;
  __shared__ float ks[2][DH], qs[2][DH], red[2][NW];
  const int h = blockIdx.x, b = threadIdx.x;
  const bool own = b < DH;
  const int lane = b & 31, warp = b >> 5;
  float col[DH];
  float* Sh = S + (size_t)h * DH * DH;
#pragma unroll
  for (int a = 0; a < DH; a++) col[a] = own ? Sh[(size_t)a * DH + b] : 0.0f;
  const float bh = bias[h];
  const float w = own && fuse ? hnw[b] : 0.0f;

  for (int i = 0; i < m; i++) {
    const int buf = i & 1;
    const size_t hb = (size_t)h * DH + b;
    float vb = 0.0f, gb = 0.0f;
    if (own) {
      ks[buf][b] = k[(size_t)i * ldk + hb];
      qs[buf][b] = q[(size_t)i * ldq + hb];
      vb = v[(size_t)i * ldv + hb];
      if (fuse) gb = gt[(size_t)i * ldg + hb];
    }
    const float d = 1.0f / (1.0f + expf(dec[(size_t)i * lddec + h] + bh));
    __syncthreads();
    float y = 0.0f;
#pragma unroll
    for (int a = 0; a < DH; a++) {
      col[a] = d * col[a] + ks[buf][a] * vb;
      y = fmaf(qs[buf][a], col[a], y);
    }
    if (!fuse) {
      if (own) out[(size_t)i * ldo + hb] = y;
      continue;
    }
    // head_norm over the DH values of this head, then the silu gate.
    float ss = warp_sum(own ? y * y : 0.0f);
    if (NW > 1) {
      if (lane == 0) red[buf][warp] = ss;
      __syncthreads();
      ss = 0.0f;
#pragma unroll
      for (int t = 0; t < NW; t++) ss += red[buf][t];
    }
    const float r = 1.0f / sqrtf(ss / (float)DH + eps);
    if (own) out[(size_t)i * ldo + hb] = silu_mul(gb, y * r * w);
  }
  if (own) {
#pragma unroll
    for (int a = 0; a < DH; a++) Sh[(size_t)a * DH + b] = col[a];
  }
}

template <int DH>
void launch(const GlaArgs& g, cudaStream_t st) {
  k_gla<DH><<<g.heads, DH < 32 ? 32 : DH, 0, st>>>(g.S, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv, g.g, g.ldg, g.dec,
                                                   g.lddec, g.bias, g.hnw, g.eps, g.m, g.heads, g.out, g.ldo,
                                                   g.fuse);
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
