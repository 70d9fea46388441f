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
#include <mutex>

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
          float* __restrict__ out, int ldo, int fuse, float* const* __restrict__ S_rows) {
  using Sh = GlaShape<DH>;
  constexpr int RQ = Sh::RQ, R = Sh::R, T = Sh::T, TC = Sh::TC;
  __shared__ float qs[TC][DH], ks[TC][DH], vs[TC][DH], ys[TC][DH], ds[TC];
  const int h = blockIdx.x, t = threadIdx.x;
  if (S_rows) {  // batched decode: sequence blockIdx.y, one token
    const int r = blockIdx.y;
    S = S_rows[r];
    q += (size_t)r * ldq, k += (size_t)r * ldk, v += (size_t)r * ldv, gt += (size_t)r * ldg;
    dec += (size_t)r * lddec, out += (size_t)r * ldo;
    m = 1;
  }
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

// ---------------------------------------------------------------------------
// Many tokens (prefill chunks): column-parallel recurrence + a norm/gate pass.
//
// A CTA owns CG = 32/RQ columns of one head's state (grid heads × DH/CG), one
// warp: each column is split over RQ = 8 lanes holding DH/8 of its rows in
// registers.  Lane rq owns the float4 chunks rq, rq + RQ, … of a row of q or
// k, so the lanes of a column read consecutive 16-byte words (no bank
// conflicts).  Tokens are staged TC at a time with cp.async, double-buffered,
// so the next stage loads while this one runs.  The bare y goes to `out`; the
// head_norm + gate (which need a whole head) follow in k_gla_norm.
// ---------------------------------------------------------------------------

#ifndef SLM_GLA_UNROLL
#define SLM_GLA_UNROLL 4
#endif
constexpr int kGlaUnroll = SLM_GLA_UNROLL;
#ifndef SLM_GLA_RQ
#define SLM_GLA_RQ 8  // lanes per state column
#endif

template <int DH>
struct GlaCols {
  // 8 lanes per column, 4 columns per one-warp CTA: heads × DH/4 CTAs (192
  // for 12 heads of 64), DH/8 rows of a column per lane.
  static constexpr int RQ = SLM_GLA_RQ, CG = 32 / RQ, R = DH / RQ, C4 = R / 4, T = CG * RQ;
  static constexpr int TC = 2048 / DH;  // tokens per stage (32 for DH 64)
};

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int DH>
__global__ void __launch_bounds__(GlaCols<DH>::T)
    k_gla_cols(float* __restrict__ S, const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
               const float* __restrict__ v, int ldv, const float* __restrict__ dec, int lddec,
               const float* __restrict__ bias, int m, float* __restrict__ out, int ldo) {
  using G = GlaCols<DH>;
  constexpr int CG = G::CG, RQ = G::RQ, C4 = G::C4, T = G::T, TC = G::TC;
  __shared__ __align__(16) float qs[2][TC][DH], ks[2][TC][DH], vs[2][TC][CG];
  __shared__ float ds[2][TC], ys[TC][CG];
  const int h = blockIdx.x, cg = blockIdx.y, t = threadIdx.x;
  const int b = t / RQ, rq = t % RQ;
  const int col0 = h * DH + cg * CG;
  float* Sh = S + (size_t)h * DH * DH;
  float col[C4][4];
#pragma unroll
  for (int c = 0; c < C4; c++)
#pragma unroll
    for (int e = 0; e < 4; e++) col[c][e] = Sh[(size_t)(4 * (rq + RQ * c) + e) * DH + cg * CG + b];
  const float bh = bias[h];

  auto stage = [&](int s) {
    const int c0 = s * TC, n = min(TC, m - c0), buf = s & 1;
    for (int e = t; e < n * (DH / 4); e += T) {
      const int i = e / (DH / 4), x = (e % (DH / 4)) * 4;
      const size_t row = (size_t)(c0 + i);
      cp16(&qs[buf][i][x], q + row * ldq + (size_t)h * DH + x);
      cp16(&ks[buf][i][x], k + row * ldk + (size_t)h * DH + x);
    }
    for (int e = t; e < n * (CG / 4); e += T) {
      const int i = e / (CG / 4), x = (e % (CG / 4)) * 4;
      cp16(&vs[buf][i][x], v + (size_t)(c0 + i) * ldv + col0 + x);
    }
    cp_commit();
    for (int i = t; i < n; i += T) ds[buf][i] = 1.0f / (1.0f + expf(dec[(size_t)(c0 + i) * lddec + h] + bh));
  };

  const int stages = (m + TC - 1) / TC;
  stage(0);
  for (int s = 0; s < stages; s++) {
    const int c0 = s * TC, n = min(TC, m - c0), buf = s & 1;
    if (s + 1 < stages) {
      stage(s + 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    // Only col[] carries from token to token: unrolled, the next tokens'
    // loads and y sums overlap this one's update.
#pragma unroll kGlaUnroll
    for (int i = 0; i < n; i++) {
      const float d = ds[buf][i], vb = vs[buf][i][b];
      const float4* q4 = reinterpret_cast<const float4*>(qs[buf][i]);
      const float4* k4 = reinterpret_cast<const float4*>(ks[buf][i]);
      float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
      for (int c = 0; c < C4; c++) {
        const float4 kk = k4[rq + RQ * c], qq = q4[rq + RQ * c];
        const float s0 = d * col[c][0] + kk.x * vb, s1 = d * col[c][1] + kk.y * vb;
        const float s2 = d * col[c][2] + kk.z * vb, s3 = d * col[c][3] + kk.w * vb;
        col[c][0] = s0, col[c][1] = s1, col[c][2] = s2, col[c][3] = s3;
        y0 = fmaf(qq.x, s0, y0);
        y1 = fmaf(qq.y, s1, y1);
        y0 = fmaf(qq.z, s2, y0);
        y1 = fmaf(qq.w, s3, y1);
      }
      float y = y0 + y1;
#pragma unroll
      for (int o = 1; o < RQ; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
      if (rq == 0) ys[i][b] = y;
    }
    __syncthreads();
    for (int e = t; e < n * CG; e += T) {
      const int i = e / CG, x = e % CG;
      out[(size_t)(c0 + i) * ldo + col0 + x] = ys[i][x];
    }
    __syncthreads();  // ys and this buffer are reused
  }
#pragma unroll
  for (int c = 0; c < C4; c++)
#pragma unroll
    for (int e = 0; e < 4; e++) Sh[(size_t)(4 * (rq + RQ * c) + e) * DH + cg * CG + b] = col[c][e];
}

// out[i][h] = silu(g[i][h]) · head_norm(y[i][h]) in place, one warp per (token, head).
template <int DH>
__global__ void __launch_bounds__(256)
    k_gla_norm(float* __restrict__ out, int ldo, const float* __restrict__ gt, int ldg, const float* __restrict__ hnw,
               float eps, int m, int heads) {
  constexpr int P = (DH + 31) / 32;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= m * heads) return;
  const int i = w / heads, h = w % heads;
  float* o = out + (size_t)i * ldo + (size_t)h * DH;
  const float* g = gt + (size_t)i * ldg + (size_t)h * DH;
  float y[P];
  float ss = 0.0f;
#pragma unroll
  for (int p = 0; p < P; p++) {
    const int x = lane + 32 * p;
    y[p] = x < DH ? o[x] : 0.0f;
    ss = fmaf(y[p], y[p], ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)DH + eps);
#pragma unroll
  for (int p = 0; p < P; p++) {
    const int x = lane + 32 * p;
    if (x < DH) o[x] = silu_mul(g[x], y[p] * r * hnw[x]);
  }
}

// ---------------------------------------------------------------------------
// Many tokens, head size 64: the chunked form of the same recurrence.  Over a
// sub-chunk of C tokens, with l_t = Σ_{u≤t} ln d_u (inclusive, from the
// sub-chunk's start) and S_0 the state before it:
//   y_t = e^{l_t} q_t·S_0 + Σ_{s≤t} e^{l_t − l_s} (q_t·k_s) v_s
//   S_C = e^{l_{C−1}} S_0 + Σ_s e^{l_{C−1} − l_s} k_s v_sᵀ
// which is the token recurrence written out (Π_{s<u≤t} d_u = e^{l_t − l_s});
// only the order of the additions differs.  The ln d_u (of the same float d
// the recurrence multiplies by; clamped at −87, below which d·S is lost to
// f32 anyway) are summed in double, so the differences l_t − l_s keep full
// precision however small the sub-chunk's decay product gets.  The
// sequential steps fall from m tokens to m / C sub-chunks of small matrix
// products in shared memory.
//
// A CTA owns kGCG columns of one head's state (grid heads × 64/kGCG, 256
// threads).  Every CTA of a head forms the same C × C matrix
// A[t][s] = e^{l_t − l_s} q_t·k_s (s ≤ t).  Rows of q, k and A are padded to
// 68 floats, so float4 reads of 8 consecutive rows fall in distinct banks.
// Sub-chunks are staged with cp.async, double-buffered.
// ---------------------------------------------------------------------------
constexpr int kGC = 64;   // tokens per sub-chunk
constexpr int kGCG = 8;   // state columns per CTA
constexpr int kGLD = 68;  // padded row of q, k and A
struct GlaChunkSmem {
  float q[2][kGC][kGLD], k[2][kGC][kGLD];
  float v[2][kGC][kGCG];
  float gd[2][kGC];    // ln d of each token (clamped), computed when the sub-chunk is staged
  float a[kGC][kGLD];  // A
  float s[64][kGCG];   // this CTA's state columns
  float w[kGC];        // e^{l_last − l_s}
  float el[kGC];       // e^{l_t}
  double l[kGC];
  float elast;
};

__global__ void __launch_bounds__(256)
    k_gla_chunk(float* __restrict__ S, const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
                const float* __restrict__ v, int ldv, const float* __restrict__ dec, int lddec,
                const float* __restrict__ bias, int m, float* __restrict__ out, int ldo) {
  constexpr int DH = 64;
  extern __shared__ __align__(16) char gsm_raw[];
  GlaChunkSmem& sm = *reinterpret_cast<GlaChunkSmem*>(gsm_raw);
  const int h = blockIdx.x, cg = blockIdx.y, t = threadIdx.x;
  const int col0 = h * DH + cg * kGCG;  // this CTA's columns of v and out
  float* Sh = S + (size_t)h * DH * DH;
  for (int e = t; e < DH * kGCG; e += 256) sm.s[e / kGCG][e % kGCG] = Sh[(size_t)(e / kGCG) * DH + cg * kGCG + e % kGCG];
  const float bh = bias[h];

  auto stage = [&](int c, int buf) {
    const int c0 = c * kGC, n = min(kGC, m - c0);
    for (int e = t; e < n * (DH / 4); e += 256) {
      const int i = e / (DH / 4), x = (e % (DH / 4)) * 4;
      const size_t row = (size_t)(c0 + i);
      cp16(&sm.q[buf][i][x], q + row * ldq + (size_t)h * DH + x);
      cp16(&sm.k[buf][i][x], k + row * ldk + (size_t)h * DH + x);
    }
    for (int e = t; e < n * (kGCG / 4); e += 256) {
      const int i = e / (kGCG / 4), x = (e % (kGCG / 4)) * 4;
      cp16(&sm.v[buf][i][x], v + (size_t)(c0 + i) * ldv + col0 + x);
    }
    cp_commit();
    for (int i = t; i < n; i += 256)
      sm.gd[buf][i] = fmaxf(logf(1.0f / (1.0f + expf(dec[(size_t)(c0 + i) * lddec + h] + bh))), -87.0f);
  };

  const int nch = (m + kGC - 1) / kGC;
  const int rb = t >> 4, cb = t & 15;    // A: rows rb + 16j, columns cb + 16k
  const int r4 = t >> 2, j2 = (t & 3) * 2;  // y row / state row, and two columns
  stage(0, 0);
  for (int c = 0; c < nch; c++) {
    const int c0 = c * kGC, n = min(kGC, m - c0), buf = c & 1;
    if (c + 1 < nch) {
      stage(c + 1, buf ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    // 1. Warp 0: ln d, their inclusive running sum (double), e^{l_t} and the
    // state weights e^{l_last − l_s}.  Rows ≥ n are never used.
    if (t < 32) {
      const int i0 = 2 * t, i1 = 2 * t + 1;
      double g0 = 0.0, g1 = 0.0;
      if (i0 < n) g0 = (double)sm.gd[buf][i0];
      if (i1 < n) g1 = (double)sm.gd[buf][i1];
      double p = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double u = __shfl_up_sync(0xffffffffu, p, o);
        if (t >= o) p += u;
      }
      double ex = __shfl_up_sync(0xffffffffu, p, 1);
      if (t == 0) ex = 0.0;
      sm.l[i0] = ex + g0;
      sm.l[i1] = (ex + g0) + g1;
      __syncwarp();
      const double lL = sm.l[n - 1];
      for (int i = t; i < kGC; i += 32) {
        sm.w[i] = i < n ? expf((float)(lL - sm.l[i])) : 0.0f;
        sm.el[i] = expf((float)sm.l[i]);
      }
      if (t == 0) sm.elast = expf((float)lL);
    }
    // 2. q_t·k_s for this thread's entries (rows rb + 16j, columns cb + 16k):
    // those with k > j lie above the diagonal (cb + 16(k − j) > rb) and are
    // not formed.
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int kk = 0; kk < 4; kk++) acc[j][kk] = 0.0f;
#pragma unroll 4
    for (int x = 0; x < DH; x += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) qv[j] = *reinterpret_cast<const float4*>(&sm.q[buf][rb + 16 * j][x]);
#pragma unroll
      for (int kk = 0; kk < 4; kk++) kv[kk] = *reinterpret_cast<const float4*>(&sm.k[buf][cb + 16 * kk][x]);
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int kk = 0; kk <= j; kk++) acc[j][kk] = dot4(qv[j], kv[kk], acc[j][kk]);
    }
    __syncthreads();  // l, w, el from warp 0
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const int r = rb + 16 * j, s = cb + 16 * kk;
        sm.a[r][s] = (s <= r && r < n) ? acc[j][kk] * expf((float)(sm.l[r] - sm.l[s])) : 0.0f;
      }
    __syncthreads();
    // 3. y_t = e^{l_t} q_t·S_0 + Σ_{s≤t} A[t][s] v_s, two columns per thread.
    if (r4 < n) {
      float y0 = 0.0f, y1 = 0.0f, z0 = 0.0f, z1 = 0.0f;
#pragma unroll 8
      for (int a = 0; a < DH; a++) {
        const float qa = sm.q[buf][r4][a];
        y0 = fmaf(qa, sm.s[a][j2], y0);
        y1 = fmaf(qa, sm.s[a][j2 + 1], y1);
      }
      for (int s = 0; s <= r4; s++) {
        const float as = sm.a[r4][s];
        z0 = fmaf(as, sm.v[buf][s][j2], z0);
        z1 = fmaf(as, sm.v[buf][s][j2 + 1], z1);
      }
      const float e = sm.el[r4];
      float* o = out + (size_t)(c0 + r4) * ldo + col0 + j2;
      o[0] = fmaf(e, y0, z0);
      o[1] = fmaf(e, y1, z1);
    }
    __syncthreads();  // every y has read S_0
    // 4. S_C = e^{l_last} S_0 + Σ_s e^{l_last − l_s} k_s v_sᵀ for state row r4.
    {
      float n0 = sm.elast * sm.s[r4][j2], n1 = sm.elast * sm.s[r4][j2 + 1];
      for (int s = 0; s < n; s++) {
        const float kw = sm.k[buf][s][r4] * sm.w[s];
        n0 = fmaf(kw, sm.v[buf][s][j2], n0);
        n1 = fmaf(kw, sm.v[buf][s][j2 + 1], n1);
      }
      sm.s[r4][j2] = n0;
      sm.s[r4][j2 + 1] = n1;
    }
    __syncthreads();  // the next sub-chunk reads the new state; this buffer is restaged
  }
  for (int e = t; e < DH * kGCG; e += 256) Sh[(size_t)(e / kGCG) * DH + cg * kGCG + e % kGCG] = sm.s[e / kGCG][e % kGCG];
}

#ifndef SLM_GLA_CHUNK_MIN
#define SLM_GLA_CHUNK_MIN 32  // fewer tokens keep the column-parallel recurrence
#endif

void launch_chunk(const GlaArgs& g, cudaStream_t st) {
  constexpr int kDevices = 64;
  static std::once_flag once[kDevices];
  int dev = 0;
  SLM_CUDA(cudaGetDevice(&dev));
  auto set = [] {
    SLM_CUDA(cudaFuncSetAttribute(k_gla_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(GlaChunkSmem)));
  };
  if (dev >= 0 && dev < kDevices)
    std::call_once(once[dev], set);
  else
    set();
  k_gla_chunk<<<dim3(g.heads, 64 / kGCG), 256, sizeof(GlaChunkSmem), st>>>(g.S, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv,
                                                                          g.dec, g.lddec, g.bias, g.m, g.out, g.ldo);
  SLM_LAUNCHED("k_gla_chunk");
  if (g.fuse) {
    const int warps = g.m * g.heads;
    k_gla_norm<64><<<(warps + 7) / 8, 256, 0, st>>>(g.out, g.ldo, g.g, g.ldg, g.hnw, g.eps, g.m, g.heads);
    SLM_LAUNCHED("k_gla_norm");
  }
}

template <int DH>
bool cols_ok(const GlaArgs& g) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return g.m >= 8 && g.ldq % 4 == 0 && g.ldk % 4 == 0 && g.ldv % 4 == 0 && al(g.q) && al(g.k) && al(g.v);
}

template <int DH>
void launch_cols(const GlaArgs& g, cudaStream_t st) {
  using G = GlaCols<DH>;
  k_gla_cols<DH><<<dim3(g.heads, DH / G::CG), G::T, 0, st>>>(g.S, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv, g.dec,
                                                             g.lddec, g.bias, g.m, g.out, g.ldo);
  SLM_LAUNCHED("k_gla_cols");
  if (g.fuse) {
    const int warps = g.m * g.heads;
    k_gla_norm<DH><<<(warps + 7) / 8, 256, 0, st>>>(g.out, g.ldo, g.g, g.ldg, g.hnw, g.eps, g.m, g.heads);
    SLM_LAUNCHED("k_gla_norm");
  }
}

template <int DH>
void launch(const GlaArgs& g, cudaStream_t st) {
  k_gla<DH><<<g.heads, GlaShape<DH>::T, 0, st>>>(g.S, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv, g.g, g.ldg, g.dec, g.lddec,
                                                 g.bias, g.hnw, g.eps, g.m, g.heads, g.out, g.ldo, g.fuse, nullptr);
  SLM_LAUNCHED("k_gla");
}

template <int DH>
void launch_rows(const GlaArgs& g, float* const* S_rows, cudaStream_t st) {
  k_gla<DH><<<dim3(g.heads, g.m), GlaShape<DH>::T, 0, st>>>(nullptr, g.q, g.ldq, g.k, g.ldk, g.v, g.ldv, g.g, g.ldg,
                                                           g.dec, g.lddec, g.bias, g.hnw, g.eps, 1, g.heads, g.out,
                                                           g.ldo, g.fuse, S_rows);
  SLM_LAUNCHED("k_gla");
}

}  // namespace

void gla(const GlaArgs& g, cudaStream_t st) {
  if (g.m == 0) return;
  switch (g.dh) {
    case 8: launch<8>(g, st); break;
    case 16: launch<16>(g, st); break;
    case 32: cols_ok<32>(g) ? launch_cols<32>(g, st) : launch<32>(g, st); break;
    case 64:
      if (cols_ok<64>(g) && g.m >= SLM_GLA_CHUNK_MIN && g.ldv % 4 == 0)
        launch_chunk(g, st);
      else
        cols_ok<64>(g) ? launch_cols<64>(g, st) : launch<64>(g, st);
      break;
    case 128: cols_ok<128>(g) ? launch_cols<128>(g, st) : launch<128>(g, st); break;
    default: fail(SLM_ERR_INVALID, "gla: head size must be one of 8, 16, 32, 64, 128");
  }
}

void gla_rows(const GlaArgs& g, float* const* S_rows, cudaStream_t st) {
  if (g.m == 0) return;
  switch (g.dh) {
    case 8: launch_rows<8>(g, S_rows, st); break;
    case 16: launch_rows<16>(g, S_rows, st); break;
    case 32: launch_rows<32>(g, S_rows, st); break;
    case 64: launch_rows<64>(g, S_rows, st); break;
    case 128: launch_rows<128>(g, S_rows, st); break;
    default: fail(SLM_ERR_INVALID, "gla: head size must be one of 8, 16, 32, 64, 128");
  }
}

}  // namespace slm
