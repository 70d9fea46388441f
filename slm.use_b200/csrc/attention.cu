// Softmax attention over ring caches (reference Ops::attend, src/ops.rs:218-227;
// CPU arithmetic src/cpu.rs:352-403; window geometry src/ops.rs:31-66).
//
// The query at position p reads cached positions lo..hi-1 with
// lo = max(0, p - reach + 1) (reach 0 = unbounded) and hi = p + 1 - gap, kept
// in ring slots p % cap of a [key_head][cap][dh] cache.  A query that sees
// nothing yields zeros.
//
// Scores are never materialised.  Each (query, head) range is cut into
// `nsplit` contiguous slices; a CTA folds its slice into a running
// (max, sum, acc[dh]) with online softmax and writes that partial, and
// k_attn_combine merges the slices.  Two shapes of the slice pass:
//  * k_attn_split (m ≤ 8, decode): 8-float lane groups walk the slice, one
//    cache row per group per step, K and V read once with 16-byte loads.
//  * k_attn_tile (m > 8, prefill chunks): 16 queries share 32-position K/V
//    tiles staged in shared memory.
// The position of the first query comes from device memory, so the same
// launch (and a CUDA graph holding it) serves every decode step.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "window.cuh"

namespace slm {

namespace {

// Merge two online-softmax partials (m, l, acc) into the first.
__device__ __forceinline__ void merge(float& m, float& l, float* acc, float om, float ol, const float* oacc, int n) {
  float M = fmaxf(m, om);
  float ca = m == -INFINITY ? 0.0f : expf(m - M);
  float cb = om == -INFINITY ? 0.0f : expf(om - M);
  l = l * ca + ol * cb;
  for (int e = 0; e < n; e++) acc[e] = acc[e] * ca + oacc[e] * cb;
  m = M;
}

// Merge of the nsplit slices of (query i, head h) into y, by the NT threads
// of a CTA: M = max_s m_s, c_s = e^{m_s − M}, L = Σ c_s l_s, then thread
// (q, e) sums c_s·acc_s[e] over splits q, q + Q, … and the Q sums are added in
// order.  cw holds up to 256 split weights; acc_sh is [4][dh + 4].
template <int NT>
__device__ void combine_pair(const float* __restrict__ part, int nsplit, int m, int heads, int dh, int i, int h,
                             float* __restrict__ y, int ldy, float* red, float* cw, float* acc_sh) {
  constexpr int NW = NT / 32;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const size_t stride = (size_t)m * heads * (dh + 2);
  const float* p0 = part + ((size_t)i * heads + h) * (dh + 2);
  float mx = -INFINITY;
  for (int s = t; s < nsplit; s += NT) mx = fmaxf(mx, __ldcg(p0 + s * stride + dh));
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = red[0];
  for (int w = 1; w < NW; w++) M = fmaxf(M, red[w]);
  __syncthreads();
  float lsum = 0.0f;
  for (int s = t; s < nsplit; s += NT) {
    const float ms = __ldcg(p0 + s * stride + dh);
    const float c = (M == -INFINITY || ms == -INFINITY) ? 0.0f : expf(ms - M);
    if (s < 256) cw[s] = c;
    lsum += __ldcg(p0 + s * stride + dh + 1) * c;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) red[warp] = lsum;
  __syncthreads();
  float L = 0.0f;
  for (int w = 0; w < NW; w++) L += red[w];
  const int Q = NT / dh >= 1 ? (NT / dh > 4 ? 4 : NT / dh) : 1;
  const int q = t / dh, e = t % dh;
  float a = 0.0f;
  if (q < Q && dh <= NT) {
    // Splits q, q + Q, … in order; eight loads in flight at a time.
    int s = q;
    for (; s + 7 * Q < nsplit; s += 8 * Q) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = __ldcg(p0 + (size_t)(s + u * Q) * stride + e);
#pragma unroll
      for (int u = 0; u < 8; u++) a = fmaf(v[u], cw[s + u * Q], a);
    }
    for (; s < nsplit; s += Q) a = fmaf(__ldcg(p0 + (size_t)s * stride + e), cw[s], a);
    acc_sh[q * (dh + 4) + e] = a;
  }
  __syncthreads();
  for (int d = t; d < dh; d += NT) {
    float v = 0.0f;
    if (dh <= NT) {
      for (int qq = 0; qq < Q; qq++) v += acc_sh[qq * (dh + 4) + d];
    } else {  // heads wider than the CTA: one thread per dimension, splits in order
      for (int s = 0; s < nsplit; s++) v = fmaf(__ldcg(p0 + (size_t)s * stride + d), cw[s], v);
    }
    y[(size_t)i * ldy + (size_t)h * dh + d] = L > 0.0f ? v / L : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// Slice pass for a few queries.  grid (nsplit, heads, m), 128 threads.
// ---------------------------------------------------------------------------
// With `rows` set, query i belongs to its own sequence: its cache is
// rows->k[i] / rows->v[i] and its position *rows->pos[i] (batched decode of
// independent sessions, one token each).
constexpr int kSplitThreads = 256;  // 8 warps: a 128-position slice is one round of loads

template <int DH>
__global__ void __launch_bounds__(kSplitThreads)
    k_attn_split(const float* __restrict__ q, int ldq, const float* __restrict__ K, const float* __restrict__ V,
                 AttnGeom g, const long long* __restrict__ pos_ptr, int nsplit, float* __restrict__ part,
                 AttnRows rows, unsigned* __restrict__ cnt, float* __restrict__ y, int ldy) {
  constexpr int G = DH / 8;        // lanes per cache row
  constexpr int PPW = 32 / G;      // rows per warp step
  constexpr int WARPS = kSplitThreads / 32;
  const int s = blockIdx.x, h = blockIdx.y, i = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % G, grp = lane / G;
  long long cap = g.cap;
  if (rows.pos) {
    K = rows.k[i];
    V = rows.v[i];
    if (rows.cap) cap = rows.cap[i];
  }
  const long long p = rows.pos ? *rows.pos[i] : (pos_ptr ? pos_ptr[0] : g.pos0) + i;
  Range r = visible(p, g.reach, g.gap);
  long long count = r.hi - r.lo;
  long long chunk = (count + nsplit - 1) / nsplit;
  long long start = r.lo + (long long)s * chunk;
  long long end = min(r.hi, start + chunk);

  const int kvh = h / (g.heads / g.key_heads);
  const float* Kb = K + (size_t)kvh * cap * DH + sub * 8;
  const float* Vb = V + (size_t)kvh * cap * DH + sub * 8;
  const float* qp = q + (size_t)i * ldq + (size_t)h * DH + sub * 8;
  float qv[8];
  {
    float4 a = *reinterpret_cast<const float4*>(qp), b = *reinterpret_cast<const float4*>(qp + 4);
    qv[0] = a.x, qv[1] = a.y, qv[2] = a.z, qv[3] = a.w, qv[4] = b.x, qv[5] = b.y, qv[6] = b.z, qv[7] = b.w;
  }
  float mx = -INFINITY, l = 0.0f, acc[8];
#pragma unroll
  for (int e = 0; e < 8; e++) acc[e] = 0.0f;

  // U cache rows per lane group per round: all their loads are issued before
  // any is used, and the running max / rescale is applied once per round.
  constexpr int U = 4;
  const long long slot0 = start < end ? start % cap : 0;
  for (long long base = start + warp * PPW * U; base < end; base += (long long)WARPS * PPW * U) {
    float4 k0[U], k1[U], v0[U], v1[U];
    bool okk[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long pp = base + u * PPW + grp;
      okk[u] = pp < end;
      k0[u] = k1[u] = v0[u] = v1[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (okk[u]) {
        long long sl = slot0 + (pp - start);
        if (sl >= cap) sl -= cap;
        if (sl >= cap) sl %= cap;
        const size_t slot = (size_t)sl;
        const float4* kr = reinterpret_cast<const float4*>(Kb + slot * DH);
        const float4* vr = reinterpret_cast<const float4*>(Vb + slot * DH);
        k0[u] = ld_stream(kr);
        k1[u] = ld_stream(kr + 1);
        v0[u] = ld_stream(vr);
        v1[u] = ld_stream(vr + 1);
      }
    }
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      sc[u] = qv[0] * k0[u].x + qv[1] * k0[u].y + qv[2] * k0[u].z + qv[3] * k0[u].w + qv[4] * k1[u].x +
              qv[5] * k1[u].y + qv[6] * k1[u].z + qv[7] * k1[u].w;
#pragma unroll
    for (int o = 1; o < G; o <<= 1)
#pragma unroll
      for (int u = 0; u < U; u++) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
    float M = mx;
#pragma unroll
    for (int u = 0; u < U; u++) {
      sc[u] *= g.scale;
      if (okk[u]) M = fmaxf(M, sc[u]);
    }
    if (M == -INFINITY) continue;  // nothing visible in this round for this group
    const float corr = mx == -INFINITY ? 0.0f : expf(mx - M);
    l *= corr;
#pragma unroll
    for (int e = 0; e < 8; e++) acc[e] *= corr;
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (!okk[u]) continue;
      const float pe = expf(sc[u] - M);
      l += pe;
      acc[0] += pe * v0[u].x, acc[1] += pe * v0[u].y, acc[2] += pe * v0[u].z, acc[3] += pe * v0[u].w;
      acc[4] += pe * v1[u].x, acc[5] += pe * v1[u].y, acc[6] += pe * v1[u].z, acc[7] += pe * v1[u].w;
    }
    mx = M;
  }
  // Merge the lane groups of the warp (they hold the same `sub` slices).
#pragma unroll
  for (int o = G; o < 32; o <<= 1) {
    float om = __shfl_xor_sync(0xffffffffu, mx, o);
    float ol = __shfl_xor_sync(0xffffffffu, l, o);
    float oacc[8];
#pragma unroll
    for (int e = 0; e < 8; e++) oacc[e] = __shfl_xor_sync(0xffffffffu, acc[e], o);
    merge(mx, l, acc, om, ol, oacc, 8);
  }
  // Merge the warps through shared memory.
  __shared__ float sm[WARPS][DH + 2];
  if (grp == 0) {
#pragma unroll
    for (int e = 0; e < 8; e++) sm[warp][sub * 8 + e] = acc[e];
    if (sub == 0) {
      sm[warp][DH] = mx;
      sm[warp][DH + 1] = l;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < DH; e += blockDim.x) {
    float m0 = sm[0][DH], l0 = sm[0][DH + 1], a0 = sm[0][e];
    for (int w = 1; w < WARPS; w++) merge(m0, l0, &a0, sm[w][DH], sm[w][DH + 1], &sm[w][e], 1);
    float* out = part + (((size_t)s * g.m + i) * g.heads + h) * (DH + 2);
    out[e] = a0;
    if (e == 0) {
      out[DH] = m0;
      out[DH + 1] = l0;
    }
  }
  if (!cnt) return;  // a separate combine launch merges the slices
  // The last slice of (i, h) to finish merges them all and puts its counter
  // back to zero for the next launch.
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* c = cnt + (size_t)i * g.heads + h;
    last = atomicAdd(c, 1u) == (unsigned)nsplit - 1;
    if (last) *c = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  __shared__ float red[WARPS], cw[256], acc_sh[4 * (DH + 4)];
  combine_pair<kSplitThreads>(part, nsplit, g.m, g.heads, DH, i, h, y, ldy, red, cw, acc_sh);
}

// ---------------------------------------------------------------------------
// Slice pass for query tiles.  grid (nsplit, ceil(m/16), heads), 128 threads;
// each warp owns 4 queries; 32-position K/V tiles in shared memory.
// ---------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(128)
    k_attn_tile(const float* __restrict__ q, int ldq, const float* __restrict__ K, const float* __restrict__ V,
                AttnGeom g, const long long* __restrict__ pos_ptr, int nsplit, float* __restrict__ part) {
  constexpr int QT = 16, QW = 4, KT = 32, LD = DH + 1;
  constexpr int DPL = (DH + 31) / 32;  // output dims per lane
  __shared__ float Ks[KT][LD], Vs[KT][LD];
  __shared__ __align__(16) float Qs[4][DH][QW];  // per warp, transposed: [warp][d][query]
  const int s = blockIdx.x, i0 = blockIdx.y * QT, h = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long pos = pos_ptr ? pos_ptr[0] : g.pos0;
  const int kvh = h / (g.heads / g.key_heads);
  const float* Kb = K + (size_t)kvh * g.cap * DH;
  const float* Vb = V + (size_t)kvh * g.cap * DH;

  // Union of the tile's ranges (ranges grow with the query position).
  int ilast = min(i0 + QT, g.m) - 1;
  Range r0 = visible(pos + i0, g.reach, g.gap), r1 = visible(pos + ilast, g.reach, g.gap);
  long long ulo = r0.lo, uhi = max(r1.hi, r0.hi);
  long long count = uhi - ulo;
  long long chunk = (count + nsplit - 1) / nsplit;
  long long start = ulo + (long long)s * chunk, end = min(uhi, start + chunk);

  // This warp's queries.
  long long qlo[QW], qhi[QW];
  bool qok[QW];
#pragma unroll
  for (int j = 0; j < QW; j++) {
    int i = i0 + warp * QW + j;
    qok[j] = i < g.m;
    Range rr = visible(pos + i, g.reach, g.gap);
    qlo[j] = qok[j] ? rr.lo : 0;
    qhi[j] = qok[j] ? rr.hi : 0;
    for (int d = lane; d < DH; d += 32)
      Qs[warp][d][j] = qok[j] ? q[(size_t)i * ldq + (size_t)h * DH + d] : 0.0f;
  }
  float mx[QW], l[QW], acc[QW][DPL];
#pragma unroll
  for (int j = 0; j < QW; j++) {
    mx[j] = -INFINITY;
    l[j] = 0.0f;
#pragma unroll
    for (int t = 0; t < DPL; t++) acc[j][t] = 0.0f;
  }
  __syncwarp();

  for (long long t0 = start; t0 < end; t0 += KT) {
    __syncthreads();
    // Stage K/V rows t0 .. t0+KT-1 (zeros past `end`).
    for (int e = threadIdx.x; e < KT * (DH / 4); e += blockDim.x) {
      int row = e / (DH / 4), c = (e % (DH / 4)) * 4;
      long long pp = t0 + row;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (pp < end) {
        size_t slot = (size_t)(pp % g.cap);
        kv = ld_stream(reinterpret_cast<const float4*>(Kb + slot * DH + c));
        vv = ld_stream(reinterpret_cast<const float4*>(Vb + slot * DH + c));
      }
      Ks[row][c] = kv.x, Ks[row][c + 1] = kv.y, Ks[row][c + 2] = kv.z, Ks[row][c + 3] = kv.w;
      Vs[row][c] = vv.x, Vs[row][c + 1] = vv.y, Vs[row][c + 2] = vv.z, Vs[row][c + 3] = vv.w;
    }
    __syncthreads();
    // Scores: lane ↔ position t0 + lane.
    float sc[QW];
#pragma unroll
    for (int j = 0; j < QW; j++) sc[j] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < DH; d++) {
      float kd = Ks[lane][d];
      float4 qd = *reinterpret_cast<const float4*>(&Qs[warp][d][0]);
      sc[0] = fmaf(qd.x, kd, sc[0]);
      sc[1] = fmaf(qd.y, kd, sc[1]);
      sc[2] = fmaf(qd.z, kd, sc[2]);
      sc[3] = fmaf(qd.w, kd, sc[3]);
    }
    long long pp = t0 + lane;
    float pe[QW];
#pragma unroll
    for (int j = 0; j < QW; j++) {
      bool vis = qok[j] && pp < end && pp >= qlo[j] && pp < qhi[j];
      float sj = vis ? sc[j] * g.scale : -INFINITY;
      float tmax = warp_max(sj);
      if (tmax == -INFINITY) {
        pe[j] = 0.0f;
        continue;
      }
      float M = fmaxf(mx[j], tmax);
      float corr = mx[j] == -INFINITY ? 0.0f : expf(mx[j] - M);
      pe[j] = vis ? expf(sj - M) : 0.0f;
      l[j] = l[j] * corr + warp_sum(pe[j]);
#pragma unroll
      for (int t = 0; t < DPL; t++) acc[j][t] *= corr;
      mx[j] = M;
    }
    // P·V: lane owns output dims lane + 32t.
    for (int k = 0; k < KT; k++) {
      float pk[QW];
#pragma unroll
      for (int j = 0; j < QW; j++) pk[j] = __shfl_sync(0xffffffffu, pe[j], k);
#pragma unroll
      for (int t = 0; t < DPL; t++) {
        int d = lane + 32 * t;
        float vd = d < DH ? Vs[k][d] : 0.0f;
#pragma unroll
        for (int j = 0; j < QW; j++) acc[j][t] = fmaf(pk[j], vd, acc[j][t]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < QW; j++) {
    int i = i0 + warp * QW + j;
    if (i >= g.m) continue;
    float* out = part + (((size_t)s * g.m + i) * g.heads + h) * (DH + 2);
#pragma unroll
    for (int t = 0; t < DPL; t++) {
      int d = lane + 32 * t;
      if (d < DH) out[d] = acc[j][t];
    }
    if (lane == 0) {
      out[DH] = mx[j];
      out[DH + 1] = l[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Slice pass for query tiles, head size 64 (prefill chunks).  grid (nsplit,
// ceil(m/64), heads), 256 threads.  64 queries × 64-key tiles, register-tiled:
// thread (ty, tx) = (t/16, t%16) scores queries 4ty..4ty+3 against keys tx,
// tx+16, tx+32, tx+48 (so a warp's K reads hit distinct banks) and accumulates
// outputs of queries 4ty.. × dims 4tx..4tx+3; rows are padded to 68 floats.
// K/V tiles are gathered from the ring with cp.async, double-buffered; the
// probabilities of a tile pass through shared memory for P·V.
// ---------------------------------------------------------------------------

constexpr int FQ = 64, FKT = 64, FLD = 68;
constexpr size_t kFlashSmem = (size_t)(FQ + 4 * FKT + FQ) * FLD * sizeof(float);

__device__ __forceinline__ void cp16z(void* dst, const void* src, bool ok) {
  unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

__global__ void __launch_bounds__(256, 2)
    k_attn_flash(const float* __restrict__ q, int ldq, const float* __restrict__ K, const float* __restrict__ V,
                 AttnGeom g, const long long* __restrict__ pos_ptr, int nsplit, float* __restrict__ part) {
  constexpr int DH = 64;
  extern __shared__ __align__(16) float fsm[];
  float(*Qs)[FLD] = reinterpret_cast<float(*)[FLD]>(fsm);
  float(*Ks)[FKT][FLD] = reinterpret_cast<float(*)[FKT][FLD]>(fsm + FQ * FLD);
  float(*Vs)[FKT][FLD] = reinterpret_cast<float(*)[FKT][FLD]>(fsm + (FQ + 2 * FKT) * FLD);
  float(*Ps)[FLD] = reinterpret_cast<float(*)[FLD]>(fsm + (FQ + 4 * FKT) * FLD);
  const int s = blockIdx.x, i0 = blockIdx.y * FQ, h = blockIdx.z;
  const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
  const long long pos = pos_ptr ? pos_ptr[0] : g.pos0;
  const int kvh = h / (g.heads / g.key_heads);
  const float* Kb = K + (size_t)kvh * g.cap * DH;
  const float* Vb = V + (size_t)kvh * g.cap * DH;

  const int ilast = min(i0 + FQ, g.m) - 1;
  const Range r0 = visible(pos + i0, g.reach, g.gap), r1 = visible(pos + ilast, g.reach, g.gap);
  const long long ulo = r0.lo, uhi = max(r1.hi, r0.hi);
  const long long count = uhi - ulo, chunk = (count + nsplit - 1) / nsplit;
  const long long start = ulo + (long long)s * chunk, end = min(uhi, start + chunk);

  long long qlo[4], qhi[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int i = i0 + 4 * ty + j;
    const Range rr = visible(pos + i, g.reach, g.gap);
    qlo[j] = i < g.m ? rr.lo : 0;
    qhi[j] = i < g.m ? rr.hi : 0;
  }
  for (int e = t; e < FQ * (DH / 4); e += 256) {
    const int row = e / (DH / 4), c = (e % (DH / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i0 + row < g.m) v = *reinterpret_cast<const float4*>(q + (size_t)(i0 + row) * ldq + (size_t)h * DH + c);
    *reinterpret_cast<float4*>(&Qs[row][c]) = v;
  }

  auto load = [&](int tile, int buf) {
    const long long base = start + (long long)tile * FKT;
    for (int e = t; e < FKT * (DH / 4); e += 256) {
      const int row = e / (DH / 4), c = (e % (DH / 4)) * 4;
      const long long pp = base + row;
      const bool ok = pp < end;
      const size_t slot = ok ? (size_t)(pp % g.cap) : 0;
      cp16z(&Ks[buf][row][c], Kb + slot * DH + c, ok);
      cp16z(&Vs[buf][row][c], Vb + slot * DH + c, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float o[4][4], mx[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    mx[j] = -INFINITY;
    l[j] = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; e++) o[j][e] = 0.0f;
  }
  const int ntiles = start < end ? (int)((end - start + FKT - 1) / FKT) : 0;
  if (ntiles > 0) load(0, 0);
  for (int tile = 0; tile < ntiles; tile++) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) {
      load(tile + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int k = 0; k < 4; k++) sc[j][k] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < DH; d += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) qv[j] = *reinterpret_cast<const float4*>(&Qs[4 * ty + j][d]);
#pragma unroll
      for (int k = 0; k < 4; k++) kv[k] = *reinterpret_cast<const float4*>(&Ks[buf][tx + 16 * k][d]);
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int k = 0; k < 4; k++) sc[j][k] = dot4(qv[j], kv[k], sc[j][k]);
    }
    const long long base = start + (long long)tile * FKT;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float tmax = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const long long kp = base + tx + 16 * k;
        const bool vis = kp < end && kp >= qlo[j] && kp < qhi[j];
        sc[j][k] = vis ? sc[j][k] * g.scale : -INFINITY;
        tmax = fmaxf(tmax, sc[j][k]);
      }
#pragma unroll
      for (int o2 = 1; o2 < 16; o2 <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o2));
      const float M = fmaxf(mx[j], tmax);
      float rs = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float p = sc[j][k] == -INFINITY ? 0.0f : expf(sc[j][k] - M);
        Ps[4 * ty + j][tx + 16 * k] = p;
        rs += p;
      }
#pragma unroll
      for (int o2 = 1; o2 < 16; o2 <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o2);
      const float corr = mx[j] == -INFINITY ? 0.0f : expf(mx[j] - M);
      l[j] = l[j] * corr + rs;
#pragma unroll
      for (int e = 0; e < 4; e++) o[j][e] *= corr;
      mx[j] = M;
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < FKT; k += 4) {
      float4 pv[4], vv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) pv[j] = *reinterpret_cast<const float4*>(&Ps[4 * ty + j][k]);
#pragma unroll
      for (int kk = 0; kk < 4; kk++) vv[kk] = *reinterpret_cast<const float4*>(&Vs[buf][k + kk][4 * tx]);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float p4[4] = {pv[j].x, pv[j].y, pv[j].z, pv[j].w};
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          o[j][0] = fmaf(p4[kk], vv[kk].x, o[j][0]);
          o[j][1] = fmaf(p4[kk], vv[kk].y, o[j][1]);
          o[j][2] = fmaf(p4[kk], vv[kk].z, o[j][2]);
          o[j][3] = fmaf(p4[kk], vv[kk].w, o[j][3]);
        }
      }
    }
    __syncthreads();  // Ps and this K/V buffer are rewritten next
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int i = i0 + 4 * ty + j;
    if (i >= g.m) continue;
    float* out = part + (((size_t)s * g.m + i) * g.heads + h) * (DH + 2);
    // Rows of dh + 2 floats are only 8-byte aligned: scalar stores.
#pragma unroll
    for (int e = 0; e < 4; e++) out[4 * tx + e] = o[j][e];
    if (tx == 0) {
      out[DH] = mx[j];
      out[DH + 1] = l[j];
    }
  }
}

// Merge the slices: y[i][h] = Σ_s e^{m_s - M} acc_s / Σ_s e^{m_s - M} l_s.
// grid m·heads, 256 threads: the slices are spread over the threads (max and
// weighted sums as block reductions), so the merge costs a few L2 round trips
// whatever the split count.  Slices combine in a fixed order per thread and
// a fixed tree across threads.
__global__ void __launch_bounds__(256) k_attn_combine(const float* __restrict__ part, int nsplit, int m, int heads,
                                                      int dh, float* __restrict__ y, int ldy) {
  __shared__ float red[8], cw[256];
  __shared__ float acc_sh[4][256 + 4];
  const int pair = blockIdx.x, i = pair / heads, h = pair % heads, t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const size_t stride = (size_t)m * heads * (dh + 2);
  const float* p0 = part + ((size_t)i * heads + h) * (dh + 2);
  // 1. M = max_s m_s.
  float mx = -INFINITY;
  for (int s = t; s < nsplit; s += 256) mx = fmaxf(mx, p0[s * stride + dh]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = red[0];
  for (int w = 1; w < 8; w++) M = fmaxf(M, red[w]);
  __syncthreads();
  // 2. c_s = e^{m_s - M} (kept per split), L = Σ c_s l_s.
  float lsum = 0.0f;
  for (int s = t; s < nsplit; s += 256) {
    const float ms = p0[s * stride + dh];
    const float c = (M == -INFINITY || ms == -INFINITY) ? 0.0f : expf(ms - M);
    if (s < 256) cw[s] = c;
    lsum += p0[s * stride + dh + 1] * c;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) red[warp] = lsum;
  __syncthreads();
  float L = 0.0f;
  for (int w = 0; w < 8; w++) L += red[w];
  // 3. Σ_s c_s acc_s[e]: thread (q, e) takes the splits q, q + Q, … for dim e.
  const int Q = 256 / dh >= 1 ? (256 / dh > 4 ? 4 : 256 / dh) : 1;
  const int q = t / dh, e = t % dh;
  float a = 0.0f;
  if (q < Q && dh <= 256) {
    // Splits q, q + Q, … in order; eight loads in flight at a time.
    int s = q;
    for (; s + 7 * Q < nsplit; s += 8 * Q) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = p0[(size_t)(s + u * Q) * stride + e];
#pragma unroll
      for (int u = 0; u < 8; u++) a = fmaf(v[u], cw[s + u * Q], a);
    }
    for (; s < nsplit; s += Q) a = fmaf(p0[(size_t)s * stride + e], cw[s], a);
  }
  if (q < Q) acc_sh[q][e] = a;
  __syncthreads();
  for (int d = t; d < dh; d += 256) {
    float v = 0.0f;
    for (int qq = 0; qq < Q; qq++) v += acc_sh[qq][d];
    y[(size_t)i * ldy + (size_t)h * dh + d] = L > 0.0f ? v / L : 0.0f;
  }
}

// The same merge for head size 64, one warp per (query, head): the splits'
// weights e^{m_s − M} live in the lanes (32 splits at a time) and every lane
// adds its two dims over the splits in order.  One wave for a chunk's
// 256 × 12 pairs, instead of a 256-thread CTA with block reductions each.
__global__ void __launch_bounds__(256) k_attn_combine64(const float* __restrict__ part, int nsplit, int m, int heads,
                                                        float* __restrict__ y, int ldy) {
  constexpr int DH = 64;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pair >= m * heads) return;  // whole warps
  const int i = pair / heads, h = pair % heads;
  const size_t stride = (size_t)m * heads * (DH + 2);
  const float* p0 = part + ((size_t)i * heads + h) * (DH + 2);
  float M = -INFINITY;
  for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, __ldcg(p0 + s * stride + DH));
  M = warp_max(M);
  float L = 0.0f, a0 = 0.0f, a1 = 0.0f;
  for (int s0 = 0; s0 < nsplit; s0 += 32) {
    const int s = s0 + lane;
    float c = 0.0f;
    if (s < nsplit) {
      const float ms = __ldcg(p0 + s * stride + DH);
      c = (M == -INFINITY || ms == -INFINITY) ? 0.0f : expf(ms - M);
      L = fmaf(__ldcg(p0 + s * stride + DH + 1), c, L);
    }
    const int n = min(32, nsplit - s0);
    for (int k = 0; k < n; k++) {
      const float ck = __shfl_sync(0xffffffffu, c, k);
      const float* ps = p0 + (size_t)(s0 + k) * stride;
      a0 = fmaf(__ldcg(ps + lane), ck, a0);
      a1 = fmaf(__ldcg(ps + 32 + lane), ck, a1);
    }
  }
  L = warp_sum(L);
  float* yo = y + (size_t)i * ldy + (size_t)h * DH;
  yo[lane] = L > 0.0f ? a0 / L : 0.0f;
  yo[32 + lane] = L > 0.0f ? a1 / L : 0.0f;
}

void combine(const float* part, int nsplit, const AttnGeom& g, float* y, int ldy, cudaStream_t st) {
  if (g.dh == 64) {
    k_attn_combine64<<<(g.m * g.heads + 7) / 8, 256, 0, st>>>(part, nsplit, g.m, g.heads, y, ldy);
    SLM_LAUNCHED("k_attn_combine64");
    return;
  }
  k_attn_combine<<<g.m * g.heads, 256, 0, st>>>(part, nsplit, g.m, g.heads, g.dh, y, ldy);
  SLM_LAUNCHED("k_attn_combine");
}

template <int DH>
void launch_tile(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g, const long long* pos_ptr,
                 int nsplit, float* part, cudaStream_t st) {
  if constexpr (DH == 64) {
    if (attention_tc_on()) {
      attention_tc(q, ldq, K, V, g, pos_ptr, nsplit, part, st);
      return;
    }
    // The shared-memory limit is a per-device function attribute: set it on
    // the first launch on each device (a process may drive several).
    constexpr int kDevices = 64;
    static std::once_flag once[kDevices];
    int dev = 0;
    SLM_CUDA(cudaGetDevice(&dev));
    auto set = [] {
      SLM_CUDA(cudaFuncSetAttribute(k_attn_flash, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlashSmem));
    };
    if (dev >= 0 && dev < kDevices)
      std::call_once(once[dev], set);
    else
      set();
    k_attn_flash<<<dim3(nsplit, cdiv(g.m, FQ), g.heads), 256, kFlashSmem, st>>>(q, ldq, K, V, g, pos_ptr, nsplit,
                                                                                part);
    SLM_LAUNCHED("k_attn_flash");
  } else if constexpr (DH <= 128) {
    k_attn_tile<DH><<<dim3(nsplit, cdiv(g.m, 16), g.heads), 128, 0, st>>>(q, ldq, K, V, g, pos_ptr, nsplit, part);
    SLM_LAUNCHED("k_attn_tile");
  }
}

// True when the slice pass merged the slices itself (a fused merge needs counters).
template <int DH>
bool launch_dh(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g, const long long* pos_ptr,
               int nsplit, float* part, unsigned* cnt, float* y, int ldy, cudaStream_t st) {
  if (g.m <= 8 || DH > 128) {
    k_attn_split<DH><<<dim3(nsplit, g.heads, g.m), kSplitThreads, 0, st>>>(q, ldq, K, V, g, pos_ptr, nsplit, part,
                                                                 AttnRows{}, cnt, y, ldy);
    SLM_LAUNCHED("k_attn_split");
    return cnt != nullptr;
  }
  launch_tile<DH>(q, ldq, K, V, g, pos_ptr, nsplit, part, st);
  return false;
}

}  // namespace

int attn_splits(const AttnGeom& g, long long max_span) {
  if (max_span < 1) max_span = 1;
  const bool tc = g.m > 8 && g.dh == 64 && attention_tc_on();
  long long ctas = (g.m <= 8 || g.dh > 128) ? (long long)g.heads * g.m
                  : tc                       ? (long long)g.heads * ((g.m + 127) / 128)
                  : g.dh == 64               ? (long long)g.heads * ((g.m + FQ - 1) / FQ)
                                             : (long long)g.heads * ((g.m + 15) / 16);
  // Decode-sized calls (the slice pass): at most two 256-thread CTAs per SM
  // (one wave at 127 registers a thread) and slices of at least 256
  // positions; the last slice of each (query, head) merges them.  Measured on
  // the m = 1 op over a 4096 window: 12.5 µs per call with 16 slices, 12.4–18
  // µs for 8 to 64 slices of 4 or 8 warps.  Chunks: two CTAs per SM; the flash tiles hold
  // exactly two per SM, so their count rounds down to one full wave.
  const bool slices = g.m <= 8 || g.dh > 128;
  constexpr long long per_sm = 2, min_pos = 256;
  // The tensor-core pass holds one CTA per SM: one wave of them.
  long long want = tc                       ? std::max(1ll, 148 / ctas)
                   : (g.m > 8 && g.dh == 64) ? std::max(1ll, (2 * 148) / ctas)
                   : slices                ? (per_sm * 148 + ctas - 1) / ctas
                                           : (2 * 148 + ctas - 1) / ctas;
  const long long step = slices ? min_pos : 128;  // positions per slice at least
  long long most = (max_span + step - 1) / step;
  long long n = want < most ? want : most;
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

size_t attn_part_floats(const AttnGeom& g, int nsplit) { return (size_t)nsplit * g.m * g.heads * (g.dh + 2); }

void attention(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g, const long long* pos_ptr,
               int nsplit, float* part, float* y, int ldy, cudaStream_t st, unsigned* cnt) {
  if (g.m == 0) return;
  SLM_REQUIRE(g.key_heads > 0 && g.heads % g.key_heads == 0, "attend: heads must be a multiple of key_heads");
  bool merged = false;
  switch (g.dh) {
    case 8: merged = launch_dh<8>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    case 16: merged = launch_dh<16>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    case 32: merged = launch_dh<32>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    case 64: merged = launch_dh<64>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    case 128: merged = launch_dh<128>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    case 256: merged = launch_dh<256>(q, ldq, K, V, g, pos_ptr, nsplit, part, cnt, y, ldy, st); break;
    default: fail(SLM_ERR_INVALID, "attend: head size must be one of 8, 16, 32, 64, 128, 256");
  }
  if (merged) return;
  combine(part, nsplit, g, y, ldy, st);
}

void attention_rows(const float* q, int ldq, const AttnRows& rows, const AttnGeom& g, int nsplit, float* part,
                    float* y, int ldy, cudaStream_t st, unsigned* cnt) {
  if (g.m == 0) return;
  SLM_REQUIRE(g.key_heads > 0 && g.heads % g.key_heads == 0, "attend: heads must be a multiple of key_heads");
  const dim3 grid(nsplit, g.heads, g.m);
#define SLM_ROWS(DHV) \
  k_attn_split<DHV><<<grid, kSplitThreads, 0, st>>>(q, ldq, nullptr, nullptr, g, nullptr, nsplit, part, rows, cnt, y, \
                                                     ldy)
  switch (g.dh) {
    case 8: SLM_ROWS(8); break;
    case 16: SLM_ROWS(16); break;
    case 32: SLM_ROWS(32); break;
    case 64: SLM_ROWS(64); break;
    case 128: SLM_ROWS(128); break;
    case 256: SLM_ROWS(256); break;
    default: fail(SLM_ERR_INVALID, "attend: head size must be one of 8, 16, 32, 64, 128, 256");
  }
#undef SLM_ROWS
  SLM_LAUNCHED("k_attn_split");
  if (cnt) return;
  combine(part, nsplit, g, y, ldy, st);
}

}  // namespace slm
