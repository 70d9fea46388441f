// Element-wise and row-wise kernels: the small `Ops` methods (reference
// src/ops.rs:93-217, arithmetic src/cpu.rs:66-350) and the fused glue the
// model step uses in their place (embedding + copy, rope + ring store,
// l2norm of q/k, the loop input, the G layer's logn scaling and key shift).
// Row reductions use one CTA per row, so results do not depend on timing.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

constexpr int EW = 256;  // threads per CTA for element-wise kernels

inline unsigned ew_grid(size_t n) {
  size_t g = (n + EW - 1) / EW;
  return (unsigned)(g < 148 * 64 ? (g == 0 ? 1 : g) : 148 * 64);
}

#define GRID_STRIDE(t, n) for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < (n); t += (size_t)gridDim.x * blockDim.x)

__global__ void k_gather(float* y, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab,
                         int* err) {
  GRID_STRIDE(t, m * d) {
    uint32_t id = ids[t / d];
    if (id >= vocab) {
      if (err) atomicOr(err, 1);
      y[t] = 0.0f;
      continue;
    }
    y[t] = w[(size_t)id * d + t % d];
  }
}

// e0 = x = embed[ids] (src/model.rs:574-575).
__global__ void k_embed(float* e0, float* x, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab,
                        int* err) {
  GRID_STRIDE(t, m * d) {
    uint32_t id = ids[t / d];
    float v = 0.0f;
    if (id < vocab)
      v = w[(size_t)id * d + t % d];
    else if (err)
      atomicOr(err, 1);
    e0[t] = v;
    x[t] = v;
  }
}

__global__ void k_copy(float* y, const float* x, size_t n) {
  GRID_STRIDE(t, n) y[t] = x[t];
}

__global__ void k_shift(float* y, const float* first, const float* x, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) y[t] = t < d ? first[t] : x[t - d];
}

__global__ void k_columns(float* y, const float* x, size_t m, size_t stride, size_t off, size_t len) {
  GRID_STRIDE(t, m * len) y[t] = x[(t / len) * stride + off + t % len];
}

__global__ void k_add(float* y, const float* a, const float* b, size_t n) {
  GRID_STRIDE(t, n) y[t] = a[t] + b[t];
}

__global__ void k_add_row(float* y, const float* x, const float* row, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) y[t] = x[t] + row[t % d];
}

__global__ void k_scale_rows(float* y, const float* x, const float* f, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) y[t] = x[t] * f[t / d];
}

__global__ void k_mix(float* y, const float* a, const float* b, size_t n, float tt) {
  GRID_STRIDE(t, n) y[t] = a[t] + tt * (b[t] - a[t]);
}

__global__ void k_silu_mul(float* y, const float* g, const float* u, size_t n) {
  GRID_STRIDE(t, n) y[t] = silu_mul(g[t], u[t]);
}

// x = (s + e_proj) + loop_embed[r] (src/model.rs:583-584).
__global__ void k_loop_in(float* x, const float* s, const float* e, const float* row, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) x[t] = (s[t] + e[t]) + row[t % d];
}

// One CTA per group: y = x·r·w with r = 1/sqrt(mean(x²) + eps)
// (src/cpu.rs:187-207); with `base`, y = base + x·r·w (the G layer's norm_e
// term, src/model.rs:497-500).
__global__ void k_rms(float* y, const float* x, const float* w, size_t size, float eps, const float* base) {
  __shared__ float red[32];
  const float* in = x + (size_t)blockIdx.x * size;
  float s = 0.0f;
  for (size_t e = threadIdx.x; e < size; e += blockDim.x) s = fmaf(in[e], in[e], s);
  s = block_sum(s, red);
  float r = 1.0f / sqrtf(s / (float)size + eps);
  float* out = y + (size_t)blockIdx.x * size;
  const float* bs = base ? base + (size_t)blockIdx.x * size : nullptr;
  for (size_t e = threadIdx.x; e < size; e += blockDim.x) {
    float v = in[e] * r * w[e];
    out[e] = bs ? bs[e] + v : v;
  }
}

// One warp per head: y = x / max(|x|, 1e-12) (src/cpu.rs:270-282).  Reads
// heads at `ldx` strides so it can take q and k straight out of the fused
// qkvg projection.
__global__ void k_l2norm(float* y, size_t ldy, const float* x, size_t ldx, size_t rows, size_t heads, size_t dh) {
  size_t t = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (t >= rows * heads) return;
  size_t i = t / heads, h = t % heads;
  const float* in = x + i * ldx + h * dh;
  float s = 0.0f;
  for (size_t e = lane; e < dh; e += 32) s = fmaf(in[e], in[e], s);
  s = warp_sum(s);
  float r = 1.0f / fmaxf(sqrtf(s), 1e-12f);
  float* out = y + i * ldy + h * dh;
  for (size_t e = lane; e < dh; e += 32) out[e] = in[e] * r;
}

__global__ void k_rope_table(float* c, float* s, const float* inv, long long pos, size_t m, size_t half) {
  GRID_STRIDE(t, m * half) {
    float a = (float)(pos + (long long)(t / half)) * inv[t % half];
    float sn, cs;
    sincosf(a, &sn, &cs);
    c[t] = cs;
    s[t] = sn;
  }
}

__global__ void k_rope(float* y, const float* x, const float* c, const float* s, size_t m, size_t heads, size_t dh) {
  size_t half = dh / 2;
  GRID_STRIDE(t, m * heads * half) {
    size_t row = t / (heads * half), hh = (t / half) % heads, i = t % half;
    const float* in = x + (row * heads + hh) * dh;
    float* out = y + (row * heads + hh) * dh;
    float cs = c[row * half + i], sn = s[row * half + i];
    float a = in[i], b = in[half + i];
    out[i] = a * cs - b * sn;
    out[half + i] = a * sn + b * cs;
  }
}

__global__ void k_store(float* cache, const float* src, size_t ldsrc, const long long* pos_ptr, long long pos,
                        size_t m, size_t cap, size_t heads, size_t dh) {
  long long p0 = pos_ptr ? pos_ptr[0] : pos;
  GRID_STRIDE(t, m * heads * dh) {
    size_t i = t / (heads * dh), hh = (t / dh) % heads, e = t % dh;
    size_t slot = (size_t)((p0 + (long long)i) % (long long)cap);
    cache[(hh * cap + slot) * dh + e] = src[i * ldsrc + hh * dh + e];
  }
}

// S mixer after its qkv projection (src/model.rs:430-438): rotate q and k by
// the angles of positions pos.. (cos/sin of (pos+i)·inv[j], the rope_table of
// src/cpu.rs:217-237, computed in place), write q to `qout` and k, v into
// ring slot (pos+i) % cap.
__global__ void k_rope_store(const float* mix, size_t ldmix, const float* inv, const long long* pos_ptr, size_t m,
                             size_t heads, size_t dh, size_t cap, float* qout, float* kc, float* vc) {
  const long long pos = pos_ptr[0];
  const size_t half = dh / 2, d = heads * dh;
  GRID_STRIDE(t, m * heads * half) {
    size_t i = t / (heads * half), hh = (t / half) % heads, j = t % half;
    float a = (float)(pos + (long long)i) * inv[j];
    float sn, cs;
    sincosf(a, &sn, &cs);
    const float* row = mix + i * ldmix;
    size_t slot = (size_t)((pos + (long long)i) % (long long)cap);
    float qa = row[hh * dh + j], qb = row[hh * dh + half + j];
    float* qo = qout + i * d + hh * dh;
    qo[j] = qa * cs - qb * sn;
    qo[half + j] = qa * sn + qb * cs;
    float ka = row[d + hh * dh + j], kb = row[d + hh * dh + half + j];
    float* ko = kc + (hh * cap + slot) * dh;
    ko[j] = ka * cs - kb * sn;
    ko[half + j] = ka * sn + kb * cs;
    float* vo = vc + (hh * cap + slot) * dh;
    vo[j] = row[2 * d + hh * dh + j];
    vo[half + j] = row[2 * d + hh * dh + half + j];
  }
}

// G mixer after its projections (src/model.rs:505-524): scale q rows by
// ln(1+p)/ln(logn) when logn != 0, and store keys/values at slot p (the
// global cache never wraps: cap ≥ pos + m).
__global__ void k_g_post(float* q, size_t d, size_t m, const long long* pos_ptr, float inv_log, int logn,
                         const float* keys, size_t ldk, const float* vals, size_t ldv, size_t kd, size_t cap,
                         size_t dh, float* kc, float* vc) {
  const long long pos = pos_ptr[0];
  GRID_STRIDE(t, m * d) {
    size_t i = t / d;
    if (logn) q[t] = q[t] * (log1pf((float)(pos + (long long)i)) * inv_log);
  }
  GRID_STRIDE(t, m * kd) {
    size_t i = t / kd, c = t % kd, hh = c / dh, e = c % dh;
    size_t slot = (size_t)(pos + (long long)i) % cap;
    kc[(hh * cap + slot) * dh + e] = keys[i * ldk + c];
    vc[(hh * cap + slot) * dh + e] = vals[i * ldv + c];
  }
}

// mid[i][j] = silu(up[i][j])·up[i][F + j]: the MLP gate on a [m][2F] product.
__global__ void k_silu_pair(float* mid, const float* up, size_t m, size_t F) {
  GRID_STRIDE(t, m * F) {
    size_t i = t / F, j = t % F;
    mid[t] = silu_mul(up[i * 2 * F + j], up[i * 2 * F + F + j]);
  }
}

// kc[h][pos + off][:] = src[h·dh …] for every cache head (one row per head).
__global__ void k_store_next(float* kc, const float* src, const long long* pos_ptr, long long off, size_t kh,
                             size_t dh, size_t cap) {
  const size_t slot = (size_t)(pos_ptr[0] + off);
  GRID_STRIDE(t, kh * dh) {
    const size_t h = t / dh, e = t % dh;
    if (slot < cap) kc[(h * cap + slot) * dh + e] = src[t];
  }
}

__global__ void k_advance_pos(long long* pos, long long m) {
  if (threadIdx.x == 0 && blockIdx.x == 0) pos[0] += m;
}

// Batched decode: row i is one token of its own sequence, at *pos[i], with
// its own ring caches k[i] / v[i] (same arithmetic as k_rope_store).
__global__ void k_rope_store_rows(const float* mix, size_t ldmix, const float* inv, long long* const* posr, size_t m,
                                  size_t heads, size_t dh, size_t cap, float* qout, float* const* kr,
                                  float* const* vr) {
  const size_t half = dh / 2, d = heads * dh;
  GRID_STRIDE(t, m * heads * half) {
    size_t i = t / (heads * half), hh = (t / half) % heads, j = t % half;
    const long long pos = *posr[i];
    float a = (float)pos * inv[j];
    float sn, cs;
    sincosf(a, &sn, &cs);
    const float* row = mix + i * ldmix;
    size_t slot = (size_t)(pos % (long long)cap);
    float qa = row[hh * dh + j], qb = row[hh * dh + half + j];
    float* qo = qout + i * d + hh * dh;
    qo[j] = qa * cs - qb * sn;
    qo[half + j] = qa * sn + qb * cs;
    float ka = row[d + hh * dh + j], kb = row[d + hh * dh + half + j];
    float* ko = kr[i] + (hh * cap + slot) * dh;
    ko[j] = ka * cs - kb * sn;
    ko[half + j] = ka * sn + kb * cs;
    float* vo = vr[i] + (hh * cap + slot) * dh;
    vo[j] = row[2 * d + hh * dh + j];
    vo[half + j] = row[2 * d + hh * dh + half + j];
  }
}

// Batched global layers: row i belongs to its own session (position *posr[i],
// caches kr[i] / vr[i] of capr[i] slots per head, previous input prev[i]).
__global__ void k_gather_rows(float* dst, float* const* src, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) dst[t] = src[t / d][t % d];
}
__global__ void k_scatter_rows(float* const* dst, const float* src, size_t m, size_t d) {
  GRID_STRIDE(t, m * d) dst[t / d][t % d] = src[t];
}
// As k_g_post, per row: q scaled by log1p(pos_i)/ln(logn), key and value
// stored at slot pos_i of row i's cache (global caches never wrap).
__global__ void k_g_post_rows(float* q, size_t d, size_t m, long long* const* posr, float inv_log, int logn,
                              const float* keys, size_t ldk, const float* vals, size_t ldv, size_t kd, size_t dh,
                              float* const* kr, float* const* vr, const long long* capr) {
  GRID_STRIDE(t, m * d) {
    const size_t i = t / d;
    if (logn) q[t] = q[t] * (log1pf((float)(*posr[i])) * inv_log);
  }
  GRID_STRIDE(t, m * kd) {
    const size_t i = t / kd, c = t % kd, hh = c / dh, e = c % dh;
    const size_t cap = (size_t)capr[i], slot = (size_t)(*posr[i]);
    if (slot >= cap) continue;
    kr[i][(hh * cap + slot) * dh + e] = keys[i * ldk + c];
    vr[i][(hh * cap + slot) * dh + e] = vals[i * ldv + c];
  }
}
// kr[i][h][*posr[i] + off] = src[i][h·dh …], skipped past row i's capacity.
__global__ void k_store_next_rows(float* const* kr, const float* src, long long* const* posr, long long off,
                                  size_t m, size_t kh, size_t dh, const long long* capr) {
  GRID_STRIDE(t, m * kh * dh) {
    const size_t i = t / (kh * dh), c = t % (kh * dh), h = c / dh, e = c % dh;
    const size_t cap = (size_t)capr[i], slot = (size_t)(*posr[i] + off);
    if (slot < cap) kr[i][(h * cap + slot) * dh + e] = src[t];
  }
}

__global__ void k_advance_rows(long long* const* posr, size_t m, unsigned* counter) {
  for (size_t i = threadIdx.x; i < m; i += blockDim.x) *posr[i] += 1;
  if (counter && threadIdx.x == 0) *counter += 1;
}

}  // namespace

void ew_gather(float* y, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab, int* err,
               cudaStream_t st) {
  k_gather<<<ew_grid(m * d), EW, 0, st>>>(y, w, ids, m, d, vocab, err);
  SLM_LAUNCHED("k_gather");
}
void ew_embed(float* e0, float* x, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab, int* err,
              cudaStream_t st) {
  k_embed<<<ew_grid(m * d), EW, 0, st>>>(e0, x, w, ids, m, d, vocab, err);
  SLM_LAUNCHED("k_embed");
}
void ew_copy(float* y, const float* x, size_t n, cudaStream_t st) {
  if (!n) return;
  k_copy<<<ew_grid(n), EW, 0, st>>>(y, x, n);
  SLM_LAUNCHED("k_copy");
}
void ew_shift(float* y, const float* first, const float* x, size_t m, size_t d, cudaStream_t st) {
  if (!m) return;
  k_shift<<<ew_grid(m * d), EW, 0, st>>>(y, first, x, m, d);
  SLM_LAUNCHED("k_shift");
}
void ew_columns(float* y, const float* x, size_t m, size_t stride, size_t off, size_t len, cudaStream_t st) {
  if (!m || !len) return;
  k_columns<<<ew_grid(m * len), EW, 0, st>>>(y, x, m, stride, off, len);
  SLM_LAUNCHED("k_columns");
}
void ew_add(float* y, const float* a, const float* b, size_t n, cudaStream_t st) {
  if (!n) return;
  k_add<<<ew_grid(n), EW, 0, st>>>(y, a, b, n);
  SLM_LAUNCHED("k_add");
}
void ew_add_row(float* y, const float* x, const float* row, size_t m, size_t d, cudaStream_t st) {
  if (!m) return;
  k_add_row<<<ew_grid(m * d), EW, 0, st>>>(y, x, row, m, d);
  SLM_LAUNCHED("k_add_row");
}
void ew_scale_rows(float* y, const float* x, const float* f, size_t m, size_t d, cudaStream_t st) {
  if (!m) return;
  k_scale_rows<<<ew_grid(m * d), EW, 0, st>>>(y, x, f, m, d);
  SLM_LAUNCHED("k_scale_rows");
}
// dst[c][r] = src[r][c] through a 32 × 33 shared tile (coalesced both ways).
__global__ void k_transpose(float* __restrict__ dst, const float* __restrict__ src, int rows, int cols) {
  __shared__ float t[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int r = r0 + j, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[j][threadIdx.x] = src[(size_t)r * cols + c];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int c = c0 + j, r = r0 + threadIdx.x;
    if (c < cols && r < rows) dst[(size_t)c * rows + r] = t[threadIdx.x][j];
  }
}

// dst[h][r][c] = src[r][h·dh + c]: the column blocks of a [rows][heads·dh]
// matrix, each contiguous.
__global__ void k_head_blocks(float* __restrict__ dst, const float* __restrict__ src, size_t rows, int heads, int dh) {
  const size_t cols = (size_t)heads * dh, n = rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, k = i % cols, h = k / dh, c = k % dh;
    dst[(h * rows + r) * dh + c] = src[i];
  }
}

void ew_head_blocks(float* dst, const float* src, size_t rows, size_t heads, size_t dh, cudaStream_t st) {
  if (!rows || !heads || !dh) return;
  k_head_blocks<<<ew_grid(rows * heads * dh), EW, 0, st>>>(dst, src, rows, (int)heads, (int)dh);
  SLM_LAUNCHED("k_head_blocks");
}

namespace {
__global__ void k_to_bf16(__nv_bfloat16* dst, const float* src, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}
}  // namespace

void ew_to_bf16(void* dst, const float* src, size_t n, cudaStream_t st) {
  if (!n) return;
  k_to_bf16<<<ew_grid(n), EW, 0, st>>>(static_cast<__nv_bfloat16*>(dst), src, n);
  SLM_LAUNCHED("k_to_bf16");
}

void ew_transpose(float* dst, const float* src, size_t rows, size_t cols, cudaStream_t st) {
  if (!rows || !cols) return;
  SLM_REQUIRE(rows <= (size_t)65535 * 32 && cols < (size_t)1 << 31, "matrix too large to transpose");
  k_transpose<<<dim3((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32)), dim3(32, 8), 0, st>>>(
      dst, src, (int)rows, (int)cols);
  SLM_LAUNCHED("k_transpose");
}

void ew_mix(float* y, const float* a, const float* b, size_t n, float t, cudaStream_t st) {
  if (!n) return;
  k_mix<<<ew_grid(n), EW, 0, st>>>(y, a, b, n, t);
  SLM_LAUNCHED("k_mix");
}
void ew_silu_mul(float* y, const float* g, const float* u, size_t n, cudaStream_t st) {
  if (!n) return;
  k_silu_mul<<<ew_grid(n), EW, 0, st>>>(y, g, u, n);
  SLM_LAUNCHED("k_silu_mul");
}
void ew_loop_in(float* x, const float* s, const float* e, const float* row, size_t m, size_t d, cudaStream_t st) {
  k_loop_in<<<ew_grid(m * d), EW, 0, st>>>(x, s, e, row, m, d);
  SLM_LAUNCHED("k_loop_in");
}
void ew_rms(float* y, const float* x, const float* w, size_t groups, size_t size, float eps, const float* base,
            cudaStream_t st) {
  if (!groups) return;
  unsigned threads = size >= 256 ? 256 : (unsigned)(32 * cdiv(size, 32));
  k_rms<<<(unsigned)groups, threads, 0, st>>>(y, x, w, size, eps, base);
  SLM_LAUNCHED("k_rms");
}
void ew_l2norm(float* y, size_t ldy, const float* x, size_t ldx, size_t rows, size_t heads, size_t dh,
               cudaStream_t st) {
  size_t warps = rows * heads;
  if (!warps) return;
  k_l2norm<<<cdiv(warps, 8), 256, 0, st>>>(y, ldy, x, ldx, rows, heads, dh);
  SLM_LAUNCHED("k_l2norm");
}
void ew_rope_table(float* c, float* s, const float* inv, long long pos, size_t m, size_t half, cudaStream_t st) {
  if (!m || !half) return;
  k_rope_table<<<ew_grid(m * half), EW, 0, st>>>(c, s, inv, pos, m, half);
  SLM_LAUNCHED("k_rope_table");
}
void ew_rope(float* y, const float* x, const float* c, const float* s, size_t m, size_t heads, size_t dh,
             cudaStream_t st) {
  if (!m) return;
  k_rope<<<ew_grid(m * heads * (dh / 2)), EW, 0, st>>>(y, x, c, s, m, heads, dh);
  SLM_LAUNCHED("k_rope");
}
void ew_store(float* cache, const float* src, size_t ldsrc, const long long* pos_ptr, long long pos, size_t m,
              size_t cap, size_t heads, size_t dh, cudaStream_t st) {
  if (!m) return;
  k_store<<<ew_grid(m * heads * dh), EW, 0, st>>>(cache, src, ldsrc, pos_ptr, pos, m, cap, heads, dh);
  SLM_LAUNCHED("k_store");
}
void ew_rope_store(const float* mix, size_t ldmix, const float* inv, const long long* pos_ptr, size_t m,
                   size_t heads, size_t dh, size_t cap, float* qout, float* kc, float* vc, cudaStream_t st) {
  k_rope_store<<<ew_grid(m * heads * (dh / 2)), EW, 0, st>>>(mix, ldmix, inv, pos_ptr, m, heads, dh, cap, qout, kc,
                                                            vc);
  SLM_LAUNCHED("k_rope_store");
}
void ew_g_post(float* q, size_t d, size_t m, const long long* pos_ptr, float inv_log, int logn, const float* keys,
               size_t ldk, const float* vals, size_t ldv, size_t kd, size_t cap, size_t dh, float* kc, float* vc,
               cudaStream_t st) {
  k_g_post<<<ew_grid(m * d), EW, 0, st>>>(q, d, m, pos_ptr, inv_log, logn, keys, ldk, vals, ldv, kd, cap, dh, kc,
                                          vc);
  SLM_LAUNCHED("k_g_post");
}
void ew_silu_pair(float* mid, const float* up, size_t m, size_t F, cudaStream_t st) {
  if (!m) return;
  k_silu_pair<<<ew_grid(m * F), EW, 0, st>>>(mid, up, m, F);
  SLM_LAUNCHED("k_silu_pair");
}
void ew_store_next(float* kc, const float* src, const long long* pos_ptr, long long off, size_t kh, size_t dh,
                   size_t cap, cudaStream_t st) {
  k_store_next<<<ew_grid(kh * dh), EW, 0, st>>>(kc, src, pos_ptr, off, kh, dh, cap);
  SLM_LAUNCHED("k_store_next");
}
void ew_advance_pos(long long* pos, long long m, cudaStream_t st) {
  k_advance_pos<<<1, 32, 0, st>>>(pos, m);
  SLM_LAUNCHED("k_advance_pos");
}
void ew_rope_store_rows(const float* mix, size_t ldmix, const float* inv, long long* const* posr, size_t m,
                        size_t heads, size_t dh, size_t cap, float* qout, float* const* kr, float* const* vr,
                        cudaStream_t st) {
  if (!m) return;
  k_rope_store_rows<<<ew_grid(m * heads * (dh / 2)), EW, 0, st>>>(mix, ldmix, inv, posr, m, heads, dh, cap, qout,
                                                                  kr, vr);
  SLM_LAUNCHED("k_rope_store_rows");
}
void ew_gather_rows(float* dst, float* const* src, size_t m, size_t d, cudaStream_t st) {
  if (!m) return;
  k_gather_rows<<<ew_grid(m * d), EW, 0, st>>>(dst, src, m, d);
  SLM_LAUNCHED("k_gather_rows");
}
void ew_scatter_rows(float* const* dst, const float* src, size_t m, size_t d, cudaStream_t st) {
  if (!m) return;
  k_scatter_rows<<<ew_grid(m * d), EW, 0, st>>>(dst, src, m, d);
  SLM_LAUNCHED("k_scatter_rows");
}
void ew_g_post_rows(float* q, size_t d, size_t m, long long* const* posr, float inv_log, int logn, const float* keys,
                    size_t ldk, const float* vals, size_t ldv, size_t kd, size_t dh, float* const* kr,
                    float* const* vr, const long long* capr, cudaStream_t st) {
  if (!m) return;
  k_g_post_rows<<<ew_grid(m * d), EW, 0, st>>>(q, d, m, posr, inv_log, logn, keys, ldk, vals, ldv, kd, dh, kr, vr,
                                               capr);
  SLM_LAUNCHED("k_g_post_rows");
}
void ew_store_next_rows(float* const* kr, const float* src, long long* const* posr, long long off, size_t m, size_t kh,
                        size_t dh, const long long* capr, cudaStream_t st) {
  if (!m) return;
  k_store_next_rows<<<ew_grid(m * kh * dh), EW, 0, st>>>(kr, src, posr, off, m, kh, dh, capr);
  SLM_LAUNCHED("k_store_next_rows");
}
void ew_advance_rows(long long* const* posr, size_t m, unsigned* counter, cudaStream_t st) {
  k_advance_rows<<<1, 256, 0, st>>>(posr, m, counter);
  SLM_LAUNCHED("k_advance_rows");
}

}  // namespace slm
