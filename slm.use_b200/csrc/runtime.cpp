// Contexts, buffers and the op-level C ABI: one entry point per method of the
// reference's `Ops` trait (src/ops.rs:68-228), each a thin check of sizes and
// offsets around the sm_100a kernels.  Outputs that are too small grow, as the
// reference CUDA backend's `ensure` does (src/cuda.rs:122-127); calls queue on
// the context's stream and slm_read waits (src/cuda.rs:160-165).
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "capi.hpp"
#include "common.cuh"
#include "kernels.cuh"

namespace slm {

thread_local std::string g_last_error;

void set_error(const std::string& s) { g_last_error = s; }

void disarm(slm_ctx* c) {
  if (!c->armed) return;
  *(volatile unsigned long long*)(c->mbox + 8) = (c->armed_seq << 32) | 0xffffffffull;
  c->armed = false;
  c->armed_owner = nullptr;
}

Device::Device(slm_ctx* c, bool keep_armed) : prev(-1) {
  if (!keep_armed) disarm(c);
  cudaGetDevice(&prev);
  if (prev != c->device) SLM_CUDA(cudaSetDevice(c->device));
}
Device::~Device() {
  if (prev >= 0) cudaSetDevice(prev);
}

void* dev_alloc(size_t bytes) {
  void* p = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(SLM_ERR_NOMEM, "cudaMalloc of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
  }
  return p;
}

void dev_free(void* p) {
  if (p) cudaFree(p);
}

void ensure(slm_buf* y, size_t n) {
  SLM_REQUIRE(y != nullptr, "output buffer is null");
  if (y->len >= n) return;
  Device dev(y->ctx);
  SLM_CUDA(cudaStreamSynchronize(y->ctx->stream));  // the old storage may still be in use
  float* p = static_cast<float*>(dev_alloc(n * sizeof(float)));
  SLM_CUDA(cudaMemsetAsync(p, 0, n * sizeof(float), y->ctx->stream));
  dev_free(y->ptr);
  y->ptr = p;
  y->len = n;
}

const float* view(const slm_buf* b, size_t off, size_t n, const char* what) {
  SLM_REQUIRE(b != nullptr, std::string(what) + ": buffer is null");
  SLM_REQUIRE(off <= b->len && n <= b->len - off,
              std::string(what) + ": reads " + std::to_string(off) + "+" + std::to_string(n) + " of a buffer of " +
                  std::to_string(b->len));
  return b->ptr + off;
}

// Host arrays staged into a context-owned device buffer (ids, factors).
void* stage(slm_ctx* c, const void* host, size_t bytes) {
  if (c->stage_bytes < bytes) {
    SLM_CUDA(cudaStreamSynchronize(c->stream));
    dev_free(c->stage);
    c->stage = dev_alloc(bytes);
    c->stage_bytes = bytes;
  }
  // Pageable source: the runtime copies it before returning, so `host` may go.
  SLM_CUDA(cudaMemcpyAsync(c->stage, host, bytes, cudaMemcpyHostToDevice, c->stream));
  return c->stage;
}

void gemm_workspace(slm_ctx* c, LinearArgs& a, bool capturing) {
  const bool b3 = b3_linear_ok(a), skinny = !b3 && skinny_ok(a), tc = !skinny && !b3 && a.m > 64 && tc_linear_ok(a);
  const bool gemv = !b3 && !skinny && !tc && a.m <= 8;
  if (skinny || b3 || tc || gemv) {
    const size_t need = skinny ? skinny_workspace(a)
                        : b3   ? b3_linear_workspace(a)
                        : tc   ? tc_linear_workspace(a)
                               : gemv_workspace(a);
    if (need > c->gemm_ws_bytes && !capturing) {
      SLM_CUDA(cudaStreamSynchronize(c->stream));
      dev_free(c->gemm_ws);
      c->gemm_ws = nullptr;
      c->gemm_ws_bytes = 0;
      c->gemm_ws = dev_alloc(need);
      c->gemm_ws_bytes = need;
      c->gemm_ws_gen++;
    }
  }
  a.ws = c->gemm_ws;
  a.ws_bytes = c->gemm_ws_bytes;
  a.cnt = c->gemv_cnt;
}

}  // namespace slm

using namespace slm;

namespace {
void destroy_ctx(slm_ctx* c) {
  {
    Device dev(c);
    cudaStreamSynchronize(c->stream);
    dev_free(c->stage);
    dev_free(c->gemm_ws);
    dev_free(c->merge_cnt);
    dev_free(c->gemv_cnt);
    dev_free(c->err);
    if (c->err_host) cudaFreeHost(c->err_host);
    if (c->mbox) cudaFreeHost(c->mbox);
    cudaStreamDestroy(c->stream);
  }
  delete c;
}
}  // namespace

namespace slm {
void ctx_retain(slm_ctx* c) { c->refs++; }
void ctx_release(slm_ctx* c) {
  if (--c->refs == 0 && c->closing) destroy_ctx(c);
}
}  // namespace slm

extern "C" {

const char* slm_last_error(void) { return g_last_error.c_str(); }
const char* slm_version(void) { return "slm-b200 0.1 (sm_100a)"; }

int slm_device_count(int* out) {
  return guard([&] {
    SLM_REQUIRE(out, "out is null");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *out = n;
  });
}

int slm_ctx_new(int device, slm_ctx** out) {
  return guard([&] {
    SLM_REQUIRE(out, "out is null");
    int n = 0;
    SLM_CUDA(cudaGetDeviceCount(&n));
    SLM_REQUIRE(device >= 0 && device < n, "no CUDA device " + std::to_string(device));
    cudaDeviceProp prop;
    SLM_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) fail(SLM_ERR_CUDA, std::string("built for sm_100a; device is ") + prop.name);
    auto* c = new slm_ctx();
    c->device = device;
    c->name = prop.name;
    c->sms = prop.multiProcessorCount;
    try {
      Device dev(c);
      SLM_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
      linear_prepare();
      c->err = static_cast<int*>(dev_alloc(sizeof(int) * 4));
      SLM_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int) * 4, c->stream));
      SLM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&c->err_host), sizeof(int) * 4, cudaHostAllocDefault));
      c->gemv_cnt = static_cast<unsigned*>(dev_alloc(kGemvCounters * sizeof(unsigned)));
      SLM_CUDA(cudaMemsetAsync(c->gemv_cnt, 0, kGemvCounters * sizeof(unsigned), c->stream));
      SLM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&c->mbox), 128, cudaHostAllocMapped));
      for (int i = 0; i < 16; i++) c->mbox[i] = 0;
      SLM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->mbox_dev), c->mbox, 0));
    } catch (...) {
      delete c;
      throw;
    }
    *out = c;
  });
}

int slm_ctx_free(slm_ctx* c) {
  return guard([&] {
    if (!c || c->closing) return;
    if (c->refs > 0) {  // buffers or models still live: the last of them frees the context
      c->closing = true;
      return;
    }
    destroy_ctx(c);
  });
}

int slm_ctx_name(slm_ctx* c, char* out, size_t cap) {
  return guard([&] {
    SLM_REQUIRE(c && out && cap, "bad arguments");
    std::string n = "b200 (" + c->name + ")";
    std::strncpy(out, n.c_str(), cap - 1);
    out[cap - 1] = 0;
  });
}

int slm_ctx_sync(slm_ctx* c) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    SLM_CUDA(cudaStreamSynchronize(c->stream));
  });
}

int slm_ctx_stream(slm_ctx* c, void** out) {
  return guard([&] {
    SLM_REQUIRE(c && out, "bad arguments");
    *out = (void*)c->stream;
  });
}

int slm_zeros(slm_ctx* c, size_t n, slm_buf** out) {
  return guard([&] {
    SLM_REQUIRE(c && out, "bad arguments");
    Device dev(c);
    auto* b = new slm_buf{c, nullptr, 0};
    ctx_retain(c);
    try {
      size_t len = n ? n : 1;  // zeros(n.max(1)), src/cuda.rs:152-154
      b->ptr = static_cast<float*>(dev_alloc(len * sizeof(float)));
      b->len = len;
      SLM_CUDA(cudaMemsetAsync(b->ptr, 0, len * sizeof(float), c->stream));
    } catch (...) {
      delete b;
      c->refs--;
      throw;
    }
    *out = b;
  });
}

int slm_upload(slm_ctx* c, const float* data, size_t n, slm_buf** out) {
  return guard([&] {
    SLM_REQUIRE(c && out && (data || n == 0), "bad arguments");
    Device dev(c);
    auto* b = new slm_buf{c, nullptr, 0};
    ctx_retain(c);
    try {
      b->ptr = static_cast<float*>(dev_alloc((n ? n : 1) * sizeof(float)));
      b->len = n ? n : 1;
      if (n) SLM_CUDA(cudaMemcpyAsync(b->ptr, data, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
      SLM_CUDA(cudaStreamSynchronize(c->stream));
    } catch (...) {
      dev_free(b->ptr);
      delete b;
      c->refs--;
      throw;
    }
    *out = b;
  });
}

int slm_read(slm_ctx* c, const slm_buf* b, size_t n, float* out) {
  return guard([&] {
    SLM_REQUIRE(c && b && (out || n == 0), "bad arguments");
    SLM_REQUIRE(n <= b->len, "read past the end of the buffer");
    Device dev(c);
    if (n) SLM_CUDA(cudaMemcpyAsync(out, b->ptr, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    SLM_CUDA(cudaStreamSynchronize(c->stream));
  });
}

int slm_buf_free(slm_buf* b) {
  return guard([&] {
    if (!b) return;
    slm_ctx* c = b->ctx;
    {
      Device dev(c);
      cudaStreamSynchronize(c->stream);
      dev_free(b->ptr);
    }
    delete b;
    ctx_release(c);
  });
}

size_t slm_buf_len(const slm_buf* b) { return b ? b->len : 0; }
float* slm_buf_ptr(slm_buf* b) { return b ? b->ptr : nullptr; }

int slm_flush(slm_ctx* c) {
  return guard([&] { SLM_REQUIRE(c, "ctx is null"); });
}

// ---------------------------------------------------------------------------
// Op level
// ---------------------------------------------------------------------------

int slm_op_gather(slm_ctx* c, slm_buf* y, const slm_buf* w, const uint32_t* ids, size_t m, size_t d) {
  return guard([&] {
    SLM_REQUIRE(c && w && (ids || m == 0) && d > 0, "gather: bad arguments");
    Device dev(c);
    size_t vocab = w->len / d;
    for (size_t i = 0; i < m; i++) SLM_REQUIRE(ids[i] < vocab, "gather: id out of range");
    ensure(y, m * d);
    if (!m) return;
    auto* dids = static_cast<const uint32_t*>(stage(c, ids, m * sizeof(uint32_t)));
    ew_gather(y->ptr, w->ptr, dids, m, d, vocab, c->err, c->stream);
  });
}

int slm_op_copy(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, size_t n) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* xs = view(x, xoff, n, "copy");
    ensure(y, n);
    ew_copy(y->ptr, xs, n, c->stream);
  });
}

int slm_op_shift(slm_ctx* c, slm_buf* y, const slm_buf* first, const slm_buf* x, size_t xoff, size_t m, size_t d) {
  return guard([&] {
    SLM_REQUIRE(c && m > 0, "shift: bad arguments");
    Device dev(c);
    const float* f = view(first, 0, d, "shift first");
    const float* xs = view(x, xoff, (m - 1) * d, "shift");
    ensure(y, m * d);
    ew_shift(y->ptr, f, xs, m, d, c->stream);
  });
}

int slm_op_columns(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t m, size_t stride, size_t off, size_t len) {
  return guard([&] {
    SLM_REQUIRE(c && off + len <= stride, "columns: bad arguments");
    Device dev(c);
    const float* xs = view(x, 0, m ? (m - 1) * stride + off + len : 0, "columns");
    ensure(y, m * len);
    ew_columns(y->ptr, xs, m, stride, off, len, c->stream);
  });
}

int slm_op_linear(slm_ctx* c, slm_buf* y, const slm_buf* w, size_t rows, size_t cols, const slm_buf* x, size_t xoff,
                  size_t m) {
  return guard([&] {
    SLM_REQUIRE(c && rows > 0 && cols > 0, "linear: bad arguments");
    SLM_REQUIRE(rows < (1u << 31) && cols < (1u << 31) && m < (1u << 31), "linear: shape too large");
    Device dev(c);
    const float* ws = view(w, 0, rows * cols, "linear weight");
    const float* xs = view(x, xoff, m * cols, "linear input");
    ensure(y, m * rows);
    LinearArgs a;
    a.w = ws, a.rows = (int)rows, a.cols = (int)cols, a.x = xs, a.ldx = (int)cols, a.m = (int)m;
    a.y = y->ptr, a.ldy = (int)rows, a.epi = EPI_STORE;
    gemm_workspace(c, a, false);
    linear(a, c->stream);
  });
}

int slm_op_add(slm_ctx* c, slm_buf* y, const slm_buf* a, size_t aoff, const slm_buf* b, size_t boff, size_t n) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* as = view(a, aoff, n, "add a");
    const float* bs = view(b, boff, n, "add b");
    ensure(y, n);
    ew_add(y->ptr, as, bs, n, c->stream);
  });
}

int slm_op_add_row(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* row, size_t rowoff, size_t m,
                   size_t d) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* xs = view(x, xoff, m * d, "add_row x");
    const float* rs = view(row, rowoff, d, "add_row row");
    ensure(y, m * d);
    ew_add_row(y->ptr, xs, rs, m, d, c->stream);
  });
}

int slm_op_scale_rows(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, const float* f, size_t m, size_t d) {
  return guard([&] {
    SLM_REQUIRE(c && (f || m == 0), "scale_rows: bad arguments");
    Device dev(c);
    const float* xs = view(x, xoff, m * d, "scale_rows");
    ensure(y, m * d);
    if (!m) return;
    auto* df = static_cast<const float*>(stage(c, f, m * sizeof(float)));
    ew_scale_rows(y->ptr, xs, df, m, d, c->stream);
  });
}

int slm_op_mix(slm_ctx* c, slm_buf* y, const slm_buf* a, size_t aoff, const slm_buf* b, size_t boff, size_t n,
               float t) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* as = view(a, aoff, n, "mix a");
    const float* bs = view(b, boff, n, "mix b");
    ensure(y, n);
    ew_mix(y->ptr, as, bs, n, t, c->stream);
  });
}

int slm_op_rms(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* w, size_t groups, size_t size,
               float eps) {
  return guard([&] {
    SLM_REQUIRE(c && size > 0, "rms: bad arguments");
    Device dev(c);
    const float* xs = view(x, xoff, groups * size, "rms x");
    const float* ws = view(w, 0, size, "rms weight");
    ensure(y, groups * size);
    ew_rms(y->ptr, xs, ws, groups, size, eps, nullptr, c->stream);
  });
}

int slm_op_silu_mul(slm_ctx* c, slm_buf* y, const slm_buf* g, size_t goff, const slm_buf* u, size_t uoff, size_t n) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* gs = view(g, goff, n, "silu_mul g");
    const float* us = view(u, uoff, n, "silu_mul u");
    ensure(y, n);
    ew_silu_mul(y->ptr, gs, us, n, c->stream);
  });
}

int slm_op_rope_table(slm_ctx* c, slm_buf* cos_out, slm_buf* sin_out, const slm_buf* inv, size_t pos, size_t m,
                      size_t half) {
  return guard([&] {
    SLM_REQUIRE(c, "ctx is null");
    Device dev(c);
    const float* is = view(inv, 0, half, "rope_table inv");
    ensure(cos_out, m * half);
    ensure(sin_out, m * half);
    ew_rope_table(cos_out->ptr, sin_out->ptr, is, (long long)pos, m, half, c->stream);
  });
}

int slm_op_rope(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* cos_in, const slm_buf* sin_in,
                size_t m, size_t heads, size_t dh) {
  return guard([&] {
    SLM_REQUIRE(c && dh % 2 == 0, "rope: bad arguments");
    Device dev(c);
    const float* xs = view(x, xoff, m * heads * dh, "rope x");
    const float* cs = view(cos_in, 0, m * dh / 2, "rope cos");
    const float* ss = view(sin_in, 0, m * dh / 2, "rope sin");
    ensure(y, m * heads * dh);
    ew_rope(y->ptr, xs, cs, ss, m, heads, dh, c->stream);
  });
}

int slm_op_l2norm(slm_ctx* c, slm_buf* y, const slm_buf* x, size_t xoff, size_t heads, size_t dh) {
  return guard([&] {
    SLM_REQUIRE(c && dh > 0, "l2norm: bad arguments");
    Device dev(c);
    const float* xs = view(x, xoff, heads * dh, "l2norm");
    ensure(y, heads * dh);
    ew_l2norm(y->ptr, dh, xs, dh, heads, 1, dh, c->stream);
  });
}

int slm_op_gla(slm_ctx* c, slm_buf* y, slm_buf* s, const slm_buf* q, size_t qoff, const slm_buf* k, size_t koff,
               const slm_buf* v, size_t voff, const slm_buf* decay, const slm_buf* bias, size_t m, size_t heads,
               size_t dh) {
  return guard([&] {
    SLM_REQUIRE(c && s, "gla: bad arguments");
    Device dev(c);
    size_t n = m * heads * dh;
    GlaArgs a{};
    a.q = view(q, qoff, n, "gla q");
    a.k = view(k, koff, n, "gla k");
    a.v = view(v, voff, n, "gla v");
    a.dec = view(decay, 0, m * heads, "gla decay");
    a.bias = view(bias, 0, heads, "gla bias");
    view(s, 0, heads * dh * dh, "gla state");
    ensure(y, n);
    a.S = s->ptr;
    a.ldq = a.ldk = a.ldv = (int)(heads * dh);
    a.g = nullptr, a.ldg = 0, a.hnw = nullptr, a.eps = 0.0f;
    a.lddec = (int)heads;
    a.m = (int)m, a.heads = (int)heads, a.dh = (int)dh;
    a.out = y->ptr, a.ldo = (int)(heads * dh), a.fuse = 0;
    gla(a, c->stream);
  });
}

int slm_op_store(slm_ctx* c, slm_buf* cache, const slm_buf* src, size_t srcoff, size_t pos, size_t m, size_t cap,
                 size_t heads, size_t dh) {
  return guard([&] {
    SLM_REQUIRE(c && cap > 0, "store: bad arguments");
    Device dev(c);
    const float* ss = view(src, srcoff, m * heads * dh, "store src");
    view(cache, 0, heads * cap * dh, "store cache");
    ew_store(cache->ptr, ss, heads * dh, nullptr, (long long)pos, m, cap, heads, dh, c->stream);
  });
}

int slm_op_attend(slm_ctx* c, slm_buf* y, slm_buf* scores, const slm_buf* q, size_t qoff, const slm_buf* k,
                  const slm_buf* v, const slm_attn* at) {
  return guard([&] {
    SLM_REQUIRE(c && at && scores, "attend: bad arguments");
    SLM_REQUIRE(at->dh <= 256, "attend: head size above 256");  // src/cuda.rs:432-434
    SLM_REQUIRE(at->key_heads > 0 && at->heads % at->key_heads == 0 && at->cap > 0 && at->reach > 0,
                "attend: bad geometry");
    Device dev(c);
    const float* qs = view(q, qoff, at->m * at->heads * at->dh, "attend q");
    view(k, 0, at->key_heads * at->cap * at->dh, "attend k");
    view(v, 0, at->key_heads * at->cap * at->dh, "attend v");
    ensure(y, at->m * at->heads * at->dh);
    if (!at->m) return;
    AttnGeom g;
    g.m = (int)at->m;
    g.reach = at->reach == SIZE_MAX ? 0 : (long long)at->reach;
    g.gap = (long long)at->gap, g.cap = (long long)at->cap;
    g.heads = (int)at->heads, g.key_heads = (int)at->key_heads, g.dh = (int)at->dh, g.scale = at->scale;
    g.err = c->err;
    // Span of positions any query sees (Attn::span, src/ops.rs:54-59).
    long long base = g.reach == 0 ? 0 : ((long long)at->pos > g.reach - 1 ? (long long)at->pos - (g.reach - 1) : 0);
    long long span = (long long)(at->pos + at->m) - g.gap - base;
    int nsplit = attn_splits(g, span < 1 ? 1 : span);
    long long pos = (long long)at->pos;
    // Scratch: two leading floats (unused), the partials, and room for q when
    // the view is not 16-byte aligned (the kernels read q in 16-byte vectors).
    const size_t parts = attn_part_floats(g, nsplit), nq = at->m * at->heads * at->dh;
    const bool copy_q = ((uintptr_t)qs & 15) != 0;
    const size_t qat = (2 + parts + 3) / 4 * 4;  // 16-byte aligned float offset
    ensure(scores, copy_q ? qat + nq : parts + 2);
    g.pos0 = pos;  // the query position travels in the launch parameters
    if (copy_q) {
      SLM_CUDA(cudaMemcpyAsync(scores->ptr + qat, qs, nq * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
      qs = scores->ptr + qat;
    }
    // Counters for merging the slices in the slice launch (kept zero between calls).
    const size_t ncnt = at->m * at->heads;
    if (c->merge_cnt_len < ncnt) {
      SLM_CUDA(cudaStreamSynchronize(c->stream));
      dev_free(c->merge_cnt);
      c->merge_cnt = nullptr, c->merge_cnt_len = 0;
      c->merge_cnt = static_cast<unsigned*>(dev_alloc(ncnt * sizeof(unsigned)));
      SLM_CUDA(cudaMemsetAsync(c->merge_cnt, 0, ncnt * sizeof(unsigned), c->stream));
      c->merge_cnt_len = ncnt;
    }
    attention(qs, (int)(at->heads * at->dh), k->ptr, v->ptr, g, nullptr, nsplit, scores->ptr + 2, y->ptr,
              (int)(at->heads * at->dh), c->stream, c->merge_cnt);
  });
}

}  // extern "C"
