// The reference CUDA backend, restated in C++ as a BASELINE (test and bench
// infrastructure only; the product library never links or loads it).
//
// It runs the reference's own kernels: kernels/slm.cu compiled from source to
// compute_60 PTX with the flags of tools/build_kernels.sh (the Makefile beside
// this file writes _ref/slm.ptx) and JIT-compiled by the driver at load time,
// as src/cuda.rs:73-120 does through cudarc.  The host side restates, because
// the Rust crate cannot be built here:
//   * src/cuda.rs:58-66, 122-491 — 32-thread blocks, the launch shapes of each
//     Ops method, zero-filled stream-ordered allocations that grow on demand,
//     the transposed copy and host synchronisation of linear() for m >= 32,
//     the host-side id / factor uploads followed by a synchronisation, the
//     three- or four-pass attention;
//   * src/model.rs:226-690 — weight upload, sessions, Model::block,
//     Model::advance, feed/chunk_at, logits (read = copy + synchronise),
//     grow() through the host.
// Everything runs on the legacy default stream of device `device`.
#include <cuda.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string g_error;

struct CuError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* s = nullptr;
    cuGetErrorString(r, &s);
    throw CuError(std::string(what) + ": " + (s ? s : "unknown CUDA error"));
  }
}
#define CK(x) check((x), #x)

// src/cuda.rs:16-22.
constexpr size_t BLOCK = 32;
constexpr size_t MAX_DH = 256;
constexpr unsigned RMS_THREADS = 64;
constexpr unsigned GLA_THREADS = 64;
constexpr size_t ATTEND_THREADS = 256;
// src/model.rs:27-30.
constexpr size_t CHUNK = 256;
constexpr size_t MAX_SCORES = size_t(1) << 28;

// A device f32 buffer (cudarc's CudaSlice<f32>): stream-ordered allocation,
// freed in stream order when dropped.
struct Buf {
  CUdeviceptr p = 0;
  size_t len = 0;
  Buf() = default;
  Buf(const Buf&) = delete;
  Buf& operator=(const Buf&) = delete;
  Buf(Buf&& o) noexcept : p(o.p), len(o.len) { o.p = 0, o.len = 0; }
  Buf& operator=(Buf&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p, len = o.len;
      o.p = 0, o.len = 0;
    }
    return *this;
  }
  ~Buf() { release(); }
  void release() {
    if (p) cuMemFreeAsync(p, nullptr);
    p = 0, len = 0;
  }
};
void swap(Buf& a, Buf& b) {
  std::swap(a.p, b.p);
  std::swap(a.len, b.len);
}

// A read-only position inside a buffer (src/ops.rs:13-29).
struct At {
  const Buf* buf;
  size_t off;
  CUdeviceptr ptr() const { return buf->p + off * sizeof(float); }
};
At at(const Buf& b, size_t off = 0) { return {&b, off}; }

// src/ops.rs:31-66.
struct Attn {
  size_t pos, m, reach, gap, cap, heads, key_heads, dh;
  float scale;
  size_t base() const { return pos > reach - 1 ? pos - (reach - 1) : 0; }
  size_t span() const {
    size_t a = pos + m, b = gap + base();
    size_t s = a > b ? a - b : 0;
    return s < 1 ? 1 : s;
  }
};

enum Kern {
  K_LINEAR, K_TRANSPOSE, K_LINEAR_MANY, K_GATHER, K_COPY, K_SHIFT, K_COLUMNS, K_ADD, K_ADD_ROW, K_SCALE,
  K_SCALE_ROWS, K_MIX, K_RMS, K_SILU_MUL, K_ROPE_TABLE, K_ROPE, K_L2NORM, K_GLA, K_STORE, K_ATTN_SCORE,
  K_ATTN_EXP, K_ATTN_SUM, K_ATTN_PART, K_ATTN_JOIN, K_COUNT
};
const char* const kNames[K_COUNT] = {
    "slm_linear", "slm_transpose", "slm_linear_many", "slm_gather", "slm_copy", "slm_shift",
    "slm_columns", "slm_add", "slm_add_row", "slm_scale", "slm_scale_rows", "slm_mix",
    "slm_rms", "slm_silu_mul", "slm_rope_table", "slm_rope", "slm_l2norm", "slm_gla",
    "slm_store", "slm_attn_score", "slm_attn_exp", "slm_attn_sum", "slm_attn_part", "slm_attn_join"};

using ptr = CUdeviceptr;

// The backend: one device, its primary context, the loaded module and the
// default stream (src/cuda.rs:52-120).
struct Cuda {
  CUdevice dev = 0;
  CUcontext ctx = nullptr;
  CUmodule mod = nullptr;
  CUfunction f[K_COUNT] = {};
  CUstream st = nullptr;
  long long launches = 0, syncs = 0;

  Cuda(const std::string& ptx_path, int device) {
    CK(cuInit(0));
    CK(cuDeviceGet(&dev, device));
    CK(cuDevicePrimaryCtxRetain(&ctx, dev));
    CK(cuCtxSetCurrent(ctx));
    std::ifstream in(ptx_path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot open " + ptx_path);
    std::stringstream ss;
    ss << in.rdbuf();
    std::string text = ss.str();
    CK(cuModuleLoadData(&mod, text.c_str()));
    for (int k = 0; k < K_COUNT; k++) CK(cuModuleGetFunction(&f[k], mod, kNames[k]));
  }
  ~Cuda() {
    cuCtxSetCurrent(ctx);
    cuStreamSynchronize(st);
    if (mod) cuModuleUnload(mod);
    cuDevicePrimaryCtxRelease(dev);
  }
  void current() { CK(cuCtxSetCurrent(ctx)); }

  template <class... A>
  void launch(Kern k, unsigned grid, unsigned block, unsigned smem, A... args) {
    void* params[] = {static_cast<void*>(&args)...};
    CK(cuLaunchKernel(f[k], grid, 1, 1, block, 1, 1, smem, st, params, nullptr));
    launches++;
  }
  // cfg(threads): ceil(threads / 32) blocks of 32 (src/cuda.rs:58-66).
  template <class... A>
  void launch_n(Kern k, size_t threads, A... args) {
    launch(k, (unsigned)((threads + BLOCK - 1) / BLOCK), (unsigned)BLOCK, 0u, args...);
  }
  void sync() {
    CK(cuStreamSynchronize(st));
    syncs++;
  }

  Buf zeros(size_t n) {
    Buf b;
    CK(cuMemAllocAsync(&b.p, n * sizeof(float), st));
    CK(cuMemsetD32Async(b.p, 0u, n, st));
    b.len = n;
    return b;
  }
  template <class T>
  Buf upload_raw(const T* data, size_t n) {  // clone_htod: allocation + copy
    Buf b;
    size_t bytes = n * sizeof(T);
    CK(cuMemAllocAsync(&b.p, bytes < 4 ? 4 : bytes, st));
    CK(cuMemcpyHtoDAsync(b.p, data, bytes, st));
    b.len = (bytes + 3) / 4;
    return b;
  }
  Buf upload(const std::vector<float>& v) { return upload_raw(v.data(), v.size()); }
  void read(const Buf& b, size_t n, float* out) {
    CK(cuMemcpyDtoHAsync(out, b.p, n * sizeof(float), st));
    sync();
  }
  void ensure(Buf& y, size_t n) {
    if (y.len < n) y = zeros(n);
  }

  // ---- Ops (src/cuda.rs:131-491) ----------------------------------------
  void copy(Buf& y, At x, size_t n) {
    ensure(y, n);
    launch_n(K_COPY, n, y.p, x.ptr(), (int)n);
  }
  void gather(Buf& y, const Buf& w, const uint32_t* ids, size_t m, size_t d) {
    ensure(y, m * d);
    if (m == 1) return copy(y, at(w, (size_t)ids[0] * d), d);
    std::vector<int32_t> list(ids, ids + m);
    Buf dl = upload_raw(list.data(), m);
    launch_n(K_GATHER, m * d, y.p, w.p, dl.p, (int)m, (int)d);
    sync();  // the ids must stay allocated until the kernel has read them
  }
  void shift(Buf& y, const Buf& first, At x, size_t m, size_t d) {
    ensure(y, m * d);
    launch_n(K_SHIFT, m * d, y.p, first.p, x.ptr(), (int)m, (int)d);
  }
  void columns(Buf& y, const Buf& x, size_t m, size_t stride, size_t off, size_t len) {
    ensure(y, m * len);
    launch_n(K_COLUMNS, m * len, y.p, x.p, (int)m, (int)stride, (int)off, (int)len);
  }
  void linear(Buf& y, const Buf& w, size_t rows, size_t cols, At x, size_t m) {
    ensure(y, m * rows);
    if (m < BLOCK) {
      launch_n(K_LINEAR, m * rows, y.p, w.p, x.ptr(), (int)rows, (int)cols, (int)m);
      return;
    }
    Buf xt = zeros(m * cols);
    launch_n(K_TRANSPOSE, m * cols, xt.p, x.ptr(), (int)m, (int)cols);
    launch_n(K_LINEAR_MANY, m * rows, y.p, w.p, xt.p, (int)rows, (int)cols, (int)m);
    sync();  // the transposed copy must stay allocated until the kernel has read it
  }
  void add(Buf& y, At a, At b, size_t n) {
    ensure(y, n);
    launch_n(K_ADD, n, y.p, a.ptr(), b.ptr(), (int)n);
  }
  void add_row(Buf& y, At x, At row, size_t m, size_t d) {
    ensure(y, m * d);
    launch_n(K_ADD_ROW, m * d, y.p, x.ptr(), row.ptr(), (int)m, (int)d);
  }
  void scale_rows(Buf& y, At x, const std::vector<float>& f, size_t d) {
    size_t m = f.size();
    ensure(y, m * d);
    if (m == 1) {
      launch_n(K_SCALE, d, y.p, x.ptr(), (int)d, f[0]);
      return;
    }
    Buf fd = upload(f);
    launch_n(K_SCALE_ROWS, m * d, y.p, x.ptr(), fd.p, (int)m, (int)d);
    sync();  // the factors must stay allocated until the kernel has read them
  }
  void mix(Buf& y, At a, At b, size_t n, float t) {
    ensure(y, n);
    launch_n(K_MIX, n, y.p, a.ptr(), b.ptr(), (int)n, t);
  }
  void rms(Buf& y, At x, const Buf& w, size_t groups, size_t size, float eps) {
    ensure(y, groups * size);
    unsigned threads = RMS_THREADS < (unsigned)size ? RMS_THREADS : (unsigned)size;
    launch(K_RMS, (unsigned)groups, threads, threads * 4u, y.p, x.ptr(), w.p, (int)groups, (int)size, eps);
  }
  void silu_mul(Buf& y, At g, At u, size_t n) {
    ensure(y, n);
    launch_n(K_SILU_MUL, n, y.p, g.ptr(), u.ptr(), (int)n);
  }
  void rope_table(Buf& c, Buf& s, const Buf& inv, size_t pos, size_t m, size_t half) {
    ensure(c, m * half);
    ensure(s, m * half);
    launch_n(K_ROPE_TABLE, m * half, c.p, s.p, inv.p, (float)pos, (int)half, (int)m);
  }
  void rope(Buf& y, At x, const Buf& c, const Buf& s, size_t m, size_t heads, size_t dh) {
    ensure(y, m * heads * dh);
    launch_n(K_ROPE, m * heads * dh / 2, y.p, x.ptr(), c.p, s.p, (int)m, (int)heads, (int)dh);
  }
  void l2norm(Buf& y, At x, size_t heads, size_t dh) {
    ensure(y, heads * dh);
    launch_n(K_L2NORM, heads, y.p, x.ptr(), (int)heads, (int)dh);
  }
  void gla(Buf& y, Buf& s, At q, At k, At v, const Buf& decay, const Buf& bias, size_t m, size_t heads,
           size_t dh) {
    ensure(y, m * heads * dh);
    unsigned threads = GLA_THREADS < (unsigned)dh ? GLA_THREADS : (unsigned)dh;
    launch(K_GLA, (unsigned)heads, threads, 0u, y.p, s.p, q.ptr(), k.ptr(), v.ptr(), decay.p, bias.p, (int)m,
           (int)heads, (int)dh);
  }
  void store(Buf& cache, At src, size_t pos, size_t m, size_t cap, size_t heads, size_t dh) {
    launch_n(K_STORE, m * heads * dh, cache.p, src.ptr(), (int)pos, (int)m, (int)cap, (int)heads, (int)dh);
  }
  void attend(Buf& y, Buf& scores, At q, const Buf& k, const Buf& v, const Attn& a) {
    if (a.dh > MAX_DH) throw std::runtime_error("head size above the 256 the kernels allow");
    size_t span = a.span(), pairs = a.heads * a.m;
    size_t slices = ATTEND_THREADS / a.m;
    if (slices < 1) slices = 1;
    if (slices > span) slices = span;
    size_t atn = pairs * span;
    ensure(y, pairs * a.dh);
    ensure(scores, atn + pairs * slices * (2 + a.dh));
    int pos = (int)a.pos, m = (int)a.m;
    int reach = (int)(a.reach < (size_t)std::numeric_limits<int>::max() ? a.reach
                                                                        : (size_t)std::numeric_limits<int>::max());
    int gap = (int)a.gap, sp = (int)span, cap = (int)a.cap, h = (int)a.heads, kh = (int)a.key_heads,
        d = (int)a.dh, p = (int)slices;
    ptr sc = scores.p, aux = scores.p + atn * sizeof(float);
    size_t threads = pairs * slices;
    launch_n(K_ATTN_SCORE, threads, sc, aux, q.ptr(), k.p, pos, m, reach, gap, sp, cap, h, kh, d, p, a.scale);
    launch_n(K_ATTN_EXP, threads, sc, aux, pos, m, reach, gap, sp, h, p);
    if (a.m < BLOCK) {
      launch_n(K_ATTN_PART, threads, sc, aux, v.p, pos, m, reach, gap, sp, cap, h, kh, d, p);
      launch_n(K_ATTN_JOIN, pairs * a.dh, y.p, aux, m, h, d, p);
    } else {
      launch_n(K_ATTN_SUM, pairs * a.dh, y.p, sc, aux, v.p, pos, m, reach, gap, sp, cap, h, kh, d, p);
    }
  }
};

// ---- Model driver (src/model.rs) -----------------------------------------

struct Config {
  size_t vocab = 0, d = 0, heads = 0, kv_heads = 4, window = 0, max_loops = 0, default_loops = 0;
  uint32_t logn = 0, kshift = 0, emb = 0, far = 0;
  float damp = 1.0f, rope_base = 10000.0f, eps = 1e-6f;
  std::string prelude, core, coda;
  size_t dh() const { return d / heads; }
};

struct Mat {
  Buf w;
  size_t rows = 0, cols = 0;
};

struct Block {
  char kind = 'S';
  Buf norm1, norm2, bias, head_norm, norm_e;
  bool has_norm_e = false;
  Mat up, down, qkv, o, qkvg, decay, q, kv;
};

struct State {
  char kind = 'S';
  Buf k, v, s, prev, scores;
  size_t cap = 0;
};

struct Scratch {
  Buf n, mix, q, k, v, g, y, y2, h, t, d, shifted, prev_kv, up, gate, mid, scores, cos, sin;
};

struct Session {
  size_t loops = 0, pos = 0;
  std::vector<State> prelude, coda;
  std::vector<std::vector<State>> core;
  Scratch sc;
  Buf x, s, e0, e_proj, last, logits;
};

struct Model {
  Cuda* cu;
  Config cfg;
  std::map<std::string, std::pair<std::vector<size_t>, std::vector<float>>> pending;
  std::vector<Block> prelude, core, coda;
  Mat embed, inject, loop_embed;
  bool looped = false;
  Buf norm_f, inv_freq;

  size_t cap() const { return cfg.window + CHUNK; }

  std::pair<std::vector<size_t>, std::vector<float>> take(const std::string& name) {
    auto it = pending.find(name);
    if (it == pending.end()) throw std::runtime_error("missing weight " + name);
    auto out = std::move(it->second);
    pending.erase(it);
    return out;
  }
  Mat mat(const std::string& name) {
    auto t = take(name);
    if (t.first.size() != 2) throw std::runtime_error(name + ": expected a matrix");
    Mat m;
    m.w = cu->upload(t.second);
    m.rows = t.first[0];
    m.cols = t.first[1];
    return m;
  }
  Buf vec(const std::string& name) { return cu->upload(take(name).second); }

  // Block::load (src/model.rs:114-153).
  Block load_block(const std::string& prefix, char kind) {
    auto n = [&](const char* s) { return prefix + "." + s; };
    Block b;
    b.kind = kind;
    if (kind == 'S') {
      b.qkv = mat(n("mixer.qkv.weight"));
      b.o = mat(n("mixer.o.weight"));
    } else if (kind == 'L') {
      b.qkvg = mat(n("mixer.qkvg.weight"));
      b.decay = mat(n("mixer.decay.weight"));
      b.bias = vec(n("mixer.decay.bias"));
      b.head_norm = vec(n("mixer.head_norm.weight"));
      b.o = mat(n("mixer.o.weight"));
    } else if (kind == 'G') {
      b.q = mat(n("mixer.q.weight"));
      b.kv = mat(n("mixer.kv.weight"));
      b.o = mat(n("mixer.o.weight"));
      if (cfg.emb != 0) {
        b.norm_e = vec(n("mixer.norm_e.weight"));
        b.has_norm_e = true;
      }
    } else {
      throw std::runtime_error(std::string("unknown layer type ") + kind);
    }
    b.norm1 = vec(n("norm1.weight"));
    b.norm2 = vec(n("norm2.weight"));
    b.up = mat(n("mlp.up.weight"));
    b.down = mat(n("mlp.down.weight"));
    return b;
  }

  // Model::load (src/model.rs:226-269), after the host tensors were handed over.
  void finish() {
    auto blocks = [&](std::vector<Block>* out, const char* name, const std::string& kinds) {
      for (size_t i = 0; i < kinds.size(); i++)
        out->push_back(load_block(std::string(name) + "." + std::to_string(i), kinds[i]));
    };
    blocks(&prelude, "prelude", cfg.prelude);
    blocks(&core, "core", cfg.core);
    blocks(&coda, "coda", cfg.coda);
    looped = !cfg.core.empty();
    if (looped) {
      inject = mat("inject_e.weight");
      loop_embed = mat("loop_embed.weight");
    }
    embed = mat("embed.weight");
    norm_f = vec("norm_f.weight");
    size_t dh = cfg.dh();
    std::vector<float> inv(dh / 2);
    for (size_t i = 0; i < dh / 2; i++) inv[i] = 1.0f / std::pow(cfg.rope_base, (float)(2 * i) / (float)dh);
    inv_freq = cu->upload(inv);
    pending.clear();
    cu->sync();
  }

  // src/model.rs:308-331.
  State new_state(const Block& b) {
    State st;
    st.kind = b.kind;
    size_t h = cfg.heads, dh = cfg.dh();
    if (b.kind == 'S') {
      st.k = cu->zeros(h * cap() * dh);
      st.v = cu->zeros(h * cap() * dh);
    } else if (b.kind == 'L') {
      st.s = cu->zeros(h * dh * dh);
    } else {
      st.cap = size_t(1) << 13;
      st.k = cu->zeros(cfg.kv_heads * st.cap * dh);
      st.v = cu->zeros(cfg.kv_heads * st.cap * dh);
      st.prev = cu->zeros(cfg.d);
      st.scores = cu->zeros(1);
    }
    return st;
  }

  // src/model.rs:333-381.
  Session* session(size_t loops) {
    if (loops == 0) loops = cfg.default_loops;
    if (looped && (loops < 1 || loops > cfg.max_loops)) throw std::runtime_error("loops out of range");
    auto* se = new Session;
    se->loops = loops;
    for (auto& b : prelude) se->prelude.push_back(new_state(b));
    for (size_t r = 0; r < loops; r++) {
      se->core.emplace_back();
      for (auto& b : core) se->core.back().push_back(new_state(b));
    }
    for (auto& b : coda) se->coda.push_back(new_state(b));
    size_t d = cfg.d, half = cfg.dh() / 2;
    Scratch& s = se->sc;
    s.n = cu->zeros(d), s.mix = cu->zeros(4 * d), s.q = cu->zeros(d), s.k = cu->zeros(d), s.v = cu->zeros(d);
    s.g = cu->zeros(d), s.y = cu->zeros(d), s.y2 = cu->zeros(d), s.h = cu->zeros(d), s.t = cu->zeros(d);
    s.d = cu->zeros(cfg.heads), s.shifted = cu->zeros(d), s.prev_kv = cu->zeros(2 * d), s.up = cu->zeros(4 * d);
    s.gate = cu->zeros(2 * d), s.mid = cu->zeros(2 * d), s.scores = cu->zeros(1), s.cos = cu->zeros(half);
    s.sin = cu->zeros(half);
    se->x = cu->zeros(d), se->s = cu->zeros(d), se->e0 = cu->zeros(d), se->e_proj = cu->zeros(d);
    se->last = cu->zeros(d), se->logits = cu->zeros(cfg.vocab);
    return se;
  }

  // Doubles a global cache through the host (src/model.rs:384-398).
  void grow(State& st) {
    size_t kh = cfg.kv_heads, dh = cfg.dh(), old = st.cap, nw = old * 2;
    for (Buf* buf : {&st.k, &st.v}) {
      std::vector<float> data(kh * old * dh), out(kh * nw * dh, 0.0f);
      cu->read(*buf, data.size(), data.data());
      for (size_t h = 0; h < kh; h++)
        std::memcpy(out.data() + h * nw * dh, data.data() + h * old * dh, old * dh * sizeof(float));
      *buf = cu->upload(out);
    }
    st.cap = nw;
  }

  // Model::block (src/model.rs:400-560).
  void block(const Block& b, State& st, Buf& x, const Buf& e0, Scratch& sc, size_t pos, size_t m) {
    Cuda& o = *cu;
    const Config& c = cfg;
    size_t d = c.d, heads = c.heads, dh = c.dh();
    float eps = c.eps, scale = 1.0f / std::sqrt((float)dh);
    size_t n = m * d;
    o.rms(sc.n, at(x), b.norm1, m, d, eps);
    // One token needs no copy to split a row: its columns are already contiguous.
    auto col = [&](Buf& y, const Buf& src, size_t stride, size_t off, size_t len) -> At {
      if (m == 1) return at(src, off);
      o.columns(y, src, m, stride, off, len);
      return at(y);
    };
    bool has_h = true;
    if (b.kind == 'S') {
      o.linear(sc.mix, b.qkv.w, b.qkv.rows, d, at(sc.n), m);
      At raw = col(sc.y, sc.mix, 3 * d, 0, d);
      o.rope(sc.q, raw, sc.cos, sc.sin, m, heads, dh);
      raw = col(sc.y, sc.mix, 3 * d, d, d);
      o.rope(sc.k, raw, sc.cos, sc.sin, m, heads, dh);
      At vals = col(sc.v, sc.mix, 3 * d, 2 * d, d);
      o.store(st.k, at(sc.k), pos, m, cap(), heads, dh);
      o.store(st.v, vals, pos, m, cap(), heads, dh);
      Attn a{pos, m, c.window, 0, cap(), heads, heads, dh, scale};
      o.attend(sc.y, sc.scores, at(sc.q), st.k, st.v, a);
      o.linear(sc.h, b.o.w, d, d, at(sc.y), m);
    } else if (b.kind == 'L') {
      o.linear(sc.mix, b.qkvg.w, b.qkvg.rows, d, at(sc.n), m);
      At raw = col(sc.y, sc.mix, 4 * d, 0, d);
      o.l2norm(sc.q, raw, m * heads, dh);
      raw = col(sc.y, sc.mix, 4 * d, d, d);
      o.l2norm(sc.k, raw, m * heads, dh);
      At vals = col(sc.v, sc.mix, 4 * d, 2 * d, d);
      At gate = col(sc.g, sc.mix, 4 * d, 3 * d, d);
      o.linear(sc.d, b.decay.w, heads, d, at(sc.n), m);
      o.gla(sc.y, st.s, at(sc.q), at(sc.k), vals, sc.d, b.bias, m, heads, dh);
      o.rms(sc.y2, at(sc.y), b.head_norm, m * heads, dh, eps);
      o.silu_mul(sc.y, gate, at(sc.y2), n);
      o.linear(sc.h, b.o.w, d, d, at(sc.y), m);
    } else {  // 'G'
      if (b.has_norm_e) {
        o.rms(sc.t, at(e0), b.norm_e, m, d, eps);
        o.add(sc.y, at(sc.n), at(sc.t), n);
        swap(sc.n, sc.y);
      }
      size_t kh = c.kv_heads, kd = c.kv_heads * dh;
      o.linear(sc.q, b.q.w, d, d, at(sc.n), m);
      o.linear(sc.mix, b.kv.w, 2 * kd, d, at(sc.n), m);
      if (c.logn != 0) {
        float lg = std::log((float)c.logn);
        std::vector<float> f(m);
        for (size_t i = 0; i < m; i++) f[i] = std::log1p((float)(pos + i)) / lg;
        o.scale_rows(sc.y, at(sc.q), f, d);
        swap(sc.q, sc.y);
      }
      while (pos + m > st.cap) grow(st);
      At keys;
      if (c.kshift != 0) {
        o.shift(sc.shifted, st.prev, at(sc.n), m, d);
        o.linear(sc.prev_kv, b.kv.w, 2 * kd, d, at(sc.shifted), m);
        o.copy(st.prev, at(sc.n, (m - 1) * d), d);
        keys = col(sc.k, sc.prev_kv, 2 * kd, 0, kd);
      } else {
        keys = col(sc.k, sc.mix, 2 * kd, 0, kd);
      }
      At vals = col(sc.v, sc.mix, 2 * kd, kd, kd);
      o.store(st.k, keys, pos, m, st.cap, kh, dh);
      o.store(st.v, vals, pos, m, st.cap, kh, dh);
      size_t far = c.far != 0 ? c.window : 0;
      if (pos + m > far) {
        Attn a{pos, m, std::numeric_limits<size_t>::max(), far, st.cap, heads, kh, dh, scale};
        o.attend(sc.y, st.scores, at(sc.q), st.k, st.v, a);
        o.linear(sc.h, b.o.w, d, d, at(sc.y), m);
      } else {
        has_h = false;
      }
    }
    if (has_h) {
      o.add(sc.t, at(x), at(sc.h), n);
      swap(x, sc.t);
    }
    o.rms(sc.n, at(x), b.norm2, m, d, eps);
    size_t hidden = b.down.cols;
    o.linear(sc.up, b.up.w, 2 * hidden, d, at(sc.n), m);
    At gate = col(sc.gate, sc.up, 2 * hidden, 0, hidden);
    At amp = col(sc.mid, sc.up, 2 * hidden, hidden, hidden);
    o.silu_mul(sc.y, gate, amp, m * hidden);
    o.linear(sc.h, b.down.w, d, hidden, at(sc.y), m);
    o.add(sc.t, at(x), at(sc.h), n);
    swap(x, sc.t);
  }

  // Model::advance (src/model.rs:563-640).
  void advance(Session& se, const uint32_t* tokens, size_t m, bool want_logits) {
    Cuda& o = *cu;
    size_t d = cfg.d, pos = se.pos;
    o.rope_table(se.sc.cos, se.sc.sin, inv_freq, pos, m, cfg.dh() / 2);
    o.gather(se.e0, embed.w, tokens, m, d);
    o.copy(se.x, at(se.e0), m * d);
    for (size_t i = 0; i < prelude.size(); i++) block(prelude[i], se.prelude[i], se.x, se.e0, se.sc, pos, m);
    if (looped) {
      o.linear(se.e_proj, inject.w, d, d, at(se.x), m);
      o.copy(se.s, at(se.x), m * d);
      for (size_t r = 0; r < se.loops; r++) {
        o.add(se.sc.t, at(se.s), at(se.e_proj), m * d);
        o.add_row(se.x, at(se.sc.t), at(loop_embed.w, r * d), m, d);
        for (size_t i = 0; i < core.size(); i++) block(core[i], se.core[r][i], se.x, se.e0, se.sc, pos, m);
        if (cfg.damp == 1.0f) {
          swap(se.s, se.x);
        } else {
          o.mix(se.sc.t, at(se.s), at(se.x), m * d, cfg.damp);
          swap(se.s, se.sc.t);
        }
      }
      swap(se.x, se.s);
    }
    for (size_t i = 0; i < coda.size(); i++) block(coda[i], se.coda[i], se.x, se.e0, se.sc, pos, m);
    if (want_logits) {
      o.copy(se.last, at(se.x, (m - 1) * d), d);
      o.rms(se.sc.n, at(se.last), norm_f, 1, d, cfg.eps);
      o.linear(se.logits, embed.w, cfg.vocab, d, at(se.sc.n), 1);
    }
    se.pos += m;
  }

  // src/model.rs:642-667.
  size_t chunk_at(size_t pos, size_t limit) const {
    size_t chunk = std::min(limit, CHUNK);
    if (cfg.coda.find('G') != std::string::npos || cfg.prelude.find('G') != std::string::npos)
      return std::min(chunk, std::max<size_t>(MAX_SCORES / cfg.heads / (pos + 1), 1));
    return chunk;
  }
  void feed(Session& se, const uint32_t* tokens, size_t n, size_t limit) {
    size_t done = 0;
    while (done < n) {
      size_t m = std::min(chunk_at(se.pos, limit), n - done);
      advance(se, tokens + done, m, done + m == n);
      done += m;
    }
  }
};

template <class F>
int guard(F&& f) {
  try {
    f();
    g_error.clear();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

}  // namespace

extern "C" {

const char* rc_error() { return g_error.c_str(); }

// Device `device`'s primary context with the module loaded from `ptx_path`.
void* rc_new(const char* ptx_path, int device) {
  Cuda* c = nullptr;
  if (guard([&] { c = new Cuda(ptx_path, device); }) != 0) return nullptr;
  return c;
}
void rc_free(void* c) { delete static_cast<Cuda*>(c); }
// Kernel launches and host synchronisations issued so far.
void rc_counts(void* c, long long* launches, long long* syncs) {
  *launches = static_cast<Cuda*>(c)->launches;
  *syncs = static_cast<Cuda*>(c)->syncs;
}

// ints: vocab, d, heads, kv_heads, window, max_loops, default_loops, logn, kshift, emb, far;
// floats: damp, rope_base, eps (src/config.rs).
void* rc_model_new(void* cuda, const char* prelude, const char* core, const char* coda, const int64_t* ints,
                   const float* floats) {
  auto* m = new Model;
  m->cu = static_cast<Cuda*>(cuda);
  Config& c = m->cfg;
  c.vocab = ints[0], c.d = ints[1], c.heads = ints[2], c.kv_heads = ints[3], c.window = ints[4];
  c.max_loops = ints[5], c.default_loops = ints[6];
  c.logn = (uint32_t)ints[7], c.kshift = (uint32_t)ints[8], c.emb = (uint32_t)ints[9], c.far = (uint32_t)ints[10];
  c.damp = floats[0], c.rope_base = floats[1], c.eps = floats[2];
  c.prelude = prelude, c.core = core, c.coda = coda;
  return m;
}
int rc_model_set(void* model, const char* name, const float* data, const int64_t* shape, int ndim) {
  return guard([&] {
    auto* m = static_cast<Model*>(model);
    std::vector<size_t> s(shape, shape + ndim);
    size_t n = 1;
    for (size_t v : s) n *= v;
    m->pending[name] = {s, std::vector<float>(data, data + n)};
  });
}
int rc_model_finish(void* model) {
  return guard([&] {
    auto* m = static_cast<Model*>(model);
    m->cu->current();
    m->finish();
  });
}
void rc_model_free(void* model) {
  auto* m = static_cast<Model*>(model);
  m->cu->current();
  delete m;
}

void* rc_session_new(void* model, int64_t loops) {
  Session* se = nullptr;
  auto* m = static_cast<Model*>(model);
  if (guard([&] {
        m->cu->current();
        se = m->session((size_t)loops);
        m->cu->sync();
      }) != 0)
    return nullptr;
  return se;
}
void rc_session_free(void* model, void* se) {
  static_cast<Model*>(model)->cu->current();
  delete static_cast<Session*>(se);
}
int64_t rc_session_pos(void* se) { return (int64_t) static_cast<Session*>(se)->pos; }

int rc_feed(void* model, void* se, const uint32_t* ids, int64_t n, int64_t limit) {
  return guard([&] {
    auto* m = static_cast<Model*>(model);
    m->cu->current();
    m->feed(*static_cast<Session*>(se), ids, (size_t)n, (size_t)limit);
  });
}
int rc_step(void* model, void* se, uint32_t id) {
  return guard([&] {
    auto* m = static_cast<Model*>(model);
    m->cu->current();
    m->advance(*static_cast<Session*>(se), &id, 1, true);
  });
}
// Model::logits (src/model.rs:670-672): a copy of the vocab logits and a synchronisation.
int rc_logits(void* model, void* se, float* out) {
  return guard([&] {
    auto* m = static_cast<Model*>(model);
    m->cu->current();
    m->cu->read(static_cast<Session*>(se)->logits, m->cfg.vocab, out);
  });
}
int rc_sync(void* cuda) {
  return guard([&] { static_cast<Cuda*>(cuda)->sync(); });
}

}  // extern "C"
