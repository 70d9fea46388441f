// CPU oracle for the SLM.use token loop.  TEST INFRASTRUCTURE ONLY: the parity
// tests, the smoke check and the CPU-baseline leg of the bench call it as the
// checker; the product library never links or calls it.
//
// It restates, in plain C++17 with OpenMP, the reference's CPU backend and its
// model driver:
//   - every operation of the `Ops` trait with the arithmetic of the CPU backend
//     (reference src/cpu.rs:9-403, trait in src/ops.rs:68-228),
//   - the looped hybrid model: block(), advance(), feed()/chunk_at(), state
//     layout and the global-cache growth (src/model.rs:226-690),
//   - the sampler pick() and the xorshift64* Rng (src/sample.rs:18-93), with one
//     documented difference: top-k keeps a canonical order (logit descending,
//     then id ascending) where the reference uses select_nth_unstable, whose
//     order is unspecified.
// Parity is pinned by the reference's own golden vectors (tests/golden/tiny:
// PyTorch logits at 40 positions, tolerance 1e-4 as in tests/parity.rs:13).
//
// Floating point: built with -ffp-contract=off so a*b+c stays two roundings as
// in the Rust source; exp/cos/sin/pow/log1p come from the C library as f32::exp
// etc. do in the reference.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <omp.h>

namespace {

// ---------------------------------------------------------------------------
// Ops (src/cpu.rs)
// ---------------------------------------------------------------------------

// 16 running sums over chunks of 16, then their sequential sum plus the tail
// (src/cpu.rs:9-21).  Cloned per ISA like the reference's multiversion targets.
__attribute__((target_clones("avx512f", "avx2", "default"))) float dot(const float* a, const float* b, size_t n) {
  float acc[16] = {0};
  size_t full = n / 16 * 16;
  for (size_t c = 0; c < full; c += 16) {
    for (int i = 0; i < 16; i++) acc[i] += a[c + i] * b[c + i];
  }
  float tail = 0.0f;
  for (size_t i = full; i < n; i++) tail += a[i] * b[i];
  float s = -0.0f;
  for (int i = 0; i < 16; i++) s += acc[i];
  return s + tail;
}

// y += a*x (src/cpu.rs:23-28).
__attribute__((target_clones("avx512f", "avx2", "default"))) void axpy(float* y, float a, const float* x, size_t n) {
  for (size_t i = 0; i < n; i++) y[i] += a * x[i];
}

// y[i] = w * x[i], w rows x cols (src/cpu.rs:111-130).
void op_linear(float* y, const float* w, size_t rows, size_t cols, const float* x, size_t m) {
  const long long total = (long long)(m * rows);
#pragma omp parallel for schedule(static)
  for (long long t = 0; t < total; t++) {
    size_t i = (size_t)t / rows, r = (size_t)t % rows;
    y[t] = dot(w + r * cols, x + i * cols, cols);
  }
}

void op_add(float* y, const float* a, const float* b, size_t n) {
  for (size_t i = 0; i < n; i++) y[i] = a[i] + b[i];
}

void op_add_row(float* y, const float* x, const float* row, size_t m, size_t d) {
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < d; j++) y[i * d + j] = x[i * d + j] + row[j];
}

void op_scale_rows(float* y, const float* x, const float* f, size_t m, size_t d) {
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < d; j++) y[i * d + j] = x[i * d + j] * f[i];
}

void op_mix(float* y, const float* a, const float* b, size_t n, float t) {
  for (size_t i = 0; i < n; i++) y[i] = a[i] + t * (b[i] - a[i]);
}

// RMSNorm per group (src/cpu.rs:187-207).
void op_rms(float* y, const float* x, const float* w, size_t groups, size_t size, float eps) {
  for (size_t g = 0; g < groups; g++) {
    const float* in = x + g * size;
    float* o = y + g * size;
    float r = 1.0f / std::sqrt(dot(in, in, size) / (float)size + eps);
    for (size_t i = 0; i < size; i++) o[i] = in[i] * r * w[i];
  }
}

// y = u*g/(1+exp(-g)) (src/cpu.rs:209-215).
void op_silu_mul(float* y, const float* g, const float* u, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float v = g[i];
    y[i] = u[i] * v / (1.0f + std::exp(-v));
  }
}

// src/cpu.rs:217-237.
void op_rope_table(float* cos_, float* sin_, const float* inv, size_t pos, size_t m, size_t half) {
  for (size_t i = 0; i < m; i++) {
    float p = (float)(pos + i);
    for (size_t j = 0; j < half; j++) {
      float a = p * inv[j];
      cos_[i * half + j] = std::cos(a);
      sin_[i * half + j] = std::sin(a);
    }
  }
}

// Half-split rotation (src/cpu.rs:239-268).
void op_rope(float* y, const float* x, const float* cos_, const float* sin_, size_t m,
             size_t heads, size_t dh) {
  size_t half = dh / 2;
  for (size_t t = 0; t < m * heads; t++) {
    size_t row = t / heads;
    const float* h = x + t * dh;
    float* o = y + t * dh;
    const float* c = cos_ + row * half;
    const float* s = sin_ + row * half;
    for (size_t i = 0; i < half; i++) {
      float a = h[i], b = h[half + i];
      o[i] = a * c[i] - b * s[i];
      o[half + i] = a * s[i] + b * c[i];
    }
  }
}

// src/cpu.rs:270-282.
void op_l2norm(float* y, const float* x, size_t heads, size_t dh) {
  for (size_t t = 0; t < heads; t++) {
    const float* h = x + t * dh;
    float r = 1.0f / std::max(std::sqrt(dot(h, h, dh)), 1e-12f);
    for (size_t i = 0; i < dh; i++) y[t * dh + i] = h[i] * r;
  }
}

// Gated linear attention, token by token per head (src/cpu.rs:284-329).
void op_gla(float* y, float* s, const float* q, const float* k, const float* v,
            const float* decay, const float* bias, size_t m, size_t heads, size_t dh) {
#pragma omp parallel for schedule(static)
  for (long long hh = 0; hh < (long long)heads; hh++) {
    size_t h = (size_t)hh;
    float* state = s + h * dh * dh;
    for (size_t i = 0; i < m; i++) {
      size_t at = (i * heads + h) * dh;
      float d = 1.0f / (1.0f + std::exp(decay[i * heads + h] + bias[h]));
      const float* vh = v + at;
      for (size_t a = 0; a < dh; a++) {
        float ka = k[at + a];
        float* row = state + a * dh;
        for (size_t b = 0; b < dh; b++) row[b] = d * row[b] + ka * vh[b];
      }
      float* o = y + at;
      for (size_t b = 0; b < dh; b++) o[b] = 0.0f;
      for (size_t a = 0; a < dh; a++) axpy(o, q[at + a], state + a * dh, dh);
    }
  }
}

// src/cpu.rs:331-350.
void op_store(float* cache, const float* src, size_t pos, size_t m, size_t cap, size_t heads,
              size_t dh) {
  for (size_t i = 0; i < m; i++) {
    size_t slot = (pos + i) % cap;
    for (size_t h = 0; h < heads; h++)
      std::memcpy(cache + (h * cap + slot) * dh, src + (i * heads + h) * dh, dh * sizeof(float));
  }
}

// Attention window (src/ops.rs:31-66).  reach == 0 stands for usize::MAX.
struct Attn {
  size_t pos, m, reach, gap, cap, heads, key_heads, dh;
  float scale;
  void range(size_t i, size_t* lo, size_t* hi) const {  // [lo, hi)
    size_t p = pos + i;
    *lo = (reach == 0 || p < reach - 1) ? 0 : p - (reach - 1);
    *hi = (p + 1 > gap) ? p + 1 - gap : 0;
    if (*hi < *lo) *hi = *lo;
  }
};

// Softmax attention per query (src/cpu.rs:352-403).
void op_attend(float* y, const float* q, const float* k, const float* v, const Attn& a) {
  size_t heads = a.heads, dh = a.dh, cap = a.cap, group = heads / a.key_heads;
#pragma omp parallel for schedule(static)
  for (long long ii = 0; ii < (long long)a.m; ii++) {
    size_t i = (size_t)ii, lo, hi;
    a.range(i, &lo, &hi);
    std::vector<float> sc(hi - lo);
    for (size_t h = 0; h < heads; h++) {
      float* o = y + (i * heads + h) * dh;
      for (size_t e = 0; e < dh; e++) o[e] = 0.0f;
      if (hi == lo) continue;
      size_t base = (h / group) * cap * dh;
      const float* qh = q + (i * heads + h) * dh;
      float mx = -INFINITY;
      for (size_t p = lo; p < hi; p++) {
        float s = dot(qh, k + base + (p % cap) * dh, dh) * a.scale;
        sc[p - lo] = s;
        mx = std::max(mx, s);
      }
      float sum = 0.0f;
      for (auto& s : sc) {
        s = std::exp(s - mx);
        sum += s;
      }
      for (size_t p = lo; p < hi; p++) axpy(o, sc[p - lo] / sum, v + base + (p % cap) * dh, dh);
    }
  }
}

// ---------------------------------------------------------------------------
// Model (src/model.rs)
// ---------------------------------------------------------------------------

constexpr size_t CHUNK = 256;            // src/model.rs:27
constexpr size_t MAX_SCORES = 1u << 28;  // src/model.rs:30

struct Config {
  size_t vocab = 0, d = 0, heads = 0, kv_heads = 4, window = 0, max_loops = 0, default_loops = 0;
  uint32_t logn = 0, kshift = 0, emb = 0, far = 0;
  float damp = 1.0f, rope_base = 10000.0f, eps = 1e-6f;
  std::string prelude, core, coda;
  size_t dh() const { return d / heads; }
};

struct Mat {
  std::vector<float> w;
  size_t rows = 0, cols = 0;
};

struct Block {
  char kind = 'S';
  std::vector<float> norm1, norm2;
  Mat up, down;
  Mat qkv, o;                                   // S (o shared by all kinds)
  Mat qkvg, decay;                              // L
  std::vector<float> bias, head_norm;           // L
  Mat q, kv;                                    // G
  std::vector<float> norm_e;                    // G, when global_emb
};

struct State {
  char kind = 'S';
  std::vector<float> k, v, s, prev;
  size_t cap = 0;
};

struct Scratch {
  std::vector<float> n, mix, q, k, v, g, y, y2, h, t, dec, shifted, prev_kv, up, gate, mid, cos_, sin_,
      e, tmp;
};

struct Model;

struct Session {
  Model* model = nullptr;
  size_t loops = 0, pos = 0;
  std::vector<State> prelude, coda;
  std::vector<std::vector<State>> core;
  Scratch sc;
  std::vector<float> x, s, e0, e_proj, last, logits;
};

struct Model {
  Config cfg;
  std::map<std::string, std::pair<std::vector<size_t>, std::vector<float>>> pending;
  std::vector<Block> prelude, core, coda;
  Mat embed, inject, loop_embed;
  bool looped = false;
  std::vector<float> norm_f, inv_freq;
  std::string error;

  size_t cap() const { return cfg.window + CHUNK; }

  bool take(const std::string& name, std::vector<float>* out, std::vector<size_t>* shape = nullptr) {
    auto it = pending.find(name);
    if (it == pending.end()) {
      error = "missing weight " + name;
      return false;
    }
    if (shape) *shape = it->second.first;
    *out = std::move(it->second.second);
    pending.erase(it);
    return true;
  }
  bool mat(const std::string& name, Mat* m) {
    std::vector<size_t> shape;
    if (!take(name, &m->w, &shape)) return false;
    if (shape.size() != 2) {
      error = name + ": expected a matrix";
      return false;
    }
    m->rows = shape[0];
    m->cols = shape[1];
    return true;
  }

  // Block::load (src/model.rs:114-153).
  bool load_block(Block* b, const std::string& prefix, char kind) {
    auto n = [&](const char* s) { return prefix + "." + s; };
    b->kind = kind;
    bool ok = true;
    if (kind == 'S') {
      ok = mat(n("mixer.qkv.weight"), &b->qkv) && mat(n("mixer.o.weight"), &b->o);
    } else if (kind == 'L') {
      ok = mat(n("mixer.qkvg.weight"), &b->qkvg) && mat(n("mixer.decay.weight"), &b->decay) &&
           take(n("mixer.decay.bias"), &b->bias) && take(n("mixer.head_norm.weight"), &b->head_norm) &&
           mat(n("mixer.o.weight"), &b->o);
    } else if (kind == 'G') {
      ok = mat(n("mixer.q.weight"), &b->q) && mat(n("mixer.kv.weight"), &b->kv) &&
           mat(n("mixer.o.weight"), &b->o);
      if (ok && cfg.emb != 0) ok = take(n("mixer.norm_e.weight"), &b->norm_e);
    } else {
      error = std::string("unknown layer type ") + kind;
      return false;
    }
    return ok && take(n("norm1.weight"), &b->norm1) && take(n("norm2.weight"), &b->norm2) &&
           mat(n("mlp.up.weight"), &b->up) && mat(n("mlp.down.weight"), &b->down);
  }

  // Model::load (src/model.rs:226-269), after the tensors have been handed over.
  bool finish() {
    auto blocks = [&](std::vector<Block>* out, const char* name, const std::string& kinds) {
      out->resize(kinds.size());
      for (size_t i = 0; i < kinds.size(); i++)
        if (!load_block(&(*out)[i], std::string(name) + "." + std::to_string(i), kinds[i])) return false;
      return true;
    };
    if (!blocks(&prelude, "prelude", cfg.prelude) || !blocks(&core, "core", cfg.core) ||
        !blocks(&coda, "coda", cfg.coda))
      return false;
    looped = !cfg.core.empty();
    if (looped && !(mat("inject_e.weight", &inject) && mat("loop_embed.weight", &loop_embed)))
      return false;
    if (!mat("embed.weight", &embed) || !take("norm_f.weight", &norm_f)) return false;
    size_t dh = cfg.dh();
    inv_freq.resize(dh / 2);
    for (size_t i = 0; i < dh / 2; i++)
      inv_freq[i] = 1.0f / std::pow(cfg.rope_base, (float)(2 * i) / (float)dh);
    return true;
  }

  // src/model.rs:308-331.
  State new_state(const Block& b) const {
    State st;
    st.kind = b.kind;
    size_t h = cfg.heads, dh = cfg.dh();
    if (b.kind == 'S') {
      st.k.assign(h * cap() * dh, 0.0f);
      st.v.assign(h * cap() * dh, 0.0f);
    } else if (b.kind == 'L') {
      st.s.assign(h * dh * dh, 0.0f);
    } else {
      st.cap = 1u << 13;
      st.k.assign(cfg.kv_heads * st.cap * dh, 0.0f);
      st.v.assign(cfg.kv_heads * st.cap * dh, 0.0f);
      st.prev.assign(cfg.d, 0.0f);
    }
    return st;
  }

  // Doubles a global cache (src/model.rs:384-398).
  void grow(State* st) const {
    size_t kh = cfg.kv_heads, dh = cfg.dh(), old = st->cap, nw = old * 2;
    for (auto* buf : {&st->k, &st->v}) {
      std::vector<float> out(kh * nw * dh, 0.0f);
      for (size_t h = 0; h < kh; h++)
        std::memcpy(out.data() + h * nw * dh, buf->data() + h * old * dh, old * dh * sizeof(float));
      *buf = std::move(out);
    }
    st->cap = nw;
  }

  static void ensure(std::vector<float>* v, size_t n) {
    if (v->size() < n) v->resize(n, 0.0f);
  }

  // columns(): y[i] = x[i][off..off+len] (src/cpu.rs:95-109).
  static void columns(std::vector<float>* y, const std::vector<float>& x, size_t m, size_t stride,
                      size_t off, size_t len) {
    ensure(y, m * len);
    for (size_t i = 0; i < m; i++)
      std::memcpy(y->data() + i * len, x.data() + i * stride + off, len * sizeof(float));
  }

  // Model::block (src/model.rs:400-560).
  void block(const Block& b, State& st, std::vector<float>& x, const std::vector<float>& e0, Scratch& sc,
             size_t pos, size_t m) const {
    const Config& c = cfg;
    size_t d = c.d, heads = c.heads, dh = c.dh();
    float eps = c.eps, scale = 1.0f / std::sqrt((float)dh);
    size_t n = m * d;
    ensure(&sc.n, n);
    op_rms(sc.n.data(), x.data(), b.norm1.data(), m, d, eps);
    bool has_h = true;
    ensure(&sc.h, n);
    ensure(&sc.y, n);
    if (b.kind == 'S') {
      ensure(&sc.mix, m * b.qkv.rows);
      op_linear(sc.mix.data(), b.qkv.w.data(), b.qkv.rows, d, sc.n.data(), m);
      columns(&sc.e, sc.mix, m, 3 * d, 0, d);
      ensure(&sc.q, n);
      op_rope(sc.q.data(), sc.e.data(), sc.cos_.data(), sc.sin_.data(), m, heads, dh);
      columns(&sc.e, sc.mix, m, 3 * d, d, d);
      ensure(&sc.k, n);
      op_rope(sc.k.data(), sc.e.data(), sc.cos_.data(), sc.sin_.data(), m, heads, dh);
      columns(&sc.v, sc.mix, m, 3 * d, 2 * d, d);
      size_t cap = this->cap();
      op_store(st.k.data(), sc.k.data(), pos, m, cap, heads, dh);
      op_store(st.v.data(), sc.v.data(), pos, m, cap, heads, dh);
      Attn a{pos, m, c.window, 0, cap, heads, heads, dh, scale};
      op_attend(sc.y.data(), sc.q.data(), st.k.data(), st.v.data(), a);
      op_linear(sc.h.data(), b.o.w.data(), d, d, sc.y.data(), m);
    } else if (b.kind == 'L') {
      ensure(&sc.mix, m * b.qkvg.rows);
      op_linear(sc.mix.data(), b.qkvg.w.data(), b.qkvg.rows, d, sc.n.data(), m);
      columns(&sc.e, sc.mix, m, 4 * d, 0, d);
      ensure(&sc.q, n);
      op_l2norm(sc.q.data(), sc.e.data(), m * heads, dh);
      columns(&sc.e, sc.mix, m, 4 * d, d, d);
      ensure(&sc.k, n);
      op_l2norm(sc.k.data(), sc.e.data(), m * heads, dh);
      columns(&sc.v, sc.mix, m, 4 * d, 2 * d, d);
      columns(&sc.g, sc.mix, m, 4 * d, 3 * d, d);
      ensure(&sc.dec, m * heads);
      op_linear(sc.dec.data(), b.decay.w.data(), heads, d, sc.n.data(), m);
      op_gla(sc.y.data(), st.s.data(), sc.q.data(), sc.k.data(), sc.v.data(), sc.dec.data(),
             b.bias.data(), m, heads, dh);
      ensure(&sc.y2, n);
      op_rms(sc.y2.data(), sc.y.data(), b.head_norm.data(), m * heads, dh, eps);
      op_silu_mul(sc.y.data(), sc.g.data(), sc.y2.data(), n);
      op_linear(sc.h.data(), b.o.w.data(), d, d, sc.y.data(), m);
    } else {  // 'G'
      if (!b.norm_e.empty()) {
        ensure(&sc.t, n);
        op_rms(sc.t.data(), e0.data(), b.norm_e.data(), m, d, eps);
        op_add(sc.y.data(), sc.n.data(), sc.t.data(), n);
        std::swap(sc.n, sc.y);
        ensure(&sc.y, n);
      }
      size_t kh = c.kv_heads, kd = c.kv_heads * dh;
      ensure(&sc.q, n);
      op_linear(sc.q.data(), b.q.w.data(), d, d, sc.n.data(), m);
      ensure(&sc.mix, m * 2 * kd);
      op_linear(sc.mix.data(), b.kv.w.data(), 2 * kd, d, sc.n.data(), m);
      if (c.logn != 0) {
        float lg = std::log((float)c.logn);
        std::vector<float> f(m);
        for (size_t i = 0; i < m; i++) f[i] = std::log1p((float)(pos + i)) / lg;
        op_scale_rows(sc.y.data(), sc.q.data(), f.data(), m, d);
        std::swap(sc.q, sc.y);
        ensure(&sc.y, n);
      }
      while (pos + m > st.cap) grow(&st);
      if (c.kshift != 0) {
        ensure(&sc.shifted, n);
        std::memcpy(sc.shifted.data(), st.prev.data(), d * sizeof(float));
        if (m > 1) std::memcpy(sc.shifted.data() + d, sc.n.data(), (m - 1) * d * sizeof(float));
        ensure(&sc.prev_kv, m * 2 * kd);
        op_linear(sc.prev_kv.data(), b.kv.w.data(), 2 * kd, d, sc.shifted.data(), m);
        std::memcpy(st.prev.data(), sc.n.data() + (m - 1) * d, d * sizeof(float));
        columns(&sc.k, sc.prev_kv, m, 2 * kd, 0, kd);
      } else {
        columns(&sc.k, sc.mix, m, 2 * kd, 0, kd);
      }
      columns(&sc.v, sc.mix, m, 2 * kd, kd, kd);
      op_store(st.k.data(), sc.k.data(), pos, m, st.cap, kh, dh);
      op_store(st.v.data(), sc.v.data(), pos, m, st.cap, kh, dh);
      size_t far = c.far != 0 ? c.window : 0;
      if (pos + m > far) {
        Attn a{pos, m, 0, far, st.cap, heads, kh, dh, scale};
        op_attend(sc.y.data(), sc.q.data(), st.k.data(), st.v.data(), a);
        op_linear(sc.h.data(), b.o.w.data(), d, d, sc.y.data(), m);
      } else {
        has_h = false;
      }
    }
    ensure(&sc.t, n);
    if (has_h) {
      op_add(sc.t.data(), x.data(), sc.h.data(), n);
      std::swap(x, sc.t);
      ensure(&sc.t, n);
    }
    op_rms(sc.n.data(), x.data(), b.norm2.data(), m, d, eps);
    size_t hidden = b.down.cols;
    ensure(&sc.up, m * 2 * hidden);
    op_linear(sc.up.data(), b.up.w.data(), 2 * hidden, d, sc.n.data(), m);
    columns(&sc.gate, sc.up, m, 2 * hidden, 0, hidden);
    columns(&sc.mid, sc.up, m, 2 * hidden, hidden, hidden);
    ensure(&sc.y, m * hidden);
    op_silu_mul(sc.y.data(), sc.gate.data(), sc.mid.data(), m * hidden);
    op_linear(sc.h.data(), b.down.w.data(), d, hidden, sc.y.data(), m);
    op_add(sc.t.data(), x.data(), sc.h.data(), n);
    std::swap(x, sc.t);
  }

  // Model::advance (src/model.rs:563-640).
  void advance(Session& se, const uint32_t* tokens, size_t m, bool want_logits) const {
    size_t d = cfg.d, pos = se.pos;
    Scratch& sc = se.sc;
    size_t half = cfg.dh() / 2;
    ensure(&sc.cos_, m * half);
    ensure(&sc.sin_, m * half);
    op_rope_table(sc.cos_.data(), sc.sin_.data(), inv_freq.data(), pos, m, half);
    ensure(&se.e0, m * d);
    for (size_t i = 0; i < m; i++)
      std::memcpy(se.e0.data() + i * d, embed.w.data() + (size_t)tokens[i] * d, d * sizeof(float));
    ensure(&se.x, m * d);
    std::memcpy(se.x.data(), se.e0.data(), m * d * sizeof(float));
    for (size_t i = 0; i < prelude.size(); i++) block(prelude[i], se.prelude[i], se.x, se.e0, sc, pos, m);
    if (looped) {
      ensure(&se.e_proj, m * d);
      op_linear(se.e_proj.data(), inject.w.data(), d, d, se.x.data(), m);
      ensure(&se.s, m * d);
      std::memcpy(se.s.data(), se.x.data(), m * d * sizeof(float));
      for (size_t r = 0; r < se.loops; r++) {
        ensure(&sc.t, m * d);
        op_add(sc.t.data(), se.s.data(), se.e_proj.data(), m * d);
        op_add_row(se.x.data(), sc.t.data(), loop_embed.w.data() + r * d, m, d);
        for (size_t i = 0; i < core.size(); i++) block(core[i], se.core[r][i], se.x, se.e0, sc, pos, m);
        if (cfg.damp == 1.0f) {
          std::swap(se.s, se.x);
        } else {
          op_mix(sc.t.data(), se.s.data(), se.x.data(), m * d, cfg.damp);
          std::swap(se.s, sc.t);
        }
        ensure(&se.x, m * d);
      }
      std::swap(se.x, se.s);
    }
    for (size_t i = 0; i < coda.size(); i++) block(coda[i], se.coda[i], se.x, se.e0, sc, pos, m);
    if (want_logits) {
      ensure(&se.last, d);
      std::memcpy(se.last.data(), se.x.data() + (m - 1) * d, d * sizeof(float));
      ensure(&sc.n, d);
      op_rms(sc.n.data(), se.last.data(), norm_f.data(), 1, d, cfg.eps);
      op_linear(se.logits.data(), embed.w.data(), cfg.vocab, d, sc.n.data(), 1);
    }
    se.pos += m;
  }

  // src/model.rs:647-654.
  size_t chunk_at(size_t pos, size_t limit) const {
    size_t chunk = std::min(limit, CHUNK);
    if (cfg.coda.find('G') != std::string::npos || cfg.prelude.find('G') != std::string::npos)
      return std::min(chunk, std::max<size_t>(MAX_SCORES / cfg.heads / (pos + 1), 1));
    return chunk;
  }

  // src/model.rs:658-667.
  void feed(Session& se, const uint32_t* tokens, size_t n, size_t limit) const {
    size_t at = 0;
    while (at < n) {
      size_t m = std::min(chunk_at(se.pos, limit), n - at);
      advance(se, tokens + at, m, at + m == n);
      at += m;
    }
  }

  // src/model.rs:674-690.
  size_t state_bytes(const Session& se) const {
    size_t dh = cfg.dh(), total = 0;
    auto one = [&](const State& st) -> size_t {
      if (st.kind == 'S') return 2 * cfg.heads * cap() * dh;
      if (st.kind == 'L') return cfg.heads * dh * dh;
      return 2 * cfg.kv_heads * se.pos * dh + cfg.d;
    };
    for (auto& st : se.prelude) total += one(st);
    for (auto& l : se.core)
      for (auto& st : l) total += one(st);
    for (auto& st : se.coda) total += one(st);
    return total * 4;
  }
};

// ---------------------------------------------------------------------------
// Sampler (src/sample.rs)
// ---------------------------------------------------------------------------

struct Sampling {
  float temperature, top_p, repeat_penalty;
  uint32_t top_k, repeat_window;
};

// xorshift64* step and its 24-bit float (src/sample.rs:25-30).
float rng_next_f32(uint64_t* st) {
  uint64_t x = *st;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *st = x;
  return (float)((x * 0x2545F4914F6CDD1Dull) >> 40) / (float)(1ull << 24);
}

// total_cmp order for floats, as Rust's f32::total_cmp.
inline int32_t total_key(float f) {
  int32_t b;
  std::memcpy(&b, &f, 4);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// pick (src/sample.rs:33-93) with a canonical candidate order.
uint32_t pick(std::vector<float> logits, const uint32_t* recent, size_t nrecent, const Sampling& s,
              uint64_t* rng) {
  if (s.repeat_penalty != 1.0f) {
    size_t start = nrecent > s.repeat_window ? nrecent - s.repeat_window : 0;
    std::vector<uint32_t> seen(recent + start, recent + nrecent);
    std::sort(seen.begin(), seen.end());
    seen.erase(std::unique(seen.begin(), seen.end()), seen.end());
    for (uint32_t t : seen) {
      float& l = logits[t];
      l = l > 0.0f ? l / s.repeat_penalty : l * s.repeat_penalty;
    }
  }
  if (s.temperature <= 0.0f) {
    size_t b = 0;
    for (size_t i = 0; i < logits.size(); i++)
      if (logits[i] > logits[b]) b = i;
    return (uint32_t)b;
  }
  std::vector<uint32_t> ids(logits.size());
  for (size_t i = 0; i < ids.size(); i++) ids[i] = (uint32_t)i;
  auto before = [&](uint32_t a, uint32_t b) {
    int32_t ka = total_key(logits[a]), kb = total_key(logits[b]);
    return ka != kb ? ka > kb : a < b;
  };
  if (s.top_k > 0 && s.top_k < ids.size()) {
    std::partial_sort(ids.begin(), ids.begin() + s.top_k, ids.end(), before);
    ids.resize(s.top_k);
  } else if (s.top_p < 1.0f) {
    std::sort(ids.begin(), ids.end(), before);
  }
  float top = -INFINITY;
  for (uint32_t i : ids) top = std::max(top, logits[i]);
  std::vector<float> weights(ids.size());
  for (size_t i = 0; i < ids.size(); i++) weights[i] = std::exp((logits[ids[i]] - top) / s.temperature);
  if (s.top_p < 1.0f) {
    float total = 0.0f;
    for (float w : weights) total += w;
    float enough = s.top_p * total, held = 0.0f;
    size_t keep = weights.size();
    for (size_t i = 0; i < weights.size(); i++) {
      held += weights[i];
      if (held >= enough) {
        keep = i + 1;
        break;
      }
    }
    ids.resize(keep);
    weights.resize(keep);
  }
  float total = 0.0f;
  for (float w : weights) total += w;
  float r = rng_next_f32(rng) * total;
  for (size_t i = 0; i < ids.size(); i++) {
    r -= weights[i];
    if (r <= 0.0f) return ids[i];
  }
  return ids.back();
}

thread_local std::string g_error;

}  // namespace

// ---------------------------------------------------------------------------
// C ABI (ctypes), used by tests/ and bench.py only.
// ---------------------------------------------------------------------------

extern "C" {

const char* orc_error() { return g_error.c_str(); }

int orc_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

// ints: vocab, d, heads, kv_heads, window, max_loops, default_loops, logn, kshift, emb, far
// floats: damp, rope_base, eps
void* orc_model_new(const char* prelude, const char* core, const char* coda, const int64_t* ints,
                    const float* floats) {
  auto* m = new Model();
  Config& c = m->cfg;
  c.prelude = prelude;
  c.core = core;
  c.coda = coda;
  c.vocab = ints[0];
  c.d = ints[1];
  c.heads = ints[2];
  c.kv_heads = ints[3];
  c.window = ints[4];
  c.max_loops = ints[5];
  c.default_loops = ints[6];
  c.logn = ints[7];
  c.kshift = ints[8];
  c.emb = ints[9];
  c.far = ints[10];
  c.damp = floats[0];
  c.rope_base = floats[1];
  c.eps = floats[2];
  return m;
}

int orc_model_set(void* model, const char* name, const float* data, const int64_t* shape, int ndim) {
  auto* m = static_cast<Model*>(model);
  std::vector<size_t> sh(shape, shape + ndim);
  size_t n = 1;
  for (size_t s : sh) n *= s;
  m->pending[name] = {sh, std::vector<float>(data, data + n)};
  return 0;
}

int orc_model_finish(void* model) {
  auto* m = static_cast<Model*>(model);
  if (!m->finish()) {
    g_error = m->error;
    return 1;
  }
  return 0;
}

void orc_model_free(void* model) { delete static_cast<Model*>(model); }

void* orc_session_new(void* model, int64_t loops) {
  auto* m = static_cast<Model*>(model);
  auto* se = new Session();
  se->model = m;
  if (m->cfg.core.empty()) {
    se->loops = 0;
  } else {
    se->loops = loops > 0 ? (size_t)loops : m->cfg.default_loops;
    if (se->loops < 1 || se->loops > m->cfg.max_loops) {
      g_error = "loops must be between 1 and " + std::to_string(m->cfg.max_loops);
      delete se;
      return nullptr;
    }
  }
  for (auto& b : m->prelude) se->prelude.push_back(m->new_state(b));
  se->core.resize(se->loops);
  for (size_t r = 0; r < se->loops; r++)
    for (auto& b : m->core) se->core[r].push_back(m->new_state(b));
  for (auto& b : m->coda) se->coda.push_back(m->new_state(b));
  se->logits.assign(m->cfg.vocab, 0.0f);
  return se;
}

void orc_session_free(void* se) { delete static_cast<Session*>(se); }

int64_t orc_session_pos(void* se) { return (int64_t) static_cast<Session*>(se)->pos; }

int orc_feed(void* se_, const uint32_t* ids, int64_t n, int64_t limit) {
  auto* se = static_cast<Session*>(se_);
  for (int64_t i = 0; i < n; i++)
    if (ids[i] >= se->model->cfg.vocab) {
      g_error = "token id out of range";
      return 1;
    }
  se->model->feed(*se, ids, (size_t)n, (size_t)limit);
  return 0;
}

int orc_step(void* se_, uint32_t id) {
  auto* se = static_cast<Session*>(se_);
  if (id >= se->model->cfg.vocab) {
    g_error = "token id out of range";
    return 1;
  }
  se->model->advance(*se, &id, 1, true);
  return 0;
}

int orc_logits(void* se_, float* out) {
  auto* se = static_cast<Session*>(se_);
  std::memcpy(out, se->logits.data(), se->logits.size() * sizeof(float));
  return 0;
}

int64_t orc_state_bytes(void* se_) {
  auto* se = static_cast<Session*>(se_);
  return (int64_t)se->model->state_bytes(*se);
}

// Puts the session at position `pos` with every cache and state filled with
// seeded values of the scale a real run leaves behind, so that a decode step at
// a full window can be timed without first reading a long prompt on the CPU.
int orc_session_fill(void* se_, int64_t pos, uint64_t seed) {
  auto* se = static_cast<Session*>(se_);
  uint64_t st = seed * 0x9E3779B97F4A7C15ull | 1;
  auto fill = [&](std::vector<float>& v, float scale) {
    for (auto& x : v) x = (rng_next_f32(&st) * 2.0f - 1.0f) * scale;
  };
  auto one = [&](State& s) {
    if (s.kind == 'G') {
      while ((size_t)pos > s.cap) se->model->grow(&s);
      fill(s.k, 1.0f);
      fill(s.v, 1.0f);
      fill(s.prev, 1.0f);
    } else if (s.kind == 'S') {
      fill(s.k, 1.0f);
      fill(s.v, 1.0f);
    } else {
      fill(s.s, 0.1f);
    }
  };
  for (auto& s : se->prelude) one(s);
  for (auto& l : se->core)
    for (auto& s : l) one(s);
  for (auto& s : se->coda) one(s);
  se->pos = (size_t)pos;
  return 0;
}

// The session's state arrays in step order (prelude, core per loop, coda);
// per block: S k, v; L s; G k, v, prev — the order of orc_session_fill and of
// the library's slm_session_state_* calls.
static std::vector<std::pair<State*, char>> state_list(Session* se) {
  std::vector<std::pair<State*, char>> out;
  auto one = [&](State& s) {
    if (s.kind == 'S') out.push_back({&s, 'k'}), out.push_back({&s, 'v'});
    else if (s.kind == 'L') out.push_back({&s, 's'});
    else out.push_back({&s, 'k'}), out.push_back({&s, 'v'}), out.push_back({&s, 'p'});
  };
  for (auto& s : se->prelude) one(s);
  for (auto& l : se->core)
    for (auto& s : l) one(s);
  for (auto& s : se->coda) one(s);
  return out;
}

int64_t orc_state_count(void* se_) { return (int64_t)state_list(static_cast<Session*>(se_)).size(); }

// info = {kind, part, cap, floats}; returns the array's data (owned by the session).
float* orc_state_info(void* se_, int64_t i, int64_t* info) {
  auto* se = static_cast<Session*>(se_);
  auto list = state_list(se);
  if (i < 0 || (size_t)i >= list.size()) return nullptr;
  State* st = list[i].first;
  const char part = list[i].second;
  std::vector<float>& v = part == 'k' ? st->k : part == 'v' ? st->v : part == 's' ? st->s : st->prev;
  info[0] = st->kind;
  info[1] = part;
  info[2] = (part == 'k' || part == 'v') ? (int64_t)(st->kind == 'S' ? se->model->cap() : st->cap) : 0;
  info[3] = (int64_t)v.size();
  return v.data();
}

// sampling: temperature, top_p, repeat_penalty; top_k, repeat_window
uint32_t orc_pick(const float* logits, int64_t vocab, const uint32_t* recent, int64_t nrecent,
                  float temperature, uint32_t top_k, float top_p, float repeat_penalty,
                  uint32_t repeat_window, uint64_t* rng_state) {
  Sampling s{temperature, top_p, repeat_penalty, top_k, repeat_window};
  std::vector<float> l(logits, logits + vocab);
  return pick(std::move(l), recent, (size_t)nrecent, s, rng_state);
}

uint64_t orc_rng_new(uint64_t seed) { return seed * 0x9E3779B97F4A7C15ull | 1; }  // src/sample.rs:21-23
float orc_rng_next(uint64_t* st) { return rng_next_f32(st); }

// Op-level entry points, one per `Ops` method, on host arrays.
void orc_linear(float* y, const float* w, int64_t rows, int64_t cols, const float* x, int64_t m) {
  op_linear(y, w, rows, cols, x, m);
}
void orc_rms(float* y, const float* x, const float* w, int64_t groups, int64_t size, float eps) {
  op_rms(y, x, w, groups, size, eps);
}
void orc_silu_mul(float* y, const float* g, const float* u, int64_t n) { op_silu_mul(y, g, u, n); }
void orc_rope_table(float* c, float* s, const float* inv, int64_t pos, int64_t m, int64_t half) {
  op_rope_table(c, s, inv, pos, m, half);
}
void orc_rope(float* y, const float* x, const float* c, const float* s, int64_t m, int64_t heads,
              int64_t dh) {
  op_rope(y, x, c, s, m, heads, dh);
}
void orc_l2norm(float* y, const float* x, int64_t heads, int64_t dh) { op_l2norm(y, x, heads, dh); }
void orc_gla(float* y, float* s, const float* q, const float* k, const float* v, const float* decay,
             const float* bias, int64_t m, int64_t heads, int64_t dh) {
  op_gla(y, s, q, k, v, decay, bias, m, heads, dh);
}
void orc_store(float* cache, const float* src, int64_t pos, int64_t m, int64_t cap, int64_t heads,
               int64_t dh) {
  op_store(cache, src, pos, m, cap, heads, dh);
}
// reach 0 = unbounded
void orc_attend(float* y, const float* q, const float* k, const float* v, int64_t pos, int64_t m,
                int64_t reach, int64_t gap, int64_t cap, int64_t heads, int64_t key_heads, int64_t dh,
                float scale) {
  Attn a{(size_t)pos, (size_t)m, (size_t)reach, (size_t)gap, (size_t)cap, (size_t)heads,
         (size_t)key_heads, (size_t)dh, scale};
  op_attend(y, q, k, v, a);
}
void orc_add(float* y, const float* a, const float* b, int64_t n) { op_add(y, a, b, n); }
void orc_add_row(float* y, const float* x, const float* row, int64_t m, int64_t d) {
  op_add_row(y, x, row, m, d);
}
void orc_scale_rows(float* y, const float* x, const float* f, int64_t m, int64_t d) {
  op_scale_rows(y, x, f, m, d);
}
void orc_mix(float* y, const float* a, const float* b, int64_t n, float t) { op_mix(y, a, b, n, t); }

}  // extern "C"
