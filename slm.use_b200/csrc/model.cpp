// The looped hybrid model on the device: weights, per-session state and the
// m-token advance (reference Model/Session, src/model.rs:196-690), with the
// fused kernels of this library in place of the reference's ~17 launches per
// block.  The m = 1 step is captured once as a CUDA graph and replayed: every
// kernel reads the position from device memory and the next token id from a
// device slot that the on-device sampler writes.
#include <atomic>
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "capi.hpp"
#include "common.cuh"
#include "kernels.cuh"
#include "loader.hpp"
#include "mega.cuh"

namespace slm {
namespace mega {
size_t smem_bytes();
void prepare();
int blocks_per_sm();
void launch(const Plan& plan, int grid, cudaStream_t st);
}  // namespace mega
}  // namespace slm

namespace slm {

constexpr size_t CHUNK = 256;            // src/model.rs:27
constexpr size_t MAX_SCORES = 1u << 28;  // src/model.rs:30
constexpr size_t G_CAP0 = 1u << 13;      // first global cache capacity, src/model.rs:320
#ifndef SLM_L2MODE
#define SLM_L2MODE 1
#endif
constexpr int kL2ModeDefault = SLM_L2MODE;  // L2 priority mode of the persistent step's copies

struct Mat {
  const float* w = nullptr;
  size_t rows = 0, cols = 0;
  const void* planes = nullptr;  // bf16 parts for chunk linears (gemm_bf16x3.cu), in the model's plane arena
  const float* t = nullptr;      // down only: the transpose ([cols][rows]) read by the fused decode MLP
  const float* hb = nullptr;     // o of S and L blocks: per-head column blocks [heads][rows][dh] (mixer + o fused)
  // bf16 copies of w, t and hb for the persistent step's bf16 plans (SLM_OPT_BF16), or null.
  const void *w16 = nullptr, *t16 = nullptr, *hb16 = nullptr;
};

struct Block {
  char kind = 'S';
  const float *norm1 = nullptr, *norm2 = nullptr;
  Mat up, down;
  Mat qkv, o;                                               // S (o: every kind)
  Mat qkvg, decay;                                          // L
  const float *bias = nullptr, *head_norm = nullptr;        // L
  Mat q, kv;                                                // G
  const float* norm_e = nullptr;                            // G with global_emb
};

struct LState {
  char kind = 'S';
  float *k = nullptr, *v = nullptr, *s = nullptr, *prev = nullptr;
  size_t cap = 0;
};

}  // namespace slm

using namespace slm;

struct slm_model {
  slm_ctx* ctx = nullptr;
  Config cfg;
  float* arena = nullptr;
  void* planes = nullptr;  // bf16x3 parts of the block and inject matrices
  float* tarena = nullptr;  // transposed down matrices (Mat::t)
  void* arena16 = nullptr;  // bf16 copies of the persistent step's matrices (Mat::w16, t16, hb16), built on request
  std::vector<Block> prelude, core, coda;
  Mat embed, inject, loop_embed;
  bool looped = false;
  const float* norm_f = nullptr;
  const float* inv_freq = nullptr;
  size_t params = 0, hidden = 0, mix_cols = 0;
  // Live sessions; slm_model_free while some live marks the model closing and
  // the last session's free frees it (as slm_ctx does for its children).
  int refs = 0;
  bool closing = false;
};

struct slm_session {
  slm_model* model = nullptr;
  slm_ctx* ctx = nullptr;
  size_t loops = 0, pos = 0;
  std::vector<LState> pre, coda;
  std::vector<std::vector<LState>> core;
  std::vector<float*> owned;  // device allocations of this session
  float *xa = nullptr, *xb = nullptr, *e0 = nullptr, *e_proj = nullptr, *n = nullptr, *mix = nullptr, *q = nullptr,
        *kb = nullptr, *kin = nullptr, *kvs = nullptr, *y = nullptr, *mid = nullptr, *dec = nullptr, *part = nullptr,
        *logits = nullptr, *work = nullptr, *nlast = nullptr, *upbuf = nullptr;
  void* nplanes = nullptr;  // bf16x3 planes of `n` for the wide chunk linears (when the model has split weights)
  long long* pos_dev = nullptr;
  uint32_t* ids_dev = nullptr;
  unsigned long long* rng_dev = nullptr;
  uint32_t* out_dev = nullptr;
  uint32_t* hist_dev = nullptr;
  size_t hist_cap = 0;
  uint32_t* outs_dev = nullptr;
  size_t outs_cap = 0;
  cudaGraphExec_t graph = nullptr;
  bool use_graph = true;
  bool capturing = false;
  int64_t step_kernels = 0;  // kernel nodes of the captured step
  int64_t graphs = 0;
  // Persistent decode kernel (decode_mega.cu)
  bool mega_ok = false, use_mega = false;
  std::string mega_why;                  // why the kernel does not apply, if it does not
  slm::mega::Plan plan_host{};
  slm::mega::Phase* phases_dev = nullptr;
  float* xc = nullptr;
  int grid = 0;
  unsigned long long* trace = nullptr;  // per-phase timeline of the last step (SLM_OPT_TRACE)
  unsigned* attn_count = nullptr;        // per-head arrival counters of the attention phases
  float* attn_part = nullptr;            // attention partials of the persistent step
  bool fuse_mlp = false;                 // the persistent step runs each MLP as one phase
  bool fuse_ao = false;                  // … and the o projection of S blocks in the attention phase
  unsigned long long* fx = nullptr;      // counted fixed-point slots of those phases (two parity sets)
  size_t fx_set_words = 0;               // words of one set (the stride between the sets)
  unsigned* epoch = nullptr;             // the persistent step's counter (tags and set parity)
  // Tagged words the persistent step's CTAs pass to each other within a step:
  // q | k | v of the position, attention partials, GLA inputs (q|k|v|g rows,
  // decay), the inject output.
  unsigned long long *tq = nullptr, *tpart = nullptr, *tmix = nullptr, *tdec = nullptr, *te = nullptr;
  bool plan_stale = false;               // a global cache moved: the phase descriptors need refreshing
  bool keys_stale = false;               // state was written from the host: the next shifted keys need recomputing
  bool wbf16 = false;                    // the persistent step reads bf16 copies of its matrices
  int in_batches = 0;                    // batches holding this session
  uint32_t* argmax_dev = nullptr;        // the persistent step's arg-max of its logits
  unsigned* merge_cnt = nullptr;         // attention slice counters of the graph path (zero between launches)
  bool argmax_valid = false;             // the logits come from a persistent step
  unsigned long long mbox_want = 0;      // mailbox sequence number of this session's pending slm_step (0: none)
  // The armed launch this session's last slm_step fed (sequence number and
  // token), kept so a launch that ran out of time before the token reached
  // it can be replaced by a plain one.
  unsigned long long fed_seq = 0;
  uint32_t fed_id = 0;
  bool greedy_loop = false;  // the last slm_sample took the mailbox: slm_step arms the next step
  // Pinned host words for the per-token transfers (ids in and out, RNG state).
  struct HostIO {
    uint32_t id_in, id_out;
    unsigned long long rng_in, rng_out;
  }* io = nullptr;
  cudaEvent_t io_event = nullptr;  // after the last copy that reads io
  bool io_busy = false;
};

// Several sessions of one model stepped together (one token each per step):
// the weights are read once per step for all of them, each row keeps its own
// caches, GLA state and position (decode_batch below).
struct slm_batch {
  slm_model* model = nullptr;
  slm_ctx* ctx = nullptr;
  std::vector<slm_session*> ses;
  size_t n = 0;
  std::vector<void*> owned;
  float *xa = nullptr, *xb = nullptr, *e0 = nullptr, *e_proj = nullptr, *nb = nullptr, *mix = nullptr, *q = nullptr,
        *kb = nullptr, *y = nullptr, *mid = nullptr, *dec = nullptr, *part = nullptr, *logits = nullptr,
        *upbuf = nullptr;
  uint32_t* ids = nullptr;           // [n] this step's tokens (the arg-max writes the next ones)
  unsigned* merge_cnt = nullptr;     // [heads·n] attention slice counters (zero between launches)
  long long** posr = nullptr;        // [n] the sessions' device positions
  std::vector<float**> tab;          // per layer instance, in step order: [4][n] k, v, s, prev pointers
  std::vector<long long*> caps;      // per layer instance: [n] cache capacities (global caches differ by session)
  float* kvs = nullptr;              // [n][kv_heads·dh] shifted keys of global layers
  unsigned* out_index = nullptr;     // steps taken since the last reset
  uint32_t* outs = nullptr;          // [outs_cap][n] picked ids
  size_t outs_cap = 0;
  int nsplit = 1;
  int gsplit = 1;  // attention splits of global layers (their reach grows with the position)
  cudaGraphExec_t graph = nullptr;
  unsigned long long graph_ws_gen = 0;  // the context's GEMM workspace generation the graph holds
  bool capturing = false;
  // Per-row sampling (slm_batch_sample_decode): the step ends with one
  // sampler CTA per row instead of the greedy arg-max; its own graph.
  cudaGraphExec_t graph_s = nullptr;
  unsigned long long graph_s_ws_gen = 0;
  SampleArgs* srows = nullptr;          // [n] device: each row's settings, history and state
  float* swork = nullptr;               // [n][3·vocab] sampler work space
  uint32_t* shist = nullptr;            // [n][shist_cap] histories (penalty windows), sampled ids appended
  size_t shist_cap = 0;
  unsigned long long* srng = nullptr;   // [n] xorshift64* states
};

namespace slm {
namespace {

struct Uploader {
  std::vector<std::pair<const float*, size_t>> items;  // host data, floats
  std::vector<size_t> offsets;
  size_t total = 0;
  size_t add(const float* data, size_t n) {
    size_t off = total;
    offsets.push_back(off);
    items.emplace_back(data, n);
    total += (n + 63) / 64 * 64;  // 256-byte aligned tensors
    return off;
  }
};

struct Loading {
  Tensors t;
  Uploader up;
  std::vector<std::pair<const float**, size_t>> fix;  // pointers to patch with arena offsets
  std::string error;
};

// Copies every tensor of `up` to its offset in `arena` (device) through two
// pinned staging buffers: the host copies chunk i + 1 into one while the copy
// engine moves chunk i out of the other, on the context's stream.
void upload_pinned(slm_ctx* ctx, float* arena, const Uploader& up) {
  constexpr size_t kChunk = size_t(16) << 20;  // bytes per staging buffer
  cudaStream_t s = ctx->stream;
  char* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  struct Release {
    char** st;
    cudaEvent_t* ev;
    ~Release() {
      for (int i = 0; i < 2; i++) {
        if (ev[i]) cudaEventSynchronize(ev[i]), cudaEventDestroy(ev[i]);
        if (st[i]) cudaFreeHost(st[i]);
      }
    }
  } rel{stage, done};
  for (int i = 0; i < 2; i++) {
    SLM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&stage[i]), kChunk, cudaHostAllocDefault));
    SLM_CUDA(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
  }
  int b = 0;
  bool used[2] = {false, false};
  for (size_t t = 0; t < up.items.size(); t++) {
    const char* src = reinterpret_cast<const char*>(up.items[t].first);
    char* dst = reinterpret_cast<char*>(arena + up.offsets[t]);
    size_t left = up.items[t].second * sizeof(float);
    while (left > 0) {
      const size_t n = std::min(left, kChunk);
      if (used[b]) SLM_CUDA(cudaEventSynchronize(done[b]));  // its previous copy has left the buffer
      std::memcpy(stage[b], src, n);
      SLM_CUDA(cudaMemcpyAsync(dst, stage[b], n, cudaMemcpyHostToDevice, s));
      SLM_CUDA(cudaEventRecord(done[b], s));
      used[b] = true;
      src += n, dst += n, left -= n;
      b ^= 1;
    }
  }
  SLM_CUDA(cudaStreamSynchronize(s));
}

const TensorView& take(Loading& L, const std::string& name) {
  auto it = L.t.map.find(name);
  if (it == L.t.map.end()) fail(SLM_ERR_IO, "missing weight " + name);
  return it->second;
}

void vec(Loading& L, const std::string& name, const float** dst, size_t want) {
  const TensorView& tv = take(L, name);
  if (want && tv.count != want) fail(SLM_ERR_IO, name + ": expected " + std::to_string(want) + " values");
  size_t off = L.up.add(tv.data, tv.count);
  L.fix.emplace_back(dst, off);
}

void mat(Loading& L, const std::string& name, Mat* m) {
  const TensorView& tv = take(L, name);
  if (tv.shape.size() != 2) fail(SLM_ERR_IO, name + ": expected a matrix");
  m->rows = tv.shape[0];
  m->cols = tv.shape[1];
  size_t off = L.up.add(tv.data, tv.count);
  L.fix.emplace_back(&m->w, off);
}

// Block::load (src/model.rs:114-153).
void load_block(Loading& L, const Config& c, Block* b, const std::string& prefix, char kind) {
  auto n = [&](const char* s) { return prefix + "." + s; };
  b->kind = kind;
  size_t d = c.d;
  if (kind == 'S') {
    mat(L, n("mixer.qkv.weight"), &b->qkv);
    mat(L, n("mixer.o.weight"), &b->o);
    if (b->qkv.rows != 3 * d || b->qkv.cols != d) fail(SLM_ERR_IO, prefix + ": qkv must be 3d × d");
  } else if (kind == 'L') {
    mat(L, n("mixer.qkvg.weight"), &b->qkvg);
    mat(L, n("mixer.decay.weight"), &b->decay);
    vec(L, n("mixer.decay.bias"), &b->bias, c.heads);
    vec(L, n("mixer.head_norm.weight"), &b->head_norm, c.dh());
    mat(L, n("mixer.o.weight"), &b->o);
    if (b->qkvg.rows != 4 * d || b->qkvg.cols != d) fail(SLM_ERR_IO, prefix + ": qkvg must be 4d × d");
    if (b->decay.rows != c.heads || b->decay.cols != d) fail(SLM_ERR_IO, prefix + ": decay must be heads × d");
  } else if (kind == 'G') {
    mat(L, n("mixer.q.weight"), &b->q);
    mat(L, n("mixer.kv.weight"), &b->kv);
    mat(L, n("mixer.o.weight"), &b->o);
    if (c.emb != 0) vec(L, n("mixer.norm_e.weight"), &b->norm_e, d);
    if (b->kv.rows != 2 * c.kv_heads * c.dh() || b->kv.cols != d) fail(SLM_ERR_IO, prefix + ": kv has the wrong shape");
  } else {
    fail(SLM_ERR_IO, std::string("unknown layer type ") + kind);
  }
  if (b->o.rows != d || b->o.cols != d) fail(SLM_ERR_IO, prefix + ": o must be d × d");
  vec(L, n("norm1.weight"), &b->norm1, d);
  vec(L, n("norm2.weight"), &b->norm2, d);
  mat(L, n("mlp.up.weight"), &b->up);
  mat(L, n("mlp.down.weight"), &b->down);
  if (b->up.cols != d || b->down.rows != d || b->up.rows != 2 * b->down.cols)
    fail(SLM_ERR_IO, prefix + ": mlp shapes do not match");
}

size_t mat_params(const Mat& m) { return m.rows * m.cols; }

void* alloc_zero(slm_session* se, size_t bytes) {
  void* p = dev_alloc(bytes);
  se->owned.push_back(static_cast<float*>(p));
  SLM_CUDA(cudaMemsetAsync(p, 0, bytes, se->ctx->stream));
  return p;
}

LState new_state(slm_session* se, const Block& b) {
  const Config& c = se->model->cfg;
  size_t h = c.heads, dh = c.dh();
  LState st;
  st.kind = b.kind;
  if (b.kind == 'S') {
    size_t cap = c.window + CHUNK;  // Model::cap, src/model.rs:304-306
    st.cap = cap;
    st.k = static_cast<float*>(alloc_zero(se, h * cap * dh * sizeof(float)));
    st.v = static_cast<float*>(alloc_zero(se, h * cap * dh * sizeof(float)));
  } else if (b.kind == 'L') {
    st.s = static_cast<float*>(alloc_zero(se, h * dh * dh * sizeof(float)));
  } else {
    st.cap = G_CAP0;
    st.k = static_cast<float*>(dev_alloc(c.kv_heads * st.cap * dh * sizeof(float)));
    st.v = static_cast<float*>(dev_alloc(c.kv_heads * st.cap * dh * sizeof(float)));
    SLM_CUDA(cudaMemsetAsync(st.k, 0, c.kv_heads * st.cap * dh * sizeof(float), se->ctx->stream));
    SLM_CUDA(cudaMemsetAsync(st.v, 0, c.kv_heads * st.cap * dh * sizeof(float), se->ctx->stream));
    st.prev = static_cast<float*>(alloc_zero(se, c.d * sizeof(float)));
  }
  return st;
}

void drop_graph(slm_session* se) {
  if (se->graph) {
    cudaGraphExecDestroy(se->graph);
    se->graph = nullptr;
  }
}

// Doubles a global cache on the device (the reference moves it through the
// host, src/model.rs:384-398).  Positions never wrap in a global cache.
void grow(slm_session* se, LState& st) {
  const Config& c = se->model->cfg;
  size_t kh = c.kv_heads, dh = c.dh(), old = st.cap, nw = old * 2;
  cudaStream_t s = se->ctx->stream;
  for (float** buf : {&st.k, &st.v}) {
    float* p = static_cast<float*>(dev_alloc(kh * nw * dh * sizeof(float)));
    SLM_CUDA(cudaMemsetAsync(p, 0, kh * nw * dh * sizeof(float), s));
    SLM_CUDA(cudaMemcpy2DAsync(p, nw * dh * sizeof(float), *buf, old * dh * sizeof(float), old * dh * sizeof(float), kh,
                               cudaMemcpyDeviceToDevice, s));
    SLM_CUDA(cudaStreamSynchronize(s));
    dev_free(*buf);
    *buf = p;
  }
  st.cap = nw;
  drop_graph(se);
  se->plan_stale = true;  // the persistent step's descriptors hold the old cache
}

void ensure_caps(slm_session* se, size_t m) {
  // With kshift a step also stores the next position's key (W_k · n of its
  // last token), so a global cache keeps one slot beyond the step.
  const size_t extra = se->model->cfg.kshift ? 1 : 0;
  auto one = [&](LState& st) {
    if (st.kind == 'G')
      while (se->pos + m + extra > st.cap) grow(se, st);
  };
  for (auto& st : se->pre) one(st);
  for (auto& l : se->core)
    for (auto& st : l) one(st);
  for (auto& st : se->coda) one(st);
}

thread_local slm_ctx* g_ctx_for_linear = nullptr;  // set by the driver around each advance
thread_local bool g_capturing = false;

void run_linear(cudaStream_t s, const Mat& w, const float* x, int ldx, int m, float* y, int ldy, int epi,
                const float* res = nullptr, int ldres = 0, size_t rows = 0, const void* xplanes = nullptr) {
  LinearArgs a;
  a.w = w.w;
  a.rows = (int)(rows ? rows : w.rows);
  a.cols = (int)w.cols;
  a.x = x;
  a.ldx = ldx;
  a.m = m;
  a.y = y;
  a.ldy = ldy;
  a.res = res;
  a.ldres = ldres;
  a.epi = epi;
  a.wplanes = w.planes;
  a.xplanes = xplanes;
  if (g_ctx_for_linear) gemm_workspace(g_ctx_for_linear, a, g_capturing);
  linear(a, s);
}

// Model::block (src/model.rs:400-560) for m tokens, x updated in place.
void block(slm_session* se, const Block& b, LState& st, float* x, size_t m) {
  slm_model* md = se->model;
  const Config& c = md->cfg;
  cudaStream_t s = se->ctx->stream;
  const size_t d = c.d, heads = c.heads, dh = c.dh();
  const float scale = 1.0f / std::sqrt((float)dh);
  const int im = (int)m, id = (int)d;
  // Chunks: the normalised input also gets its bf16x3 planes for the wide
  // linears that read it (qkv, qkvg, up), in the same kernel.
  const bool split = m > 64 && se->nplanes && b.kind != 'G';
  if (split)
    b3_rms_split(se->n, se->nplanes, x, b.norm1, m, d, c.eps, s);
  else
    ew_rms(se->n, x, b.norm1, m, d, c.eps, nullptr, s);
  const void* np = split ? se->nplanes : nullptr;
  bool has_h = true;
  if (b.kind == 'S') {
    run_linear(s, b.qkv, se->n, id, im, se->mix, (int)(3 * d), EPI_STORE, nullptr, 0, 0, np);
    ew_rope_store(se->mix, 3 * d, md->inv_freq, se->pos_dev, m, heads, dh, st.cap, se->q, st.k, st.v, s);
    AttnGeom g{im, (long long)c.window, 0, (long long)st.cap, (int)heads, (int)heads, (int)dh, scale};
    g.err = se->ctx->err;
    int ns = attn_splits(g, (long long)(c.window + m - 1));
    attention(se->q, id, st.k, st.v, g, se->pos_dev, ns, se->part, se->y, id, s, se->merge_cnt);
  } else if (b.kind == 'L') {
    run_linear(s, b.qkvg, se->n, id, im, se->mix, (int)(4 * d), EPI_STORE, nullptr, 0, 0, np);
    run_linear(s, b.decay, se->n, id, im, se->dec, (int)heads, EPI_STORE);
    ew_l2norm(se->q, d, se->mix, 4 * d, m, heads, dh, s);
    ew_l2norm(se->kb, d, se->mix + d, 4 * d, m, heads, dh, s);
    GlaArgs a{};
    a.S = st.s;
    a.q = se->q, a.ldq = id;
    a.k = se->kb, a.ldk = id;
    a.v = se->mix + 2 * d, a.ldv = (int)(4 * d);
    a.g = se->mix + 3 * d, a.ldg = (int)(4 * d);
    a.dec = se->dec, a.lddec = (int)heads;
    a.bias = b.bias, a.hnw = b.head_norm, a.eps = c.eps;
    a.m = im, a.heads = (int)heads, a.dh = (int)dh;
    a.out = se->y, a.ldo = id, a.fuse = 1;
    gla(a, s);
  } else {
    if (b.norm_e) ew_rms(se->n, se->e0, b.norm_e, m, d, c.eps, se->n, s);  // n += rms(e0)·w_e
    const size_t kh = c.kv_heads, kd = kh * dh;
    run_linear(s, b.q, se->n, id, im, se->q, id, EPI_STORE);
    run_linear(s, b.kv, se->n, id, im, se->mix, (int)(2 * kd), EPI_STORE);
    const float* keys = se->mix;
    size_t ldk = 2 * kd;
    if (c.kshift) {
      ew_shift(se->kin, st.prev, se->n, m, d, s);
      run_linear(s, b.kv, se->kin, id, im, se->kvs, (int)kd, EPI_STORE, nullptr, 0, kd);  // key rows only
      ew_copy(st.prev, se->n + (m - 1) * d, d, s);
      keys = se->kvs;
      ldk = kd;
    }
    float inv_log = c.logn ? 1.0f / std::log((float)c.logn) : 0.0f;
    ew_g_post(se->q, d, m, se->pos_dev, inv_log, c.logn ? 1 : 0, keys, ldk, se->mix + kd, 2 * kd, kd, st.cap, dh,
              st.k, st.v, s);
    if (c.kshift) {
      // The next position's key, W_k · n of this chunk's last token (now in
      // prev): the persistent step relies on it being in the cache already,
      // and the next chunk overwrites it with the same value.
      run_linear(s, b.kv, st.prev, id, 1, se->kvs, (int)kd, EPI_STORE, nullptr, 0, kd);
      ew_store_next(st.k, se->kvs, se->pos_dev, (long long)m, kh, dh, st.cap, s);
    }
    size_t far = c.far ? c.window : 0;
    if (se->capturing || se->pos + m > far) {
      AttnGeom g{im, 0, (long long)far, (long long)st.cap, (int)heads, (int)kh, (int)dh, scale};
      g.err = se->ctx->err;
      long long span = (long long)(se->capturing ? st.cap : se->pos + m);
      int ns = attn_splits(g, span);
      attention(se->q, id, st.k, st.v, g, se->pos_dev, ns, se->part, se->y, id, s, se->merge_cnt);
    } else {
      has_h = false;
    }
  }
  if (has_h) run_linear(s, b.o, se->y, id, im, x, id, EPI_ADD, x, id);  // x += o·y
  const bool split2 = m > 64 && se->nplanes;
  if (split2)
    b3_rms_split(se->n, se->nplanes, x, b.norm2, m, d, c.eps, s);
  else
    ew_rms(se->n, x, b.norm2, m, d, c.eps, nullptr, s);
  const size_t hidden = b.down.cols;
  if (m > 8 && hidden % 4 == 0) {
    // Chunks: the [m][2F] product on the tensor cores, then the gate.
    run_linear(s, b.up, se->n, id, im, se->upbuf, (int)(2 * hidden), EPI_STORE, nullptr, 0, 0,
               split2 ? se->nplanes : nullptr);
    ew_silu_pair(se->mid, se->upbuf, m, hidden, s);
  } else {
    run_linear(s, b.up, se->n, id, im, se->mid, (int)hidden, EPI_SILU);  // silu(gate)·amp
  }
  run_linear(s, b.down, se->mid, (int)hidden, im, x, id, EPI_ADD, x, id);       // x += down·mid
}

// Model::advance (src/model.rs:563-640).  Ids are already in se->ids_dev.
void advance(slm_session* se, size_t m, bool want_logits) {
  se->argmax_valid = false;
  g_ctx_for_linear = se->ctx;
  g_capturing = se->capturing;
  slm_model* md = se->model;
  const Config& c = md->cfg;
  cudaStream_t s = se->ctx->stream;
  const size_t d = c.d;
  float* x = se->xa;
  ew_embed(se->e0, x, md->embed.w, se->ids_dev, m, d, c.vocab, se->ctx->err, s);
  for (size_t i = 0; i < md->prelude.size(); i++) block(se, md->prelude[i], se->pre[i], x, m);
  if (md->looped) {
    run_linear(s, md->inject, x, (int)d, (int)m, se->e_proj, (int)d, EPI_STORE);
    float* sbuf = x;  // s = x (no copy: the loop writes the other buffer)
    for (size_t r = 0; r < se->loops; r++) {
      const float* le = md->loop_embed.w + r * d;
      float* xr = (sbuf == se->xa) ? se->xb : se->xa;
      ew_loop_in(xr, sbuf, se->e_proj, le, m, d, s);
      for (size_t i = 0; i < md->core.size(); i++) block(se, md->core[i], se->core[r][i], xr, m);
      if (c.damp == 1.0f) {
        sbuf = xr;
      } else {
        ew_mix(sbuf, sbuf, xr, m * d, c.damp, s);  // s = s + damp·(x − s), in place
      }
    }
    x = sbuf;
  }
  for (size_t i = 0; i < md->coda.size(); i++) block(se, md->coda[i], se->coda[i], x, m);
  if (want_logits) {
    ew_rms(se->nlast, x + (m - 1) * d, md->norm_f, 1, d, c.eps, nullptr, s);
    run_linear(s, md->embed, se->nlast, (int)d, 1, se->logits, (int)c.vocab, EPI_STORE);  // tied head
  }
  ew_advance_pos(se->pos_dev, (long long)m, s);
  se->pos += m;
}

// SLM_MEGA_FUSE_MLP=0 keeps the MLP of the persistent step as two phases
// (gate/up, then down) with float residual adds; the default fuses them.
bool fuse_mlp_enabled() {
  const char* e = std::getenv("SLM_MEGA_FUSE_MLP");
  return !(e && e[0] == '0');
}

// SLM_MEGA_FUSE_ATTN_O=0 keeps the o projection of S and L blocks as its own
// phase (the default runs it in the attention or GLA phase).
bool fuse_attn_o_enabled() {
  const char* e = std::getenv("SLM_MEGA_FUSE_ATTN_O");
  return !(e && e[0] == '0');
}

// L2 priority of the persistent step's bulk copies (SLM_MEGA_L2MODE): 0 none,
// 1 loop-block weights evict_last and the rest evict_first, 2 loop-block
// weights evict_last and the rest normal.
int l2mode_setting() {
  const char* e = std::getenv("SLM_MEGA_L2MODE");
  const int v = e && *e ? std::atoi(e) : kL2ModeDefault;
  return v < 0 || v > 2 ? 0 : v;
}

// SLM_MEGA_MLP_CTA=1 splits each fused MLP tile's rows over the CTA's warps
// (a CTA barrier per tile) instead of giving each warp whole hidden units.
bool mlp_cta_setting() {
  const char* e = std::getenv("SLM_MEGA_MLP_CTA");
  return e && e[0] == '1';
}

// Why the persistent decode kernel cannot run this model ("" if it can).
std::string mega_unsupported(const slm_model* md) {
  const Config& c = md->cfg;
  if (c.dh() != (size_t)mega::kDH) return "head size is not 64";
  // A GEMV row is split over one warp (≤ 1536 columns) or two; each warp holds
  // cols/128 (per split) float4 of the input in registers: 1, 2, 3, 4, 6, 8 or 12.
  auto cols_ok = [](size_t cols) {
    size_t k = cols / (cols > 1536 ? 2 : 1) / 128;
    return cols % (cols > 1536 ? 256 : 128) == 0 && (k <= 4 || k == 6 || k == 8 || k == 12);
  };
  if (!cols_ok(c.d) || c.d > (size_t)mega::kMaxD) return "d_model must be 128·{1,2,3,4,6,8} (at most 1024)";
  if (!cols_ok(md->hidden) || md->hidden > (size_t)mega::kMaxCols) return "FFN width must suit the GEMV split, <= 3072";
  if (c.damp != 1.0f) return "damp != 1";
  if (c.prelude.empty()) return "no prelude block";
  const bool has_g = (c.prelude + c.core + c.coda).find('G') != std::string::npos;
  if (has_g) {
    // A global block forms its own input (x, and e0 for global_emb): it cannot
    // be the first block of the prelude or of the loop.
    if (c.prelude[0] == 'G' || (!c.core.empty() && c.core[0] == 'G'))
      return "a global-attention layer opens the prelude or the loop";
    if (c.kv_heads == 0 || c.heads % c.kv_heads != 0 || c.heads / c.kv_heads > 3)
      return "global layers need heads / kv_heads in 1..3";
  }
  return "";
}

// bf16 copies (round to nearest even) of every matrix the persistent step
// streams, in one device arena: each block's projections, o (row-major and
// per-head blocks), up, down (transposed), the inject matrix and the tied
// head.  Built once per model, on the first request.
void build_bf16(slm_model* md) {
  if (md->arena16) return;
  std::vector<std::pair<const float*, const void**>> parts;
  std::vector<size_t> sizes;
  auto add = [&](const float* src, const void** dst, size_t n) {
    if (!src) return;
    parts.emplace_back(src, dst);
    sizes.push_back(n);
  };
  auto mat = [&](Mat& m) {
    const size_t n = m.rows * m.cols;
    add(m.w, &m.w16, n);
    add(m.t, &m.t16, n);
    add(m.hb, &m.hb16, n);
  };
  for (auto* bs : {&md->prelude, &md->core, &md->coda})
    for (auto& b : *bs)
      for (Mat* m : {&b.qkv, &b.o, &b.up, &b.down, &b.qkvg, &b.decay, &b.q, &b.kv}) mat(*m);
  mat(md->inject);
  mat(md->embed);
  size_t total = 0;
  for (size_t n : sizes) total += (n * 2 + 255) / 256 * 256;
  char* at = static_cast<char*>(dev_alloc(total));
  md->arena16 = at;
  cudaStream_t s = md->ctx->stream;
  for (size_t i = 0; i < parts.size(); i++) {
    ew_to_bf16(at, parts[i].first, sizes[i], s);
    *parts[i].second = at;
    at += (sizes[i] * 2 + 255) / 256 * 256;
  }
  SLM_CUDA(cudaStreamSynchronize(s));
}

// Why the persistent step cannot read bf16 weights for this session ("" if it can).
std::string bf16_unsupported(const slm_session* se) {
  const Config& c = se->model->cfg;
  if (!se->mega_ok) return "the persistent decode kernel is unavailable: " + se->mega_why;
  if (!se->fuse_mlp || !se->fuse_ao) return "bf16 weights need the fused MLP and mixer phases";
  if (se->plan_host.mlp_cta) return "bf16 weights need d_model <= 768";
  if (c.d % 256 != 0) return "bf16 weights need d_model a multiple of 256";
  return "";
}

// The m = 1 step as phases (decode_mega.cu), for this session's buffers.
// refresh: only regenerate the phase descriptors (a global cache moved or
// grew); counters, outputs and the rest of the plan stay.
void build_plan(slm_session* se, bool refresh = false) {
  using namespace mega;
  slm_model* md = se->model;
  const Config& c = md->cfg;
  const int G = se->grid;
  const int d = (int)c.d, H = (int)c.heads;
  // The matrices the step streams: f32, or their bf16 copies (SLM_OPT_BF16).
  const bool bf = se->wbf16;
  auto W = [&](const Mat& m) { return bf ? static_cast<const float*>(m.w16) : m.w; };
  auto WT = [&](const Mat& m) { return bf ? static_cast<const float*>(m.t16) : m.t; };
  auto WH = [&](const Mat& m) { return bf ? static_cast<const float*>(m.hb16) : m.hb; };
  std::vector<Phase> ph;
  auto per = [&](int rows, int items_wanted, int multiple) {
    int p = (rows + items_wanted - 1) / items_wanted;
    p = (p + multiple - 1) / multiple * multiple;
    return std::min(p, kMaxItemOut / multiple * multiple);
  };
  auto seg = [&](const float* w, int rows, int p, float* out) {
    Segment sg{};
    sg.w = w, sg.rows = rows, sg.per_item = p, sg.items = (rows + p - 1) / p, sg.out = out;
    return sg;
  };
  auto gemv = [&](int cols, int in_mode, const float* a, const float* b, const float* cc, const float* nw, float* xout,
                  int out_mode, Segment s0) {
    Phase p{};
    p.kind = PH_GEMV;
    p.cols = cols;
    p.in_mode = in_mode, p.in_a = a, p.in_b = b, p.in_c = cc, p.norm_w = nw, p.xout = xout;
    p.out_mode = out_mode;
    p.nseg = 1;
    p.seg[0] = s0;
    p.items = s0.items;
    return p;
  };
  const int splits = std::min(kMaxSplits, std::max(1, G / H));
  // The merge in the o prologue keeps m, l of every (head, split) on chip.
  SLM_REQUIRE(2 * H * splits <= (kMaxSplits / 2) * (kDH + 2) && H <= (kMaxSplits / 2) * (kDH + 2),
              "too many attention partials for the decode kernel");
  const float scale = 1.0f / std::sqrt((float)c.dh());
  // Global layers: items are cache heads × splits (each serving heads / kv_heads queries).
  const int kh = (int)c.kv_heads;
  const int gsplits = std::min(kMaxSplits, std::max(1, G / kh));
  SLM_REQUIRE(2 * H * gsplits <= (kMaxSplits / 2) * (kDH + 2), "too many attention partials for the decode kernel");
  // Attention partials (heads × splits × (dh + 2)) and per-head arrival counters.
  if (!refresh) {
    se->attn_part = static_cast<float*>(
        alloc_zero(se, (size_t)H * std::max(splits, gsplits) * (kDH + 2) * sizeof(float)));
    se->attn_count = static_cast<unsigned*>(alloc_zero(se, (size_t)H * sizeof(unsigned)));
    using u64 = unsigned long long;
    auto tw = [&](size_t n) { return static_cast<u64*>(alloc_zero(se, n * sizeof(u64))); };
    se->tq = tw((size_t)3 * d);
    se->tpart = tw((size_t)H * std::max(splits, gsplits) * (kDH + 2));
    se->tmix = tw((size_t)4 * d);
    se->tdec = tw((size_t)H);
    se->te = tw((size_t)d);
    se->epoch = static_cast<unsigned*>(alloc_zero(se, 64 * sizeof(unsigned)));
  }
  float* attn_part = se->attn_part;
  unsigned* attn_count = se->attn_count;
  float* X0 = se->xa;
  // Fused MLP phases: one fixed-point slot each, in plan order.  fx_of(buf)
  // is the slot holding buffer buf's current value when a fused MLP wrote it
  // last (its readers take the slot; the float buffer is stale).
  const size_t nmlp = md->prelude.size() + se->loops * md->core.size() + md->coda.size();
  // S and L blocks: the mixer (attention, GLA) and o in one phase (items ≤
  // grid, so every split of a head is resident while it waits; o rows split
  // evenly over the splits).
  auto nS = [](const std::string& k) {
    return (size_t)(std::count(k.begin(), k.end(), 'S') + std::count(k.begin(), k.end(), 'L'));
  };
  const size_t nao = nS(c.prelude) + se->loops * nS(c.core) + nS(c.coda);
  const bool fuse_ao = se->fuse_mlp && se->fuse_ao && H * splits <= G && d % splits == 0 && d / splits <= kMaxItemOut &&
                       (size_t)(d / splits) * kDH * 4 <= (size_t)kStageBytes;
  const size_t slot_words = (size_t)d + 2;
  const size_t nslots = se->fuse_mlp ? nmlp + (fuse_ao ? nao : 0) : 0;
  const size_t ncnt = fuse_ao ? nao * H : 0;
  if (!refresh && se->fuse_mlp) {
    se->fx_set_words = (nslots * slot_words + ncnt + 31) / 32 * 32;
    se->fx = static_cast<unsigned long long*>(alloc_zero(se, 2 * se->fx_set_words * sizeof(unsigned long long)));
  }
  size_t next_slot = 0, next_cnt = 0;
  // Which fixed-point slot holds each buffer's current value, and how many
  // contributions make it final (every CTA for an MLP, one per head for a
  // mixer with o).
  struct FxHold {
    const float* buf;
    unsigned long long* slot;
    int cnt;
    int arrive;  // CTAs that announce their adds in the slot's word d (MLP slots)
  };
  std::vector<FxHold> fxw;
  auto fx_of = [&](const float* buf) -> const unsigned long long* {
    for (auto& e : fxw)
      if (e.buf == buf) return e.slot;
    return nullptr;
  };
  auto fx_cnt_of = [&](const float* buf) -> int {
    for (auto& e : fxw)
      if (e.buf == buf) return e.cnt;
    return 0;
  };
  auto fx_set = [&](const float* buf, unsigned long long* slot, int cnt = 0, int arrive = 0) {
    for (auto& e : fxw)
      if (e.buf == buf) {
        e.slot = slot, e.cnt = cnt, e.arrive = arrive;
        return;
      }
    fxw.push_back(FxHold{buf, slot, cnt, arrive});
  };
  // A phase reading buffer `buf` as its `a` input.
  auto read_x = [&](Phase& p, const float* buf) {
    p.fx_in = fx_of(buf);
    p.fx_cnt = fx_cnt_of(buf);
    for (auto& e : fxw)
      if (e.buf == buf) p.fx_arrive = e.arrive;
  };
  struct In {
    int mode;
    const float *a, *b, *c;
    float* xout;
  };
  auto block_mlp = [&](const Block& b, float* X) {
    const int F = (int)b.down.cols;
    if (se->fuse_mlp) {
      Phase u = gemv(d, IN_RMS, X, nullptr, nullptr, b.norm2, nullptr, OUT_MLP, seg(W(b.up), F, per(F, G, 1), nullptr));
      u.wt = WT(b.down);
      read_x(u, X);
      u.sync = u.fx_in ? 0 : 1;  // after a G block's o, x is a float buffer
      u.fx_out = se->fx + slot_words * next_slot++;
      ph.push_back(u);
      fx_set(X, u.fx_out, G, G);  // every CTA adds into every value, and announces it
      return;
    }
    ph.push_back(gemv(d, IN_RMS, X, nullptr, nullptr, b.norm2, nullptr, OUT_SILU,
                      seg(W(b.up), F, per(F, G, 1), se->mid)));
    ph.push_back(gemv(F, IN_PLAIN, se->mid, nullptr, nullptr, nullptr, nullptr, OUT_ADD,
                      seg(b.down.w, d, per(d, G, 1), X)));
    ph.back().res_smem = 1;
  };
  // The loop input's inject term, tagged by the inject phase.
  int inject_phase = -1;
  auto loop_input = [&](Phase& p, const In& in) {
    if (in.mode != IN_LOOP_RMS) return;
    p.tin_b = se->te;
    p.tag_in = inject_phase;
  };
  auto block = [&](const Block& b, LState& st, float* X, In in) {
    const float* ia = in.mode == IN_RMS ? X : in.a;
    if (b.kind == 'S') {
      Phase p = gemv(d, in.mode, ia, in.b, in.c, b.norm1, in.xout, OUT_ROPE,
                     seg(W(b.qkv), 3 * d / 2, per(3 * d / 2, G, 8), nullptr));
      p.q = se->q, p.kc = st.k, p.vc = st.v, p.cap = (long long)st.cap, p.inv_freq = md->inv_freq;
      p.tq = se->tq;
      read_x(p, ia);
      loop_input(p, in);
      const int proj = (int)ph.size();
      ph.push_back(p);
      if (in.mode == IN_LOOP_RMS || in.mode == IN_EMBED_RMS) fx_set(X, nullptr);  // that prologue wrote x to X
      Phase a{};
      a.kind = PH_ATTN;
      a.kc = st.k, a.vc = st.v, a.q = se->q, a.cap = (long long)st.cap, a.window = (long long)c.window;
      a.heads = H, a.splits = splits, a.part = attn_part, a.counters = attn_count;
      a.y = se->y, a.scale = scale, a.items = H * splits;
      a.tq = se->tq, a.tkv = se->tq + d, a.tpart = se->tpart, a.tag_in = proj;
      if (fuse_ao && b.o.hb) {
        a.wo = WH(b.o);
        a.orows = d / splits;
        a.cnt = se->fx + nslots * slot_words + H * next_cnt++;
        a.in_a = X;
        a.fx_out = se->fx + slot_words * next_slot++;
        ph.push_back(a);
        fx_set(X, a.fx_out, H);  // one part per head
        block_mlp(b, X);
        return;
      }
      ph.push_back(a);
    } else if (b.kind == 'G') {
      // q and kv from n = rms(x)·w (+ rms(e0)·w_e); n becomes the next shift
      // input; items split between the two products by rows.
      const int kd = kh * kDH;
      const int qi = std::max(1, G * d / (d + 2 * kd)), ki = std::max(1, G - qi);
      Phase p = gemv(d, IN_RMS_E, X, nullptr, b.norm_e, b.norm1, c.kshift ? st.prev : nullptr, OUT_G,
                     seg(W(b.q), d, per(d, qi, 1), se->q));
      p.nseg = 2;
      p.seg[1] = seg(W(b.kv), 2 * kd, per(2 * kd, ki, 1), nullptr);
      p.items = p.seg[0].items + p.seg[1].items;
      p.kc = st.k, p.vc = st.v, p.cap = (long long)st.cap, p.heads = kh, p.kshift = c.kshift ? 1 : 0;
      p.inv_log = c.logn ? 1.0f / std::log((float)c.logn) : 0.0f;
      p.seg[0].tout = se->tq;
      read_x(p, X);
      const int proj = (int)ph.size();
      ph.push_back(p);
      Phase a{};
      a.kind = PH_ATTN;
      a.kc = st.k, a.vc = st.v, a.q = se->q, a.cap = (long long)st.cap, a.window = 0;
      a.gap = c.far ? (long long)c.window : 0;
      a.heads = H, a.qg = H / kh, a.splits = gsplits, a.part = attn_part, a.counters = attn_count;
      a.y = se->y, a.scale = scale, a.items = kh * gsplits;
      a.tq = se->tq, a.tpart = se->tpart, a.tag_in = proj;
      a.sync = 1;  // the projection stored this position's value (and key) in the cache
      ph.push_back(a);
    } else {
      Phase p = gemv(d, in.mode, ia, in.b, in.c, b.norm1, in.xout, OUT_STORE,
                     seg(W(b.qkvg), 4 * d, per(4 * d, std::max(1, G - 1), 1), se->mix));
      p.nseg = 2;
      p.seg[1] = seg(W(b.decay), H, per(H, 1, 1), se->dec);
      p.items = p.seg[0].items + p.seg[1].items;
      p.seg[0].tout = se->tmix, p.seg[1].tout = se->tdec;
      read_x(p, ia);
      loop_input(p, in);
      const int proj = (int)ph.size();
      ph.push_back(p);
      if (in.mode == IN_LOOP_RMS || in.mode == IN_EMBED_RMS) fx_set(X, nullptr);  // that prologue wrote x to X
      Phase g{};
      g.kind = PH_GLA;
      g.state = st.s, g.mix = se->mix, g.dec = se->dec, g.bias = b.bias, g.hnw = b.head_norm, g.y = se->y;
      g.tmix = se->tmix, g.tdec = se->tdec, g.tag_in = proj;
      g.items = H;
      if (fuse_ao && b.o.hb) {  // every split of a head runs the GLA, every split its o rows
        g.items = H * splits;
        g.splits = splits;
        g.wo = WH(b.o);
        g.orows = d / splits;
        g.cnt = se->fx + nslots * slot_words + H * next_cnt++;
        g.in_a = X;
        g.fx_out = se->fx + slot_words * next_slot++;
        ph.push_back(g);
        fx_set(X, g.fx_out, H);  // one part per head
        block_mlp(b, X);
        return;
      }
      ph.push_back(g);
    }
    // The residual of o and down is the x of the phase two back, whose
    // normalising prologue left it in shared memory on every CTA.  After an
    // S mixer, o's input is merged from the attention partials.
    if (b.kind == 'S' || b.kind == 'G') {
      Phase o = gemv(d, IN_ATTN, attn_part, nullptr, nullptr, nullptr, nullptr, OUT_ADD, seg(W(b.o), d, per(d, G, 1), X));
      o.heads = H, o.splits = b.kind == 'G' ? gsplits : splits;
      o.tpart = se->tpart, o.tag_in = (int)ph.size() - 1;  // the attention phase's partials
      o.sync = 1;
      ph.push_back(o);
    } else {
      ph.push_back(gemv(d, IN_PLAIN, se->y, nullptr, nullptr, nullptr, nullptr, OUT_ADD, seg(W(b.o), d, per(d, G, 1), X)));
    }
    ph.back().res_smem = 1;
    fx_set(X, nullptr);  // o wrote the float x
    block_mlp(b, X);
  };
  for (size_t i = 0; i < md->prelude.size(); i++)
    block(md->prelude[i], se->pre[i], X0, In{i == 0 ? IN_EMBED_RMS : IN_RMS, nullptr, nullptr, nullptr, nullptr});
  float* X = X0;
  if (md->looped) {
    inject_phase = (int)ph.size();
    ph.push_back(gemv(d, IN_PLAIN, X0, nullptr, nullptr, nullptr, nullptr, OUT_STORE,
                      seg(W(md->inject), d, per(d, G, 1), se->e_proj)));
    read_x(ph.back(), X0);
    ph.back().seg[0].tout = se->te;
    ph.back().sync = ph.back().fx_in ? 0 : 1;
    const float* sbuf = X0;
    for (size_t r = 0; r < se->loops; r++) {
      float* xr = (r % 2 == 0) ? se->xb : se->xc;
      for (size_t j = 0; j < md->core.size(); j++) {
        In in = j == 0 ? In{IN_LOOP_RMS, sbuf, se->e_proj, md->loop_embed.w + r * c.d, xr}
                       : In{IN_RMS, nullptr, nullptr, nullptr, nullptr};
        const size_t first = ph.size();
        block(md->core[j], se->core[r][j], xr, in);
        for (size_t k = first; k < ph.size(); k++) ph[k].l2keep = 1;  // read again by the next loop
      }
      sbuf = xr;
    }
    X = const_cast<float*>(sbuf);
  }
  for (size_t i = 0; i < md->coda.size(); i++)
    block(md->coda[i], se->coda[i], X, In{IN_RMS, nullptr, nullptr, nullptr, nullptr});
  ph.push_back(gemv(d, IN_RMS, X, nullptr, nullptr, md->norm_f, nullptr, OUT_LOGITS,
                    seg(W(md->embed), (int)c.vocab, per((int)c.vocab, G, 1), se->logits)));
  read_x(ph.back(), X);
  ph.back().sync = ph.back().fx_in ? 0 : 1;
  SLM_REQUIRE(ph.size() < (1u << kTagPhaseBits), "too many phases for the decode kernel's tags");
  const int logit_items = ph.back().items;
  SLM_REQUIRE(next_slot <= nslots && next_cnt * H <= ncnt, "fused-phase slots out of step");

  if (refresh) {
    SLM_REQUIRE((int)ph.size() == se->plan_host.nphases, "decode plan changed shape");
    SLM_CUDA(cudaMemcpyAsync(se->phases_dev, ph.data(), ph.size() * sizeof(Phase), cudaMemcpyHostToDevice,
                             se->ctx->stream));
    se->plan_stale = false;
    return;
  }
  // Device memory of the plan: phases, arg-max partials, counters, barrier words.
  se->phases_dev = static_cast<Phase*>(alloc_zero(se, ph.size() * sizeof(Phase)));
  SLM_CUDA(cudaMemcpyAsync(se->phases_dev, ph.data(), ph.size() * sizeof(Phase), cudaMemcpyHostToDevice,
                           se->ctx->stream));
  auto* words = static_cast<unsigned*>(alloc_zero(se, 64 * sizeof(unsigned)));
  Plan& P = se->plan_host;
  P = Plan{};
  P.nphases = (int)ph.size();
  P.phases = se->phases_dev;
  P.d = d, P.heads = H, P.vocab = (int)c.vocab, P.eps = c.eps;
  P.embed = md->embed.w;
  P.inv_freq = md->inv_freq;
  P.ids = se->ids_dev;
  P.e0 = se->e0, P.x0 = X0;
  P.pos = se->pos_dev;
  P.arg_count = words;
  P.bar = words + 4;
  P.out_index = words + 8;
  se->argmax_dev = words + 12;
  P.argmax = se->argmax_dev;
  P.argmax2 = reinterpret_cast<uint32_t*>(se->ctx->err + 1);
  P.host_id = -1;
  P.global = (c.prelude + c.core + c.coda).find('G') != std::string::npos ? 1 : 0;
  P.arg_part = static_cast<unsigned long long*>(alloc_zero(se, logit_items * sizeof(unsigned long long)));
  P.fx = se->fx;
  P.fx_words = se->fuse_mlp ? (int)(nslots * slot_words + ncnt) : 0;
  P.fx_stride = (long long)se->fx_set_words;
  P.epoch = se->epoch;
  // The unfused variants pass plain buffers between phases: a barrier before each.
  P.all_sync = !se->fuse_mlp || !fuse_ao ? 1 : 0;
  P.mlp_cta = d > kMaxCols / 4 || mlp_cta_setting() ? 1 : 0;
  P.wbytes = bf ? 2 : 4;
  P.l2mode = l2mode_setting();
  {
    const char* e = std::getenv("SLM_MEGA_INFLIGHT");
    P.inflight = e && *e ? std::atoi(e) : kStages;
  }
  P.nsteps = 1;
  P.next_tagged = static_cast<unsigned long long*>(alloc_zero(se, 4 * sizeof(unsigned long long)));
  // Zero point: the first phase whose input every CTA reads from an MLP's
  // fixed-point slot (every CTA adds into it, so by then every CTA has
  // finished the previous step).  Without one, steps run one per launch.
  P.zero_phase = -1;
  for (size_t i = 0; i + 1 < ph.size(); i++) {
    const Phase& q = ph[i];
    const bool everyone = q.kind == PH_GEMV && q.in_mode != IN_PLAIN && q.in_mode != IN_ATTN;
    if (everyone && q.fx_in && q.fx_cnt == G) {
      P.zero_phase = (int)i;
      break;
    }
  }
  P.next_id = se->ids_dev;
  P.err = se->ctx->err;
}

// Points the plan's greedy outputs at `out` (nullptr: logits only).
void plan_outputs(slm_session* se, bool greedy, uint32_t* out, uint32_t* hist, unsigned long long hist_base) {
  mega::Plan& P = se->plan_host;
  P.greedy = greedy ? 1 : 0;
  P.out_ids = out;
  P.hist = hist;
  P.hist_base = hist_base;  // the plan travels by value with each launch
  SLM_CUDA(cudaMemsetAsync(P.out_index, 0, sizeof(unsigned), se->ctx->stream));
}

// With kshift the persistent step expects the key of its own position in
// every global cache already (W_k · prev, stored by the step or chunk before).
// After the state was written from the host, compute those keys from prev.
void refresh_next_keys(slm_session* se) {
  slm_model* md = se->model;
  const Config& c = md->cfg;
  se->keys_stale = false;
  if (!c.kshift) return;
  g_ctx_for_linear = se->ctx;
  g_capturing = false;
  cudaStream_t s = se->ctx->stream;
  const size_t kh = c.kv_heads, dh = c.dh(), kd = kh * dh;
  auto one = [&](const Block& b, LState& st) {
    if (b.kind != 'G') return;
    run_linear(s, b.kv, st.prev, (int)c.d, 1, se->kvs, (int)kd, EPI_STORE, nullptr, 0, kd);  // key rows only
    ew_store_next(st.k, se->kvs, se->pos_dev, 0, kh, dh, st.cap, s);
  };
  for (size_t i = 0; i < md->prelude.size(); i++) one(md->prelude[i], se->pre[i]);
  for (size_t r = 0; r < se->loops; r++)
    for (size_t j = 0; j < md->core.size(); j++) one(md->core[j], se->core[r][j]);
  for (size_t i = 0; i < md->coda.size(); i++) one(md->coda[i], se->coda[i]);
}

// host_id ≥ 0: the step's token, passed in the launch parameters (no copy);
// else the kernel reads ids_dev[0].
void mega_step(slm_session* se, long long host_id = -1) {
  if (se->plan_stale) build_plan(se, true);
  if (se->keys_stale) refresh_next_keys(se);
  if (host_id >= 0) {
    mega::Plan p = se->plan_host;
    p.host_id = host_id;
    p.host_mbox = se->ctx->mbox_dev;
    p.host_seq = ++se->ctx->mbox_seq;
    se->mbox_want = p.host_seq;
    mega::launch(p, se->grid, se->ctx->stream);
  } else {
    mega::launch(se->plan_host, se->grid, se->ctx->stream);
  }
  se->pos += 1;
  se->argmax_valid = true;
  se->ctx->argmax_owner = se;
}

// Arming: in a greedy step/sample loop, slm_step queues the next persistent
// step right behind the one it issues, waiting (bounded) on the context's gate
// word; the next slm_step only writes its token there.  The launch and the
// kernel's start then overlap the running step and the host's turn-around
// instead of following them.  SLM_MEGA_ARM=0 disables it.
// It is off where launches are serialised (CUDA_LAUNCH_BLOCKING=1, or a
// profiler that waits for each kernel): there an armed step runs while the
// host is still inside the launch call, so it can only run out of time.  arm()
// notices that (the stream is already idle when the launch returns) and turns
// arming off for the rest of the process.
std::atomic<bool> g_arm_serialised{false};
bool arm_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SLM_MEGA_ARM");
    if (e && *e == '0') return false;
    const char* b = std::getenv("CUDA_LAUNCH_BLOCKING");
    return !(b && *b == '1');
  }();
  return on && !g_arm_serialised.load(std::memory_order_relaxed);
}

void arm(slm_session* se) {
  slm_ctx* c = se->ctx;
  ensure_caps(se, 1);
  if (se->plan_stale) build_plan(se, true);
  if (se->keys_stale) refresh_next_keys(se);
  mega::Plan p = se->plan_host;
  p.host_gate = c->mbox_dev + 8;
  p.gate_seq = ++c->mbox_seq;
  p.host_mbox = c->mbox_dev;
  p.host_seq = p.gate_seq;
  mega::launch(p, se->grid, c->stream);
  c->armed = true;
  c->armed_seq = p.gate_seq;
  c->armed_owner = se;
  // The armed kernel waits for a token no one has written yet: an idle stream
  // here means the launch returned only after the kernel had given up.
  const cudaError_t q = cudaStreamQuery(c->stream);
  if (q == cudaErrorNotReady) {
    if (cudaPeekAtLastError() == cudaErrorNotReady) (void)cudaGetLastError();  // the query's answer, not an error
  } else if (q == cudaSuccess) {
    g_arm_serialised.store(true, std::memory_order_relaxed);
    c->armed = false;
    c->armed_owner = nullptr;
  }
}

// n greedy persistent steps for the id in ids_dev[0], as few launches as the
// plan allows: one launch runs the steps back to back (each step's arg-max is
// the next one's token), so later steps pay neither a launch nor a cold
// start.  Global caches grow first to hold all n positions.
// SLM_MEGA_STEPS=1 runs one step per launch (for comparison).
size_t mega_steps_per_launch() {
  const char* e = std::getenv("SLM_MEGA_STEPS");
  const long v = e && *e ? std::atol(e) : 4096;
  return v < 1 ? 1 : (size_t)v;
}

void mega_steps(slm_session* se, size_t n) {
  const size_t most = mega_steps_per_launch();
  while (n > 0) {
    const size_t m = se->plan_host.zero_phase >= 0 ? std::min(n, most) : 1;
    ensure_caps(se, m);
    if (se->plan_stale) build_plan(se, true);
    if (se->keys_stale) refresh_next_keys(se);
    mega::Plan p = se->plan_host;
    p.nsteps = (int)m;
    mega::launch(p, se->grid, se->ctx->stream);
    se->pos += m;
    n -= m;
  }
  se->argmax_valid = true;
  se->ctx->argmax_owner = se;
}

// One decode step for the id already in ids_dev[0]: graph replay when enabled.
void step_device(slm_session* se) {
  ensure_caps(se, 1);
  cudaStream_t s = se->ctx->stream;
  if (se->use_mega) {
    mega_step(se);
    return;
  }
  se->argmax_valid = false;  // graph replays do not write the arg-max word
  if (!se->use_graph) {
    advance(se, 1, true);
    return;
  }
  if (!se->graph) {
    cudaGraph_t g = nullptr;
    SLM_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    se->capturing = true;
    size_t pos0 = se->pos;
    try {
      advance(se, 1, true);
    } catch (...) {
      se->capturing = false;
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      se->pos = pos0;
      throw;
    }
    se->capturing = false;
    se->pos = pos0;  // the capture enqueued nothing
    SLM_CUDA(cudaStreamEndCapture(s, &g));
    size_t count = 0;
    cudaGraphGetNodes(g, nullptr, &count);
    std::vector<cudaGraphNode_t> nodes(count);
    if (count) cudaGraphGetNodes(g, nodes.data(), &count);
    int64_t kernels = 0;
    for (auto nd : nodes) {
      cudaGraphNodeType t;
      if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
    }
    se->step_kernels = kernels;
    se->graphs++;
    cudaError_t e = cudaGraphInstantiate(&se->graph, g, 0);
    cudaGraphDestroy(g);
    SLM_CUDA(e);
  }
  SLM_CUDA(cudaGraphLaunch(se->graph, s));
  se->pos += 1;
}

void check_device_error(slm_ctx* c, slm_session* se = nullptr) {
  SLM_CUDA(cudaMemcpyAsync(c->err_host, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  SLM_CUDA(cudaStreamSynchronize(c->stream));
  const int h = *c->err_host;
  if (h) {
    SLM_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
    if ((h & (8 | 16)) && se && se->mega_ok) {
      // A step that gave up left its barrier and arrival counters and its
      // fixed-point sums mid-way, and did not advance the step counter: reset
      // them, and advance the counter so no tag of that step is taken for a
      // later one.
      SLM_CUDA(cudaMemsetAsync(se->plan_host.arg_count, 0, 16 * sizeof(unsigned), c->stream));
      SLM_CUDA(cudaMemsetAsync(se->attn_count, 0, se->model->cfg.heads * sizeof(unsigned), c->stream));
      if (se->fx)
        SLM_CUDA(cudaMemsetAsync(se->fx, 0, 2 * se->fx_set_words * sizeof(unsigned long long), c->stream));
      unsigned e = 0;
      SLM_CUDA(cudaMemcpyAsync(&e, se->epoch, sizeof(e), cudaMemcpyDeviceToHost, c->stream));
      SLM_CUDA(cudaStreamSynchronize(c->stream));
      e += 1;
      SLM_CUDA(cudaMemcpyAsync(se->epoch, &e, sizeof(e), cudaMemcpyHostToDevice, c->stream));
      SLM_CUDA(cudaStreamSynchronize(c->stream));
    }
    std::string why;
    if (h & 1) why += " token id out of range;";
    if (h & 8) why += " a bounded wait in the decode kernel expired (state of this step is undefined);";
    if (h & 32) why += " a bounded wait in the tensor-core attention pass expired (its output is undefined);";
    if (h & 16)
      why += " a residual value in the decode kernel was non-finite or beyond 2^22 in magnitude (state of this step "
             "is undefined);";
    fail(SLM_ERR_DEVICE, "device reported:" + why);
  }
}

// ---------------------------------------------------------------------------
// Batched decode: n sessions, one token each per step.  No counterpart in the
// reference (its server runs one request at a time, src/serve.rs:1-3); the
// arithmetic of each row is Model::block / Model::advance (src/model.rs:
// 400-640) for m = 1, on that session's state.
// ---------------------------------------------------------------------------

void* balloc(slm_batch* bt, size_t bytes) {
  void* p = dev_alloc(bytes);
  bt->owned.push_back(p);
  SLM_CUDA(cudaMemsetAsync(p, 0, bytes, bt->ctx->stream));
  return p;
}

// The sessions' per-layer pointers and capacities, in step order (prelude,
// each loop's core, coda), copied into the batch's device tables (whose
// addresses the captured step holds).
void batch_tables(slm_batch* bt) {
  slm_model* md = bt->model;
  const size_t n = bt->n;
  std::vector<const LState*> inst;  // [instance][session], flattened
  for (size_t i = 0; i < n; i++) {
    slm_session* se = bt->ses[i];
    size_t at = 0;
    auto put = [&](const LState& st) {
      if (inst.size() < (at + 1) * n) inst.resize((at + 1) * n);
      inst[at * n + i] = &st;
      at++;
    };
    for (auto& st : se->pre) put(st);
    for (auto& l : se->core)
      for (auto& st : l) put(st);
    for (auto& st : se->coda) put(st);
  }
  cudaStream_t s = bt->ctx->stream;
  std::vector<float*> host(4 * n);
  std::vector<long long> caps(n);
  for (size_t k = 0; k < bt->tab.size(); k++) {
    for (size_t i = 0; i < n; i++) {
      const LState* st = inst[k * n + i];
      host[i] = st->k, host[n + i] = st->v, host[2 * n + i] = st->s, host[3 * n + i] = st->prev;
      caps[i] = (long long)st->cap;
    }
    SLM_CUDA(cudaMemcpyAsync(bt->tab[k], host.data(), 4 * n * sizeof(float*), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemcpyAsync(bt->caps[k], caps.data(), n * sizeof(long long), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaStreamSynchronize(s));  // host arrays are reused for the next instance
  }
  (void)md;
}

// Global caches of every session hold the next step (grown on the device if
// not); the batch's tables follow them.
void batch_caps(slm_batch* bt) {
  const Config& c = bt->model->cfg;
  if ((c.prelude + c.core + c.coda).find('G') == std::string::npos) return;
  bool grew = false;
  for (auto* se : bt->ses) {
    std::vector<size_t> before;
    auto note = [&](std::vector<LState>& v) {
      for (auto& st : v) before.push_back(st.cap);
    };
    note(se->pre);
    for (auto& l : se->core) note(l);
    note(se->coda);
    ensure_caps(se, 1);
    size_t at = 0;
    auto cmp = [&](std::vector<LState>& v) {
      for (auto& st : v) grew |= st.cap != before[at++];
    };
    cmp(se->pre);
    for (auto& l : se->core) cmp(l);
    cmp(se->coda);
  }
  if (grew) batch_tables(bt);
}

void batch_block(slm_batch* bt, const Block& b, size_t li, float* x) {
  slm_model* md = bt->model;
  const Config& c = md->cfg;
  cudaStream_t s = bt->ctx->stream;
  const size_t d = c.d, heads = c.heads, dh = c.dh(), m = bt->n;
  const float scale = 1.0f / std::sqrt((float)dh);
  const int im = (int)m, id = (int)d;
  float* const* K = bt->tab[li];
  float* const* V = bt->tab[li] + m;
  float* const* S = bt->tab[li] + 2 * m;
  float* const* PV = bt->tab[li] + 3 * m;
  const long long* CAP = bt->caps[li];
  ew_rms(bt->nb, x, b.norm1, m, d, c.eps, nullptr, s);
  if (b.kind == 'S') {
    run_linear(s, b.qkv, bt->nb, id, im, bt->mix, (int)(3 * d), EPI_STORE);
    const size_t cap = c.window + CHUNK;
    ew_rope_store_rows(bt->mix, 3 * d, md->inv_freq, bt->posr, m, heads, dh, cap, bt->q, K, V, s);
    AttnGeom g{im, (long long)c.window, 0, (long long)cap, (int)heads, (int)heads, (int)dh, scale};
    AttnRows rows;
    rows.k = K, rows.v = V, rows.pos = bt->posr;
    attention_rows(bt->q, id, rows, g, bt->nsplit, bt->part, bt->y, id, s, bt->merge_cnt);
  } else if (b.kind == 'G') {
    // Model::block's global mixer (src/model.rs:487-543) per row, on the
    // row's own cache, position and previous input.
    if (b.norm_e) ew_rms(bt->nb, bt->e0, b.norm_e, m, d, c.eps, bt->nb, s);  // n += rms(e0)·w_e
    const size_t kh = c.kv_heads, kd = kh * dh;
    run_linear(s, b.q, bt->nb, id, im, bt->q, id, EPI_STORE);
    run_linear(s, b.kv, bt->nb, id, im, bt->mix, (int)(2 * kd), EPI_STORE);
    const float* keys = bt->mix;
    size_t ldk = 2 * kd;
    if (c.kshift) {  // this position's key from the row's previous input, which becomes this n
      ew_gather_rows(bt->kb, PV, m, d, s);
      run_linear(s, b.kv, bt->kb, id, im, bt->kvs, (int)kd, EPI_STORE, nullptr, 0, kd);  // key rows only
      ew_scatter_rows(PV, bt->nb, m, d, s);
      keys = bt->kvs;
      ldk = kd;
    }
    const float inv_log = c.logn ? 1.0f / std::log((float)c.logn) : 0.0f;
    ew_g_post_rows(bt->q, d, m, bt->posr, inv_log, c.logn ? 1 : 0, keys, ldk, bt->mix + kd, 2 * kd, kd, dh, K, V,
                   CAP, s);
    if (c.kshift) {  // the next position's key (the persistent step relies on it)
      run_linear(s, b.kv, bt->nb, id, im, bt->kvs, (int)kd, EPI_STORE, nullptr, 0, kd);
      ew_store_next_rows(K, bt->kvs, bt->posr, 1, m, kh, dh, CAP, s);
    }
    // A row that sees nothing yet (position within the far gap) gets y = 0,
    // so o adds exactly 0 — what the reference's skipped o gives.
    const long long far = c.far ? (long long)c.window : 0;
    AttnGeom g{im, 0, far, 1ll << 40, (int)heads, (int)kh, (int)dh, scale};
    AttnRows rows;
    rows.k = K, rows.v = V, rows.pos = bt->posr, rows.cap = CAP;
    attention_rows(bt->q, id, rows, g, bt->gsplit, bt->part, bt->y, id, s, bt->merge_cnt);
  } else {  // 'L'
    run_linear(s, b.qkvg, bt->nb, id, im, bt->mix, (int)(4 * d), EPI_STORE);
    run_linear(s, b.decay, bt->nb, id, im, bt->dec, (int)heads, EPI_STORE);
    ew_l2norm(bt->q, d, bt->mix, 4 * d, m, heads, dh, s);
    ew_l2norm(bt->kb, d, bt->mix + d, 4 * d, m, heads, dh, s);
    GlaArgs a{};
    a.q = bt->q, a.ldq = id;
    a.k = bt->kb, a.ldk = id;
    a.v = bt->mix + 2 * d, a.ldv = (int)(4 * d);
    a.g = bt->mix + 3 * d, a.ldg = (int)(4 * d);
    a.dec = bt->dec, a.lddec = (int)heads;
    a.bias = b.bias, a.hnw = b.head_norm, a.eps = c.eps;
    a.m = im, a.heads = (int)heads, a.dh = (int)dh;
    a.out = bt->y, a.ldo = id, a.fuse = 1;
    gla_rows(a, S, s);
  }
  run_linear(s, b.o, bt->y, id, im, x, id, EPI_ADD, x, id);  // x += o·y
  ew_rms(bt->nb, x, b.norm2, m, d, c.eps, nullptr, s);
  const size_t hidden = b.down.cols;
  if (m > 8 && hidden % 4 == 0) {
    run_linear(s, b.up, bt->nb, id, im, bt->upbuf, (int)(2 * hidden), EPI_STORE);
    ew_silu_pair(bt->mid, bt->upbuf, m, hidden, s);
  } else {
    run_linear(s, b.up, bt->nb, id, im, bt->mid, (int)hidden, EPI_SILU);
  }
  run_linear(s, b.down, bt->mid, (int)hidden, im, x, id, EPI_ADD, x, id);
}

// One step of every session: tokens in bt->ids; the greedy ids of the next
// step go back to bt->ids and to outs[*out_index]; positions advance.
void batch_advance(slm_batch* bt, bool sampled) {
  g_ctx_for_linear = bt->ctx;
  g_capturing = bt->capturing;
  slm_model* md = bt->model;
  const Config& c = md->cfg;
  cudaStream_t s = bt->ctx->stream;
  const size_t d = c.d, m = bt->n;
  const size_t loops = bt->ses[0]->loops;
  float* x = bt->xa;
  ew_embed(bt->e0, x, md->embed.w, bt->ids, m, d, c.vocab, bt->ctx->err, s);
  size_t li = 0;
  for (size_t i = 0; i < md->prelude.size(); i++) batch_block(bt, md->prelude[i], li++, x);
  if (md->looped) {
    run_linear(s, md->inject, x, (int)d, (int)m, bt->e_proj, (int)d, EPI_STORE);
    float* sbuf = x;
    for (size_t r = 0; r < loops; r++) {
      float* xr = (sbuf == bt->xa) ? bt->xb : bt->xa;
      ew_loop_in(xr, sbuf, bt->e_proj, md->loop_embed.w + r * d, m, d, s);
      for (size_t j = 0; j < md->core.size(); j++) batch_block(bt, md->core[j], li++, xr);
      if (c.damp == 1.0f)
        sbuf = xr;
      else
        ew_mix(sbuf, sbuf, xr, m * d, c.damp, s);
    }
    x = sbuf;
  }
  for (size_t i = 0; i < md->coda.size(); i++) batch_block(bt, md->coda[i], li++, x);
  ew_rms(bt->nb, x, md->norm_f, m, d, c.eps, nullptr, s);
  run_linear(s, md->embed, bt->nb, (int)d, (int)m, bt->logits, (int)c.vocab, EPI_STORE);  // tied head, every row
  if (sampled)
    sample_rows(bt->srows, m, bt->out_index, bt->outs, s);  // next ids into bt->ids, histories extended
  else
    argmax_rows(bt->logits, c.vocab, m, bt->ids, bt->outs, bt->out_index, s);
  ew_advance_rows(bt->posr, m, bt->out_index, s);
}

void batch_drop_graph(slm_batch* bt) {
  for (cudaGraphExec_t* g : {&bt->graph, &bt->graph_s})
    if (*g) {
      cudaGraphExecDestroy(*g);
      *g = nullptr;
    }
}

// Grows the context's GEMM workspace for every linear of a batch step, so
// the capture (which cannot allocate) gets the tensor-core path.
void batch_workspace(slm_batch* bt) {
  slm_model* md = bt->model;
  const Config& c = md->cfg;
  const int m = (int)bt->n, d = (int)c.d;
  auto one = [&](const Mat& w, int ldx, int ldy, int epi, size_t rows = 0) {
    LinearArgs a;
    a.w = w.w, a.rows = (int)(rows ? rows : w.rows), a.cols = (int)w.cols, a.m = m, a.wplanes = w.planes;
    a.x = bt->nb, a.ldx = ldx, a.y = bt->upbuf, a.ldy = ldy, a.epi = epi;
    a.res = epi == EPI_ADD ? bt->upbuf : nullptr, a.ldres = epi == EPI_ADD ? ldy : 0;
    gemm_workspace(bt->ctx, a, false);
  };
  auto block = [&](const Block& b) {
    if (b.kind == 'S') one(b.qkv, d, 3 * d, EPI_STORE);
    if (b.kind == 'L') one(b.qkvg, d, 4 * d, EPI_STORE), one(b.decay, d, (int)c.heads, EPI_STORE);
    if (b.kind == 'G') {
      const int kd = (int)(c.kv_heads * c.dh());
      one(b.q, d, d, EPI_STORE), one(b.kv, d, 2 * kd, EPI_STORE), one(b.kv, d, kd, EPI_STORE, (size_t)kd);
    }
    one(b.o, d, d, EPI_ADD);
    one(b.up, d, (int)(2 * b.down.cols), EPI_STORE);
    one(b.down, (int)b.down.cols, d, EPI_ADD);
  };
  for (auto& b : md->prelude) block(b);
  for (auto& b : md->core) block(b);
  for (auto& b : md->coda) block(b);
  if (md->looped) one(md->inject, d, d, EPI_STORE);
  one(md->embed, d, (int)c.vocab, EPI_STORE);
}

// One step, replayed from a CUDA graph captured on first use (and again
// after the context's GEMM workspace has moved).
void batch_step_device(slm_batch* bt, bool sampled = false) {
  cudaStream_t s = bt->ctx->stream;
  batch_caps(bt);  // global caches hold this step (their tables are updated in place)
  cudaGraphExec_t& graph = sampled ? bt->graph_s : bt->graph;
  unsigned long long& gen = sampled ? bt->graph_s_ws_gen : bt->graph_ws_gen;
  if (graph && gen != bt->ctx->gemm_ws_gen) batch_drop_graph(bt);
  if (!graph) {
    batch_workspace(bt);
    gen = bt->ctx->gemm_ws_gen;
    cudaGraph_t g = nullptr;
    SLM_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    bt->capturing = true;
    try {
      batch_advance(bt, sampled);
    } catch (...) {
      bt->capturing = false;
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    bt->capturing = false;
    SLM_CUDA(cudaStreamEndCapture(s, &g));
    cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
    cudaGraphDestroy(g);
    SLM_CUDA(e);
  }
  SLM_CUDA(cudaGraphLaunch(graph, s));
  for (auto* se : bt->ses) se->pos += 1;
}

void batch_outs(slm_batch* bt, size_t steps) {
  if (steps <= bt->outs_cap) return;
  size_t cap = std::max<size_t>(steps, 2 * bt->outs_cap);
  SLM_CUDA(cudaStreamSynchronize(bt->ctx->stream));
  auto* p = static_cast<uint32_t*>(dev_alloc(cap * bt->n * sizeof(uint32_t)));
  for (auto& o : bt->owned)
    if (o == bt->outs) {
      dev_free(o);
      o = p;
    }
  bt->outs = p;
  bt->outs_cap = cap;
  batch_drop_graph(bt);  // the graph holds the old pointer
}

void ensure_u32(slm_session* se, uint32_t** p, size_t* cap, size_t n) {
  if (*cap >= n) return;
  SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
  dev_free(*p);
  size_t c = n < 1024 ? 1024 : n;
  *p = static_cast<uint32_t*>(dev_alloc(c * sizeof(uint32_t)));
  *cap = c;
}

void check_sampling(const slm_sampling* sp) {
  SLM_REQUIRE(sp, "sampling is null");
  SLM_REQUIRE(!(sp->top_p != sp->top_p) && !(sp->temperature != sp->temperature), "NaN sampling parameter");
}

SampleArgs sample_args(slm_session* se, const slm_sampling* sp) {
  SampleArgs a{};
  a.logits = se->logits;
  a.work = se->work;
  a.vocab = (int)se->model->cfg.vocab;
  a.temperature = sp->temperature;
  a.top_p = sp->top_p;
  a.penalty = sp->repeat_penalty;
  a.top_k = sp->top_k;
  a.window = sp->repeat_window;
  a.rng = se->rng_dev;
  a.err = se->ctx->err;
  return a;
}

// The session's state arrays in step order (prelude, core per loop, coda);
// per layer: S k, v; L s; G k, v, prev.
struct StateRef {
  LState* st;
  char part;
};
std::vector<StateRef> state_list(slm_session* se) {
  std::vector<StateRef> out;
  auto one = [&](LState& st) {
    if (st.kind == 'S') out.push_back({&st, 'k'}), out.push_back({&st, 'v'});
    else if (st.kind == 'L') out.push_back({&st, 's'});
    else out.push_back({&st, 'k'}), out.push_back({&st, 'v'}), out.push_back({&st, 'p'});
  };
  for (auto& st : se->pre) one(st);
  for (auto& l : se->core)
    for (auto& st : l) one(st);
  for (auto& st : se->coda) one(st);
  return out;
}

slm_state_array state_desc(const slm_session* se, const StateRef& r) {
  const Config& c = se->model->cfg;
  slm_state_array a{};
  a.kind = r.st->kind;
  a.part = r.part;
  a.dh = c.dh();
  if (r.part == 's') {
    a.heads = c.heads, a.cap = 0, a.floats = c.heads * c.dh() * c.dh();
  } else if (r.part == 'p') {
    a.heads = 1, a.cap = 0, a.dh = c.d, a.floats = c.d;
  } else {
    a.heads = r.st->kind == 'G' ? c.kv_heads : c.heads;
    a.cap = r.st->cap;
    a.floats = a.heads * a.cap * a.dh;
  }
  return a;
}

float* state_ptr(const StateRef& r) {
  return r.part == 'k' ? r.st->k : r.part == 'v' ? r.st->v : r.part == 's' ? r.st->s : r.st->prev;
}

}  // namespace
}  // namespace slm

extern "C" {

int slm_model_load(slm_ctx* ctx, const char* dir, slm_model** out) {
  return guard([&] {
    SLM_REQUIRE(ctx && dir && out, "bad arguments");
    Device dev(ctx);
    auto md = std::make_unique<slm_model>();
    md->ctx = ctx;
    md->cfg = load_config(dir);
    const Config& c = md->cfg;
    Loading L;
    L.t = load_safetensors(dir);
    auto blocks = [&](std::vector<Block>& out_b, const char* name, const std::string& kinds) {
      out_b.resize(kinds.size());
      for (size_t i = 0; i < kinds.size(); i++)
        load_block(L, c, &out_b[i], std::string(name) + "." + std::to_string(i), kinds[i]);
    };
    blocks(md->prelude, "prelude", c.prelude);
    blocks(md->core, "core", c.core);
    blocks(md->coda, "coda", c.coda);
    md->looped = !c.core.empty();
    if (md->looped) {
      mat(L, "inject_e.weight", &md->inject);
      mat(L, "loop_embed.weight", &md->loop_embed);
      SLM_REQUIRE(md->loop_embed.rows >= c.max_loops && md->loop_embed.cols == c.d, "loop_embed has the wrong shape");
    }
    mat(L, "embed.weight", &md->embed);
    vec(L, "norm_f.weight", &md->norm_f, c.d);
    SLM_REQUIRE(md->embed.rows == c.vocab && md->embed.cols == c.d, "embed must be vocab × d");
    const size_t dh = c.dh();
    SLM_REQUIRE(dh % 2 == 0 && c.d % 4 == 0, "head size must be even and d_model a multiple of 4");
    std::vector<float> inv(dh / 2);
    for (size_t i = 0; i < dh / 2; i++) inv[i] = 1.0f / std::pow(c.rope_base, (float)(2 * i) / (float)dh);
    L.t.map["__inv_freq"] = TensorView{{dh / 2}, inv.data(), dh / 2};
    vec(L, "__inv_freq", &md->inv_freq, dh / 2);
    md->arena = static_cast<float*>(dev_alloc(L.up.total * sizeof(float)));
    upload_pinned(ctx, md->arena, L.up);
    for (auto& f : L.fix) *f.first = md->arena + f.second;
    // Model::params (src/model.rs:275-302).
    size_t p = 0;
    for (auto* bs : {&md->prelude, &md->core, &md->coda})
      for (auto& b : *bs) {
        size_t mixer = 0;
        if (b.kind == 'S') mixer = mat_params(b.qkv) + mat_params(b.o);
        if (b.kind == 'L') mixer = mat_params(b.qkvg) + mat_params(b.decay) + mat_params(b.o) + c.heads + dh;
        if (b.kind == 'G') mixer = mat_params(b.q) + mat_params(b.kv) + mat_params(b.o) + (b.norm_e ? c.d : 0);
        p += mixer + 2 * c.d + mat_params(b.up) + mat_params(b.down);
        md->hidden = std::max(md->hidden, b.down.cols);
      }
    p += mat_params(md->embed) + c.d + mat_params(md->inject) + mat_params(md->loop_embed);
    md->params = p;
    md->mix_cols = std::max({3 * c.d, 4 * c.d, 2 * c.kv_heads * dh});
    // bf16x3 parts of every matrix a prefill chunk multiplies (all but the
    // tied head, which only ever sees the last token).
    std::vector<Mat*> mats;
    for (auto* bs : {&md->prelude, &md->core, &md->coda})
      for (auto& b : *bs)
        for (Mat* m : {&b.qkv, &b.o, &b.up, &b.down, &b.qkvg, &b.decay, &b.q, &b.kv})
          if (m->w) mats.push_back(m);
    if (md->inject.w) mats.push_back(&md->inject);
    size_t total = 0;
    for (Mat* m : mats) total += (b3_planes_bytes(m->rows, m->cols) + 255) / 256 * 256;
    if (total) {
      md->planes = dev_alloc(total);
      char* at = static_cast<char*>(md->planes);
      for (Mat* m : mats) {
        b3_split_weights(m->w, m->rows, m->cols, at, ctx->stream);
        m->planes = at;
        at += (b3_planes_bytes(m->rows, m->cols) + 255) / 256 * 256;
      }
      SLM_CUDA(cudaStreamSynchronize(ctx->stream));
    }
    // The fused phases of the persistent step read down by columns and the
    // o of S blocks by head: keep those layouts beside the originals when that
    // kernel can run.
    if (mega_unsupported(md.get()).empty() && fuse_mlp_enabled()) {
      std::vector<Mat*> downs, os;
      for (auto* bs : {&md->prelude, &md->core, &md->coda})
        for (auto& b : *bs) {
          downs.push_back(&b.down);
          if (b.kind == 'S' || b.kind == 'L') os.push_back(&b.o);
        }
      size_t tot = 0;
      for (Mat* m : downs) tot += (m->rows * m->cols + 63) / 64 * 64;
      for (Mat* m : os) tot += (m->rows * m->cols + 63) / 64 * 64;
      md->tarena = static_cast<float*>(dev_alloc(tot * sizeof(float)));
      float* at = md->tarena;
      for (Mat* m : downs) {
        ew_transpose(at, m->w, m->rows, m->cols, ctx->stream);
        m->t = at;
        at += (m->rows * m->cols + 63) / 64 * 64;
      }
      for (Mat* m : os) {
        ew_head_blocks(at, m->w, m->rows, c.heads, c.dh(), ctx->stream);
        m->hb = at;
        at += (m->rows * m->cols + 63) / 64 * 64;
      }
      SLM_CUDA(cudaStreamSynchronize(ctx->stream));
    }
    ctx_retain(ctx);
    *out = md.release();
  });
}

namespace {
void destroy_model(slm_model* md) {
  slm_ctx* c = md->ctx;
  {
    Device dev(c);
    cudaStreamSynchronize(c->stream);
    dev_free(md->arena);
    dev_free(md->planes);
    dev_free(md->tarena);
    dev_free(md->arena16);
  }
  delete md;
  ctx_release(c);
}
void model_release(slm_model* md) {
  if (--md->refs == 0 && md->closing) destroy_model(md);
}
}  // namespace

int slm_model_free(slm_model* md) {
  return guard([&] {
    if (!md || md->closing) return;
    if (md->refs > 0) {  // sessions still live: the last of them frees the model
      md->closing = true;
      return;
    }
    destroy_model(md);
  });
}

int slm_model_info_get(const slm_model* md, slm_model_info* out) {
  return guard([&] {
    SLM_REQUIRE(md && out, "bad arguments");
    const Config& c = md->cfg;
    std::memset(out, 0, sizeof(*out));
    out->vocab = c.vocab, out->d_model = c.d, out->heads = c.heads, out->head_dim = c.dh();
    out->kv_heads = c.kv_heads, out->hidden = md->hidden, out->window = c.window;
    out->max_loops = c.max_loops, out->default_loops = c.default_loops, out->params = md->params;
    std::strncpy(out->prelude, c.prelude.c_str(), sizeof(out->prelude) - 1);
    std::strncpy(out->core, c.core.c_str(), sizeof(out->core) - 1);
    std::strncpy(out->coda, c.coda.c_str(), sizeof(out->coda) - 1);
  });
}

int slm_session_new(slm_model* md, size_t loops, slm_session** out) {
  return guard([&] {
    SLM_REQUIRE(md && out, "bad arguments");
    const Config& c = md->cfg;
    // Config::loops (src/config.rs:96-105).
    if (c.core.empty()) {
      loops = 0;
    } else {
      if (loops == 0) loops = c.default_loops;
      SLM_REQUIRE(loops >= 1 && loops <= c.max_loops, "loops must be between 1 and " + std::to_string(c.max_loops));
    }
    Device dev(md->ctx);
    auto se = std::make_unique<slm_session>();
    se->model = md;
    se->ctx = md->ctx;
    se->loops = loops;
    try {
      for (auto& b : md->prelude) se->pre.push_back(new_state(se.get(), b));
      se->core.resize(loops);
      for (size_t r = 0; r < loops; r++)
        for (auto& b : md->core) se->core[r].push_back(new_state(se.get(), b));
      for (auto& b : md->coda) se->coda.push_back(new_state(se.get(), b));
      const size_t d = c.d, dh = c.dh(), kd = c.kv_heads * dh;
      auto f = [&](size_t n) { return static_cast<float*>(alloc_zero(se.get(), n * sizeof(float))); };
      se->xa = f(CHUNK * d);
      se->xb = f(CHUNK * d);
      se->e0 = f(CHUNK * d);
      se->e_proj = f(CHUNK * d);
      se->n = f(CHUNK * d);
      se->mix = f(CHUNK * md->mix_cols);
      se->q = f(CHUNK * d);
      se->kb = f(CHUNK * d);
      se->kin = f(CHUNK * d);
      se->kvs = f(CHUNK * kd);
      se->y = f(CHUNK * d);
      se->mid = f(CHUNK * std::max<size_t>(md->hidden, 1));
      se->upbuf = f(CHUNK * 2 * std::max<size_t>(md->hidden, 1));
      if (md->planes) se->nplanes = alloc_zero(se.get(), CHUNK * 6 * c.d * 2);
      se->dec = f(CHUNK * c.heads);
      se->nlast = f(d);
      se->logits = f(c.vocab);
      se->work = f(3 * c.vocab);  // sampler: logits, sorted weights, sorted ids
      size_t part = 0;
      for (size_t m = 1; m <= CHUNK; m++) {
        AttnGeom g{(int)m, 0, 0, 1, (int)c.heads, 1, (int)dh, 1.0f};
        part = std::max(part, attn_part_floats(g, attn_splits(g, 1ll << 40)));
      }
      se->part = f(part);
      se->merge_cnt = static_cast<unsigned*>(alloc_zero(se.get(), c.heads * CHUNK * sizeof(unsigned)));
      se->xc = f(CHUNK * d);
      se->pos_dev = reinterpret_cast<long long*>(alloc_zero(se.get(), sizeof(long long)));
      se->ids_dev = reinterpret_cast<uint32_t*>(alloc_zero(se.get(), CHUNK * sizeof(uint32_t)));
      se->rng_dev = reinterpret_cast<unsigned long long*>(alloc_zero(se.get(), sizeof(unsigned long long)));
      se->out_dev = reinterpret_cast<uint32_t*>(alloc_zero(se.get(), sizeof(uint32_t) * 4));
      SLM_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&se->io), sizeof(slm_session::HostIO), cudaHostAllocDefault));
      SLM_CUDA(cudaEventCreateWithFlags(&se->io_event, cudaEventDisableTiming));
      se->mega_why = mega_unsupported(md);
      if (se->mega_why.empty()) {
        int coop = 0;
        SLM_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, se->ctx->device));
        if (coop) {
          mega::prepare();
          if (mega::blocks_per_sm() >= 1) {
            se->grid = se->ctx->sms;  // one CTA per SM, all resident (cooperative launch)
            // At most 255 CTAs add into a fused MLP slot, each part below 2^23.
            se->fuse_mlp = md->tarena != nullptr && se->grid <= 255 && fuse_mlp_enabled();
            se->fuse_ao = fuse_attn_o_enabled();
            build_plan(se.get());
            se->mega_ok = true;
            se->use_mega = true;
          } else {
            se->mega_why = "the decode kernel does not fit on an SM";
          }
        } else {
          se->mega_why = "device has no cooperative launch";
        }
      }
      SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
    } catch (...) {
      cudaStreamSynchronize(se->ctx->stream);
      if (se->io) cudaFreeHost(se->io);
      if (se->io_event) cudaEventDestroy(se->io_event);
      for (float* p : se->owned) dev_free(p);
      for (auto* v : {&se->pre, &se->coda})
        for (auto& st : *v)
          if (st.kind == 'G') dev_free(st.k), dev_free(st.v);
      for (auto& l : se->core)
        for (auto& st : l)
          if (st.kind == 'G') dev_free(st.k), dev_free(st.v);
      throw;
    }
    md->refs++;
    *out = se.release();
  });
}

int slm_session_free(slm_session* se) {
  return guard([&] {
    if (!se) return;
    SLM_REQUIRE(se->in_batches == 0, "the session belongs to a batch: free the batch first");
    Device dev(se->ctx);
    cudaStreamSynchronize(se->ctx->stream);
    drop_graph(se);
    for (float* p : se->owned) dev_free(p);
    auto g = [&](LState& st) {
      if (st.kind == 'G') dev_free(st.k), dev_free(st.v);
    };
    for (auto& st : se->pre) g(st);
    for (auto& l : se->core)
      for (auto& st : l) g(st);
    for (auto& st : se->coda) g(st);
    dev_free(se->hist_dev);
    dev_free(se->outs_dev);
    if (se->io) cudaFreeHost(se->io);
    if (se->io_event) cudaEventDestroy(se->io_event);
    if (se->ctx->argmax_owner == se) se->ctx->argmax_owner = nullptr;
    slm_model* md = se->model;
    delete se;
    model_release(md);
  });
}

int slm_session_pos(const slm_session* se, size_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    *out = se->pos;
  });
}

int slm_session_loops(const slm_session* se, size_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    *out = se->loops;
  });
}

int slm_session_set(slm_session* se, int option, int64_t value) {
  return guard([&] {
    SLM_REQUIRE(se, "session is null");
    disarm(se->ctx);  // a launch armed with the old settings must not run
    if (option == SLM_OPT_GRAPH) {
      Device dev(se->ctx);
      se->use_graph = value != 0;
      if (!se->use_graph) drop_graph(se);
      return;
    }
    if (option == SLM_OPT_TRACE) {
      SLM_REQUIRE(se->mega_ok, "tracing needs the persistent decode kernel");
      Device dev(se->ctx);
      if (value && !se->trace) {
        size_t n = (size_t)se->plan_host.nphases * se->grid * 8;
        se->trace = static_cast<unsigned long long*>(alloc_zero(se, n * sizeof(unsigned long long)));
      }
      se->plan_host.trace = value ? se->trace : nullptr;
      return;
    }
    if (option == SLM_OPT_BF16) {
      Device dev(se->ctx);
      const bool on = value != 0;
      if (on) {
        const std::string why = bf16_unsupported(se);
        if (!why.empty()) fail(SLM_ERR_INVALID, "bf16 weights unavailable: " + why);
        build_bf16(se->model);
      }
      if (on == se->wbf16) return;
      SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
      se->wbf16 = on;
      build_plan(se, true);  // the phase descriptors point at the other copies
      se->plan_host.wbytes = on ? 2 : 4;
      SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
      return;
    }
    if (option == SLM_OPT_TEST_STALL) {
      SLM_REQUIRE(se->mega_ok, "the stall test needs the persistent decode kernel");
      se->plan_host.test_stall = value != 0;
      return;
    }
    if (option == SLM_OPT_MEGA) {
      if (value && !se->mega_ok) fail(SLM_ERR_INVALID, "persistent decode kernel unavailable: " + se->mega_why);
      se->use_mega = value != 0;
      return;
    }
    fail(SLM_ERR_INVALID, "unknown option");
  });
}

int slm_session_stat(const slm_session* se, int what, int64_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    if (what == SLM_STAT_STEP_KERNELS) *out = se->use_mega ? 1 : se->step_kernels;
    else if (what == SLM_STAT_GRAPHS) *out = se->graphs;
    else if (what == SLM_STAT_MEGA) *out = se->use_mega ? 1 : 0;
    else if (what == SLM_STAT_PHASES) *out = se->mega_ok ? se->plan_host.nphases : 0;
    else fail(SLM_ERR_INVALID, "unknown counter");
  });
}

int slm_session_trace(slm_session* se, uint64_t* out, size_t cap, size_t* n_out) {
  return guard([&] {
    SLM_REQUIRE(se && n_out && (out || cap == 0), "bad arguments");
    SLM_REQUIRE(se->trace, "tracing is off (SLM_OPT_TRACE)");
    Device dev(se->ctx);
    size_t n = (size_t)se->plan_host.nphases * se->grid * 8;
    *n_out = n;
    if (cap >= n) {
      SLM_CUDA(cudaMemcpyAsync(out, se->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost, se->ctx->stream));
      SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
    }
  });
}

int slm_feed(slm_session* se, const uint32_t* ids, size_t n, size_t limit) {
  return guard([&] {
    SLM_REQUIRE(se && (ids || n == 0), "bad arguments");
    SLM_REQUIRE(limit >= 1, "limit must be at least 1");
    const Config& c = se->model->cfg;
    for (size_t i = 0; i < n; i++) SLM_REQUIRE(ids[i] < c.vocab, "token id out of range");
    Device dev(se->ctx);
    bool global_outside = c.coda.find('G') != std::string::npos || c.prelude.find('G') != std::string::npos;
    size_t at = 0;
    while (at < n) {
      // Model::chunk_at (src/model.rs:647-654).
      size_t chunk = std::min(limit, CHUNK);
      if (global_outside) chunk = std::min(chunk, std::max<size_t>(MAX_SCORES / c.heads / (se->pos + 1), 1));
      size_t m = std::min(chunk, n - at);
      if (m == 1 && se->use_graph) {
        SLM_CUDA(cudaMemcpyAsync(se->ids_dev, ids + at, sizeof(uint32_t), cudaMemcpyHostToDevice, se->ctx->stream));
        step_device(se);  // the last chunk always wants logits; middle ones do too here (harmless)
      } else {
        ensure_caps(se, m);
        SLM_CUDA(cudaMemcpyAsync(se->ids_dev, ids + at, m * sizeof(uint32_t), cudaMemcpyHostToDevice, se->ctx->stream));
        advance(se, m, at + m == n);
      }
      at += m;
    }
  });
}

int slm_step(slm_session* se, uint32_t id) {
  return guard([&] {
    SLM_REQUIRE(se, "session is null");
    SLM_REQUIRE(id < se->model->cfg.vocab, "token id out of range");
    slm_ctx* c = se->ctx;
    const volatile unsigned long long* mb = c->mbox;
    if (se->use_mega && c->armed && c->armed_owner == se && mb[2] != c->armed_seq) {
      // This session's armed launch is waiting: hand it the token.
      *(volatile unsigned long long*)(c->mbox + 8) = (c->armed_seq << 32) | id;
      se->mbox_want = se->fed_seq = c->armed_seq;
      se->fed_id = id;
      c->armed = false;
      c->armed_owner = nullptr;
      se->pos += 1;
      se->argmax_valid = true;
      c->argmax_owner = se;
      if (se->greedy_loop && arm_enabled()) {
        Device dev(c, true);
        arm(se);
      }
      return;
    }
    Device dev(se->ctx);  // (cancels an armed launch that is not this step's)
    if (se->use_mega) {  // the id travels with the launch
      ensure_caps(se, 1);
      mega_step(se, id);
      if (se->greedy_loop && arm_enabled()) arm(se);
      return;
    }
    // The pinned word is read by the copy engine in stream order; wait for an
    // earlier step's copy of it before overwriting.
    if (se->io_busy) SLM_CUDA(cudaEventSynchronize(se->io_event));
    se->io->id_in = id;
    SLM_CUDA(cudaMemcpyAsync(se->ids_dev, &se->io->id_in, sizeof(uint32_t), cudaMemcpyHostToDevice, se->ctx->stream));
    SLM_CUDA(cudaEventRecord(se->io_event, se->ctx->stream));
    se->io_busy = true;
    step_device(se);
  });
}

int slm_logits(slm_session* se, float* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    Device dev(se->ctx);
    SLM_CUDA(cudaMemcpyAsync(out, se->logits, se->model->cfg.vocab * sizeof(float), cudaMemcpyDeviceToHost,
                             se->ctx->stream));
    check_device_error(se->ctx, se);
  });
}

int slm_state_bytes(const slm_session* se, size_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    const Config& c = se->model->cfg;
    size_t dh = c.dh(), total = 0;
    auto one = [&](const LState& st) -> size_t {
      if (st.kind == 'S') return 2 * c.heads * (c.window + CHUNK) * dh;
      if (st.kind == 'L') return c.heads * dh * dh;
      return 2 * c.kv_heads * se->pos * dh + c.d;
    };
    for (auto& st : se->pre) total += one(st);
    for (auto& l : se->core)
      for (auto& st : l) total += one(st);
    for (auto& st : se->coda) total += one(st);
    *out = total * 4;
  });
}

int slm_session_state_count(const slm_session* se, size_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    *out = state_list(const_cast<slm_session*>(se)).size();
  });
}

int slm_session_state_info(const slm_session* se, size_t i, slm_state_array* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    auto list = state_list(const_cast<slm_session*>(se));
    SLM_REQUIRE(i < list.size(), "state array index out of range");
    *out = state_desc(se, list[i]);
  });
}

int slm_session_state_read(slm_session* se, size_t i, float* out) {
  return guard([&] {
    SLM_REQUIRE(se && out, "bad arguments");
    auto list = state_list(se);
    SLM_REQUIRE(i < list.size(), "state array index out of range");
    Device dev(se->ctx);
    const slm_state_array a = state_desc(se, list[i]);
    SLM_CUDA(cudaStreamSynchronize(se->ctx->stream));
    SLM_CUDA(cudaMemcpy(out, state_ptr(list[i]), a.floats * sizeof(float), cudaMemcpyDeviceToHost));
  });
}

int slm_session_state_write(slm_session* se, size_t i, const float* in, size_t cap) {
  return guard([&] {
    SLM_REQUIRE(se && in, "bad arguments");
    auto list = state_list(se);
    SLM_REQUIRE(i < list.size(), "state array index out of range");
    Device dev(se->ctx);
    const StateRef& r = list[i];
    const slm_state_array a = state_desc(se, r);
    float* dst = state_ptr(r);
    cudaStream_t s = se->ctx->stream;
    SLM_CUDA(cudaStreamSynchronize(s));
    if (a.cap == 0) {
      SLM_CUDA(cudaMemcpy(dst, in, a.floats * sizeof(float), cudaMemcpyHostToDevice));
    } else {
      // Ring slots are position mod cap: a window cache must come at its own
      // capacity.  Global caches never wrap: copy the slots both hold.
      if (r.st->kind == 'S')
        SLM_REQUIRE(cap == a.cap, "a window cache must be written at its capacity " + std::to_string(a.cap));
      SLM_REQUIRE(cap > 0, "cap must be positive");
      const size_t rows = std::min(cap, a.cap);
      if (rows < a.cap) SLM_CUDA(cudaMemset(dst, 0, a.floats * sizeof(float)));
      SLM_CUDA(cudaMemcpy2D(dst, a.cap * a.dh * sizeof(float), in, cap * a.dh * sizeof(float),
                            rows * a.dh * sizeof(float), a.heads, cudaMemcpyHostToDevice));
    }
    if (r.st->kind == 'G') se->keys_stale = true;
    se->argmax_valid = false;
  });
}

int slm_session_set_pos(slm_session* se, size_t pos) {
  return guard([&] {
    SLM_REQUIRE(se, "session is null");
    Device dev(se->ctx);
    cudaStream_t s = se->ctx->stream;
    SLM_CUDA(cudaStreamSynchronize(s));
    se->pos = pos;
    long long p = (long long)pos;
    SLM_CUDA(cudaMemcpy(se->pos_dev, &p, sizeof(p), cudaMemcpyHostToDevice));
    ensure_caps(se, 1);  // global caches hold the next step
    SLM_CUDA(cudaStreamSynchronize(s));
    se->keys_stale = true;
    se->argmax_valid = false;
  });
}

uint64_t slm_rng_seed(uint64_t seed) { return seed * 0x9E3779B97F4A7C15ull | 1; }

int slm_sample(slm_session* se, const slm_sampling* sp, const uint32_t* recent, size_t n_recent, uint64_t* rng_state,
               uint32_t* out_id) {
  return guard([&] {
    SLM_REQUIRE(se && rng_state && out_id && (recent || n_recent == 0), "bad arguments");
    check_sampling(sp);
    cudaStream_t s = se->ctx->stream;
    // Greedy without a penalty on logits of a persistent step: that step
    // already computed the arg-max (same order: first maximum, NaN never
    // wins) and pick draws nothing from the RNG (src/sample.rs:33-45).
    const bool fast = se->argmax_valid && sp->temperature <= 0.0f && (sp->repeat_penalty == 1.0f || n_recent == 0);
    se->greedy_loop = false;
    {
      slm_ctx* c = se->ctx;
      if (fast && c->argmax_owner == se && se->mbox_want) {
        // (This session's armed next step, queued behind, stays armed.)
        Device dev(c, true);
        // slm_step's launch hands its arg-max over in the mailbox: poll it
        // while the stream runs; a step that gave up writes none, so once the
        // stream is idle without it, the copy below reports the error.
        unsigned long long want = se->mbox_want;
        se->mbox_want = 0;
        const volatile unsigned long long* mb = c->mbox;
        bool got = false;
        for (int attempt = 0; attempt < 2; attempt++) {
          for (unsigned it = 1;; it++) {
            if (mb[0] == want) {
              got = true;
              break;
            }
            if ((it & 255) == 0 && cudaStreamQuery(s) != cudaErrorNotReady) {
              got = mb[0] == want;
              break;
            }
#if defined(__x86_64__)
            __builtin_ia32_pause();
#endif
          }
          if (got || se->fed_seq != want || mb[2] != want) break;
          // The armed launch ran out of time before slm_step's token reached
          // it and ended without its step: run that step now (after ending
          // the launch armed behind it).
          disarm(c);
          se->pos -= 1;
          mega_step(se, se->fed_id);
          want = se->mbox_want;
          se->mbox_want = 0;
        }
        if (cudaPeekAtLastError() == cudaErrorNotReady) (void)cudaGetLastError();  // the queries' answer, not an error
        if (got) {
          std::atomic_thread_fence(std::memory_order_acquire);
          const unsigned long long w = mb[1];
          if ((w >> 32) == 0) {
            se->io_busy = false;
            *out_id = static_cast<uint32_t>(w);
            se->greedy_loop = se->use_mega;  // slm_step arms the steps after the next one
            return;
          }
        }
      }
    }
    Device dev(se->ctx);
    if (fast) {
      slm_ctx* c = se->ctx;
      if (c->argmax_owner == se) {  // one copy: the error word and this step's arg-max beside it
        SLM_CUDA(cudaMemcpyAsync(c->err_host, c->err, 2 * sizeof(int), cudaMemcpyDeviceToHost, s));
        SLM_CUDA(cudaStreamSynchronize(s));
        if (c->err_host[0]) check_device_error(c, se);  // reports it
        se->io_busy = false;
        *out_id = static_cast<uint32_t>(c->err_host[1]);
        return;
      }
      SLM_CUDA(cudaMemcpyAsync(&se->io->id_out, se->argmax_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
      check_device_error(c, se);
      se->io_busy = false;  // the stream is idle
      *out_id = se->io->id_out;
      return;
    }
    ensure_u32(se, &se->hist_dev, &se->hist_cap, n_recent + 1);
    if (n_recent)
      SLM_CUDA(cudaMemcpyAsync(se->hist_dev, recent, n_recent * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    if (se->io_busy) SLM_CUDA(cudaEventSynchronize(se->io_event));
    se->io->rng_in = *rng_state;
    SLM_CUDA(cudaMemcpyAsync(se->rng_dev, &se->io->rng_in, sizeof(unsigned long long), cudaMemcpyHostToDevice, s));
    SampleArgs a = sample_args(se, sp);
    a.recent = se->hist_dev;
    a.nrecent = (long long)n_recent;
    a.out = se->out_dev;
    sample(a, s);
    SLM_CUDA(cudaMemcpyAsync(&se->io->id_out, se->out_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    SLM_CUDA(cudaMemcpyAsync(&se->io->rng_out, se->rng_dev, sizeof(unsigned long long), cudaMemcpyDeviceToHost, s));
    check_device_error(se->ctx, se);
    se->io_busy = false;
    *out_id = se->io->id_out;
    *rng_state = se->io->rng_out;
  });
}

int slm_pick(slm_ctx* c, const slm_buf* logits, size_t vocab, const slm_sampling* sp, const uint32_t* recent,
             size_t n_recent, uint64_t* rng_state, uint32_t* out_id) {
  return guard([&] {
    SLM_REQUIRE(c && rng_state && out_id && (recent || n_recent == 0) && vocab > 0, "bad arguments");
    SLM_REQUIRE(vocab < (1u << 31), "vocab too large");
    check_sampling(sp);
    const float* l = view(logits, 0, vocab, "pick logits");
    Device dev(c);
    cudaStream_t s = c->stream;
    const size_t work = 3 * vocab;  // sampler: logits, sorted weights, sorted ids
    size_t words = work + n_recent + 8;
    float* scratch = static_cast<float*>(dev_alloc(words * sizeof(float)));
    struct Free {
      float* p;
      ~Free() { dev_free(p); }
    } fr{scratch};
    auto* hist = reinterpret_cast<uint32_t*>(scratch + work);
    auto* rng = reinterpret_cast<unsigned long long*>(scratch + work + n_recent + 2 - ((work + n_recent) & 1));
    auto* outd = reinterpret_cast<uint32_t*>(rng + 2);
    if (n_recent) SLM_CUDA(cudaMemcpyAsync(hist, recent, n_recent * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    unsigned long long st = *rng_state;
    SLM_CUDA(cudaMemcpyAsync(rng, &st, sizeof(st), cudaMemcpyHostToDevice, s));
    SampleArgs a{};
    a.logits = l;
    a.work = scratch;
    a.vocab = (int)vocab;
    a.temperature = sp->temperature, a.top_p = sp->top_p, a.penalty = sp->repeat_penalty;
    a.top_k = sp->top_k, a.window = sp->repeat_window;
    a.recent = hist, a.nrecent = (long long)n_recent;
    a.rng = rng, a.out = outd, a.err = c->err;
    sample(a, s);
    uint32_t id = 0;
    SLM_CUDA(cudaMemcpyAsync(&id, outd, sizeof(id), cudaMemcpyDeviceToHost, s));
    SLM_CUDA(cudaMemcpyAsync(&st, rng, sizeof(st), cudaMemcpyDeviceToHost, s));
    check_device_error(c);
    *out_id = id;
    *rng_state = st;
  });
}

int slm_decode(slm_session* se, uint32_t first, size_t n, const slm_sampling* sp, const uint32_t* recent,
               size_t n_recent, uint64_t* rng_state, uint32_t* out) {
  return guard([&] {
    SLM_REQUIRE(se && rng_state && (out || n == 0) && (recent || n_recent == 0), "bad arguments");
    SLM_REQUIRE(first < se->model->cfg.vocab, "token id out of range");
    check_sampling(sp);
    if (n == 0) return;
    Device dev(se->ctx);
    cudaStream_t s = se->ctx->stream;
    ensure_u32(se, &se->hist_dev, &se->hist_cap, n_recent + n + 1);
    ensure_u32(se, &se->outs_dev, &se->outs_cap, n);
    if (n_recent)
      SLM_CUDA(cudaMemcpyAsync(se->hist_dev, recent, n_recent * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    unsigned long long st = *rng_state;
    SLM_CUDA(cudaMemcpyAsync(se->rng_dev, &st, sizeof(st), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemcpyAsync(se->ids_dev, &first, sizeof(first), cudaMemcpyHostToDevice, s));
    SampleArgs a = sample_args(se, sp);
    a.recent = se->hist_dev;
    a.hist_out = se->hist_dev;
    a.next_id = se->ids_dev;
    const bool fused = se->use_mega && sp->temperature <= 0.0f && sp->repeat_penalty == 1.0f;
    if (fused) plan_outputs(se, true, se->outs_dev, se->hist_dev, n_recent);
    try {
      if (fused) {
        mega_steps(se, n);  // each step's own arg-max is the next id
      } else {
        for (size_t t = 0; t < n; t++) {
          step_device(se);
          a.nrecent = (long long)(n_recent + t);
          a.out = se->outs_dev + t;
          sample(a, s);
        }
      }
    } catch (...) {
      if (fused) plan_outputs(se, false, nullptr, nullptr, 0);
      throw;
    }
    if (fused) plan_outputs(se, false, nullptr, nullptr, 0);
    SLM_CUDA(cudaMemcpyAsync(out, se->outs_dev, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    SLM_CUDA(cudaMemcpyAsync(&st, se->rng_dev, sizeof(st), cudaMemcpyDeviceToHost, s));
    check_device_error(se->ctx, se);
    *rng_state = st;
  });
}

int slm_batch_new(slm_session* const* sessions, size_t n, slm_batch** out) {
  return guard([&] {
    SLM_REQUIRE(sessions && out && n >= 1, "bad arguments");
    slm_model* md = sessions[0] ? sessions[0]->model : nullptr;
    SLM_REQUIRE(md, "bad arguments");
    const Config& c = md->cfg;
    for (size_t i = 0; i < n; i++) {
      SLM_REQUIRE(sessions[i] && sessions[i]->model == md, "every session of a batch must use the same model");
      SLM_REQUIRE(sessions[i]->loops == sessions[0]->loops, "every session of a batch must run the same loops");
      for (size_t j = 0; j < i; j++) SLM_REQUIRE(sessions[j] != sessions[i], "a session appears twice in the batch");
    }
    Device dev(md->ctx);
    auto bt = std::make_unique<slm_batch>();
    bt->model = md, bt->ctx = md->ctx, bt->n = n;
    bt->ses.assign(sessions, sessions + n);
    cudaStream_t s = md->ctx->stream;
    try {
      const size_t d = c.d;
      auto f = [&](size_t k) { return static_cast<float*>(balloc(bt.get(), k * sizeof(float))); };
      bt->xa = f(n * d), bt->xb = f(n * d), bt->e0 = f(n * d), bt->e_proj = f(n * d), bt->nb = f(n * d);
      bt->mix = f(n * md->mix_cols), bt->q = f(n * d), bt->kb = f(n * d), bt->y = f(n * d);
      bt->mid = f(n * std::max<size_t>(md->hidden, 1)), bt->upbuf = f(n * 2 * std::max<size_t>(md->hidden, 1));
      bt->dec = f(n * c.heads), bt->logits = f(n * c.vocab);
      // Attention splits: about 16 resident 128-thread CTAs per SM over
      // heads × n rows (enough loads in flight to stream the rings), at least
      // 128 positions per slice.
      const long long ctas = (long long)c.heads * (long long)n;
      long long want = (16 * bt->ctx->sms + ctas - 1) / ctas, most = ((long long)c.window + 127) / 128;
      bt->nsplit = (int)std::max<long long>(1, std::min<long long>(std::min(want, most), 256));
      // Global layers see up to the whole history: as many splits as a
      // window's worth of CTAs allows, slices of at least 512 positions.
      bt->gsplit = (int)std::max<long long>(1, std::min<long long>(want * 2, 256));
      AttnGeom g{(int)n, 0, 0, 1, (int)c.heads, 1, (int)c.dh(), 1.0f};
      bt->part = f(attn_part_floats(g, std::max(bt->nsplit, bt->gsplit)));
      bt->merge_cnt = static_cast<unsigned*>(balloc(bt.get(), c.heads * n * sizeof(unsigned)));
      bt->ids = static_cast<uint32_t*>(balloc(bt.get(), n * sizeof(uint32_t)));
      bt->out_index = static_cast<unsigned*>(balloc(bt.get(), 4 * sizeof(unsigned)));
      bt->outs = static_cast<uint32_t*>(balloc(bt.get(), n * sizeof(uint32_t)));
      bt->outs_cap = 1;
      std::vector<long long*> pos(n);
      for (size_t i = 0; i < n; i++) pos[i] = sessions[i]->pos_dev;
      bt->posr = static_cast<long long**>(balloc(bt.get(), n * sizeof(long long*)));
      SLM_CUDA(cudaMemcpyAsync(bt->posr, pos.data(), n * sizeof(long long*), cudaMemcpyHostToDevice, s));
      bt->kvs = f(n * c.kv_heads * c.dh());
      const size_t ninst = md->prelude.size() + sessions[0]->loops * md->core.size() + md->coda.size();
      for (size_t k = 0; k < ninst; k++) {
        bt->tab.push_back(static_cast<float**>(balloc(bt.get(), 4 * n * sizeof(float*))));
        bt->caps.push_back(static_cast<long long*>(balloc(bt.get(), n * sizeof(long long))));
      }
      batch_tables(bt.get());
    } catch (...) {
      cudaStreamSynchronize(s);
      for (void* p : bt->owned) dev_free(p);
      throw;
    }
    for (auto* se : bt->ses) se->in_batches++;
    *out = bt.release();
  });
}

int slm_batch_free(slm_batch* bt) {
  return guard([&] {
    if (!bt) return;
    Device dev(bt->ctx);
    cudaStreamSynchronize(bt->ctx->stream);
    batch_drop_graph(bt);
    for (void* p : bt->owned) dev_free(p);
    for (auto* se : bt->ses) se->in_batches--;
    delete bt;
  });
}

int slm_batch_size(const slm_batch* bt, size_t* out) {
  return guard([&] {
    SLM_REQUIRE(bt && out, "bad arguments");
    *out = bt->n;
  });
}

int slm_batch_step(slm_batch* bt, const uint32_t* ids) {
  return guard([&] {
    SLM_REQUIRE(bt && ids, "bad arguments");
    for (size_t i = 0; i < bt->n; i++) SLM_REQUIRE(ids[i] < bt->model->cfg.vocab, "token id out of range");
    Device dev(bt->ctx);
    cudaStream_t s = bt->ctx->stream;
    SLM_CUDA(cudaMemcpyAsync(bt->ids, ids, bt->n * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemsetAsync(bt->out_index, 0, sizeof(unsigned), s));
    batch_step_device(bt);
    check_device_error(bt->ctx);
  });
}

int slm_batch_logits(slm_batch* bt, float* out) {
  return guard([&] {
    SLM_REQUIRE(bt && out, "bad arguments");
    Device dev(bt->ctx);
    cudaStream_t s = bt->ctx->stream;
    SLM_CUDA(cudaMemcpyAsync(out, bt->logits, bt->n * bt->model->cfg.vocab * sizeof(float), cudaMemcpyDeviceToHost,
                             s));
    SLM_CUDA(cudaStreamSynchronize(s));
  });
}

int slm_batch_decode(slm_batch* bt, const uint32_t* first, size_t steps, uint32_t* out) {
  return guard([&] {
    SLM_REQUIRE(bt && first && (out || steps == 0), "bad arguments");
    for (size_t i = 0; i < bt->n; i++) SLM_REQUIRE(first[i] < bt->model->cfg.vocab, "token id out of range");
    if (steps == 0) return;
    Device dev(bt->ctx);
    cudaStream_t s = bt->ctx->stream;
    batch_outs(bt, steps);
    SLM_CUDA(cudaMemcpyAsync(bt->ids, first, bt->n * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemsetAsync(bt->out_index, 0, sizeof(unsigned), s));
    for (size_t t = 0; t < steps; t++) batch_step_device(bt);
    SLM_CUDA(cudaMemcpyAsync(out, bt->outs, steps * bt->n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    check_device_error(bt->ctx);
  });
}

int slm_batch_sample_decode(slm_batch* bt, const uint32_t* first, size_t steps, const slm_sampling* sp,
                            const uint32_t* const* recent, const size_t* n_recent, uint64_t* rng_state,
                            uint32_t* out) {
  return guard([&] {
    SLM_REQUIRE(bt && first && sp && rng_state && (out || steps == 0), "bad arguments");
    const size_t n = bt->n, V = bt->model->cfg.vocab;
    size_t most = 0;
    for (size_t i = 0; i < n; i++) {
      SLM_REQUIRE(first[i] < V, "token id out of range");
      check_sampling(sp + i);
      const size_t r = n_recent ? n_recent[i] : 0;
      SLM_REQUIRE(r == 0 || (recent && recent[i]), "bad arguments");
      most = std::max(most, r);
    }
    if (steps == 0) return;
    Device dev(bt->ctx);
    cudaStream_t s = bt->ctx->stream;
    batch_outs(bt, steps);
    if (!bt->srows) {
      bt->srows = static_cast<SampleArgs*>(balloc(bt, n * sizeof(SampleArgs)));
      bt->swork = static_cast<float*>(balloc(bt, n * 3 * V * sizeof(float)));
      bt->srng = static_cast<unsigned long long*>(balloc(bt, n * sizeof(unsigned long long)));
    }
    if (most + steps > bt->shist_cap) {  // the rows' histories, each with room for the sampled ids
      SLM_CUDA(cudaStreamSynchronize(s));
      const size_t cap = std::max<size_t>(1024, std::max(most + steps, 2 * bt->shist_cap));
      auto* p = static_cast<uint32_t*>(dev_alloc(n * cap * sizeof(uint32_t)));
      for (auto& o : bt->owned)
        if (o == bt->shist) {
          dev_free(o);
          o = p;
        }
      if (!bt->shist) bt->owned.push_back(p);
      bt->shist = p;
      bt->shist_cap = cap;
    }
    std::vector<SampleArgs> rows(n);
    for (size_t i = 0; i < n; i++) {
      const size_t r = n_recent ? n_recent[i] : 0;
      uint32_t* h = bt->shist + i * bt->shist_cap;
      if (r) SLM_CUDA(cudaMemcpyAsync(h, recent[i], r * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
      SampleArgs& a = rows[i];
      a = SampleArgs{};
      a.logits = bt->logits + i * V;
      a.work = bt->swork + i * 3 * V;
      a.vocab = (int)V;
      a.temperature = sp[i].temperature, a.top_p = sp[i].top_p, a.penalty = sp[i].repeat_penalty;
      a.top_k = sp[i].top_k, a.window = sp[i].repeat_window;
      a.recent = h, a.nrecent = (long long)r, a.hist_out = h;
      a.rng = bt->srng + i;
      a.next_id = bt->ids + i;
      a.err = bt->ctx->err;
    }
    SLM_CUDA(cudaMemcpyAsync(bt->srows, rows.data(), n * sizeof(SampleArgs), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemcpyAsync(bt->srng, rng_state, n * sizeof(uint64_t), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemcpyAsync(bt->ids, first, n * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    SLM_CUDA(cudaMemsetAsync(bt->out_index, 0, sizeof(unsigned), s));
    for (size_t t = 0; t < steps; t++) batch_step_device(bt, true);
    SLM_CUDA(cudaMemcpyAsync(out, bt->outs, steps * n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    SLM_CUDA(cudaMemcpyAsync(rng_state, bt->srng, n * sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
    check_device_error(bt->ctx);
  });
}

}  // extern "C"
