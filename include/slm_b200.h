/*
 * slm_b200.h — C ABI of the B200 (sm_100a) backend for the SLM.use token loop.
 *
 * Two levels, both plain C: opaque handles, pointers and sizes, an int status
 * on every call (0 = ok; the message of the last failure on this thread comes
 * from slm_last_error()).  Nothing here throws or aborts.
 *
 * 1. Op level: one entry point per method of the reference's `Ops` trait
 *    (reference src/ops.rs:68-228), on device buffers (`slm_buf`).  A buffer
 *    stands for `Ops::Buf`; an (slm_buf*, offset) pair stands for `At`
 *    (src/ops.rs:13-29).  Output buffers that are too small are reallocated,
 *    as the reference CUDA backend's `ensure` does (src/cuda.rs:122-127).
 *    Calls are asynchronous on the context's stream; slm_read synchronises
 *    (src/cuda.rs:160-165).
 *
 * 2. Model level: what the reference's `Model`/`Session` offer
 *    (src/model.rs:225-690) — load, session, feed, step, logits,
 *    state_bytes — plus on-device sampling (src/sample.rs:33-93) and an
 *    n-token decode that keeps every id on the device.  This level runs the
 *    fused sm_100a kernels and captures the m = 1 token step in a CUDA graph.
 *
 * Threading: a context owns one device and one stream; use a context from one
 * host thread at a time (the reference pins its model to one thread,
 * src/serve.rs:1-3).  Sessions of one model may live on different contexts.
 */
#ifndef SLM_B200_H
#define SLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SLM_OK 0
#define SLM_ERR_INVALID 1  /* bad argument or shape */
#define SLM_ERR_CUDA 2     /* a CUDA call failed */
#define SLM_ERR_IO 3       /* a model file could not be read or parsed */
#define SLM_ERR_NOMEM 4    /* device allocation failed */
#define SLM_ERR_DEVICE 5   /* a kernel reported an error word (bounded wait expired, bad id) */

typedef struct slm_ctx slm_ctx;
typedef struct slm_buf slm_buf;
typedef struct slm_model slm_model;
typedef struct slm_session slm_session;
typedef struct slm_batch slm_batch;

/* Message of the last failed call on this thread ("" if none). */
const char* slm_last_error(void);
/* Library version string. */
const char* slm_version(void);

/* ---------------------------------------------------------------------- */
/* Context (replaces Cuda::probe, reference src/cuda.rs:71-120).           */
/* ---------------------------------------------------------------------- */

/* Number of visible CUDA devices (0 when there is no driver or GPU). */
int slm_device_count(int* out);
/* Binds `device`, creates a stream.  Fails with SLM_ERR_CUDA when the device
 * is not an sm_100 part or cannot be opened. */
int slm_ctx_new(int device, slm_ctx** out);
int slm_ctx_free(slm_ctx* ctx);
/* Device name, as Ops::name (src/ops.rs:71, src/cuda.rs:145-150). */
int slm_ctx_name(slm_ctx* ctx, char* out, size_t cap);
/* Waits for all work on the context's stream. */
int slm_ctx_sync(slm_ctx* ctx);
/* The context's cudaStream_t (as void*), for callers that time or order work
 * around the library's launches. */
int slm_ctx_stream(slm_ctx* ctx, void** out);

/* ---------------------------------------------------------------------- */
/* Buffers: Ops::zeros / upload / read / flush (src/ops.rs:72-91).         */
/* ---------------------------------------------------------------------- */

int slm_zeros(slm_ctx* ctx, size_t n, slm_buf** out);
int slm_upload(slm_ctx* ctx, const float* data, size_t n, slm_buf** out);
/* Waits for pending work and copies the first n values to `out`. */
int slm_read(slm_ctx* ctx, const slm_buf* buf, size_t n, float* out);
int slm_buf_free(slm_buf* buf);
size_t slm_buf_len(const slm_buf* buf);
/* Device address of the buffer's first value (valid until it is resized). */
float* slm_buf_ptr(slm_buf* buf);
/* Ops::flush: a no-op, kept for the trait's shape (src/cuda.rs:167-169). */
int slm_flush(slm_ctx* ctx);

/* ---------------------------------------------------------------------- */
/* Op level: one call per Ops method.  Offsets are in floats.              */
/* ---------------------------------------------------------------------- */

/* Ops::gather (src/ops.rs:94): y[i] = w[ids[i]], ids on the host. */
int slm_op_gather(slm_ctx* ctx, slm_buf* y, const slm_buf* w, const uint32_t* ids, size_t m, size_t d);
/* Ops::copy (src/ops.rs:95). */
int slm_op_copy(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, size_t n);
/* Ops::shift (src/ops.rs:97-104): y[0] = first, y[i] = x[i-1]. */
int slm_op_shift(slm_ctx* ctx, slm_buf* y, const slm_buf* first, const slm_buf* x, size_t xoff,
                 size_t m, size_t d);
/* Ops::columns (src/ops.rs:107-115). */
int slm_op_columns(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t m, size_t stride, size_t off,
                   size_t len);
/* Ops::linear (src/ops.rs:118-126): y[i] = w·x[i], w rows × cols row-major. */
int slm_op_linear(slm_ctx* ctx, slm_buf* y, const slm_buf* w, size_t rows, size_t cols,
                  const slm_buf* x, size_t xoff, size_t m);
/* Ops::add (src/ops.rs:127). */
int slm_op_add(slm_ctx* ctx, slm_buf* y, const slm_buf* a, size_t aoff, const slm_buf* b, size_t boff,
               size_t n);
/* Ops::add_row (src/ops.rs:129-136). */
int slm_op_add_row(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* row,
                   size_t rowoff, size_t m, size_t d);
/* Ops::scale_rows (src/ops.rs:138): factors on the host, m = number of factors. */
int slm_op_scale_rows(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, const float* f, size_t m,
                      size_t d);
/* Ops::mix (src/ops.rs:140-147): y = a + t·(b − a). */
int slm_op_mix(slm_ctx* ctx, slm_buf* y, const slm_buf* a, size_t aoff, const slm_buf* b, size_t boff,
               size_t n, float t);
/* Ops::rms (src/ops.rs:150-158). */
int slm_op_rms(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* w, size_t groups,
               size_t size, float eps);
/* Ops::silu_mul (src/ops.rs:160-166): y = silu(g)·u. */
int slm_op_silu_mul(slm_ctx* ctx, slm_buf* y, const slm_buf* g, size_t goff, const slm_buf* u,
                    size_t uoff, size_t n);
/* Ops::rope_table (src/ops.rs:169-177). */
int slm_op_rope_table(slm_ctx* ctx, slm_buf* cos_out, slm_buf* sin_out, const slm_buf* inv, size_t pos,
                      size_t m, size_t half);
/* Ops::rope (src/ops.rs:179-188). */
int slm_op_rope(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, const slm_buf* cos_in,
                const slm_buf* sin_in, size_t m, size_t heads, size_t dh);
/* Ops::l2norm (src/ops.rs:190). */
int slm_op_l2norm(slm_ctx* ctx, slm_buf* y, const slm_buf* x, size_t xoff, size_t heads, size_t dh);
/* Ops::gla (src/ops.rs:191-205). */
int slm_op_gla(slm_ctx* ctx, slm_buf* y, slm_buf* s, const slm_buf* q, size_t qoff, const slm_buf* k,
               size_t koff, const slm_buf* v, size_t voff, const slm_buf* decay, const slm_buf* bias,
               size_t m, size_t heads, size_t dh);
/* Ops::store (src/ops.rs:207-217). */
int slm_op_store(slm_ctx* ctx, slm_buf* cache, const slm_buf* src, size_t srcoff, size_t pos, size_t m,
                 size_t cap, size_t heads, size_t dh);

/* Attn (src/ops.rs:31-46).  reach = SIZE_MAX means unbounded. */
typedef struct slm_attn {
  size_t pos, m, reach, gap, cap, heads, key_heads, dh;
  float scale;
} slm_attn;
/* Ops::attend (src/ops.rs:218-227).  `scores` is scratch (resized as needed). */
int slm_op_attend(slm_ctx* ctx, slm_buf* y, slm_buf* scores, const slm_buf* q, size_t qoff,
                  const slm_buf* k, const slm_buf* v, const slm_attn* a);

/* Ops::attend without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc — code running
 * between kernels of a latency-critical loop (cudaMalloc/cudaFree may
 * synchronise the device) or a process whose device memory is reserved up
 * front by its own allocator.  y, q, k, v are device pointers laid out as for
 * slm_op_attend (q and y: m × heads × dh; k, v: key_heads × cap × dh).  The
 * scratch is a fixed 4 MiB __device__ array per device: calls need
 * m·heads·(dh + 2) ≤ 1,048,512 floats and fail with SLM_ERR_INVALID above
 * it.  The first call on a device looks up that array's address (set-up, no
 * allocation); make that first call before any stream capture.  The address is
 * kept for the life of the process: it assumes the device's primary context
 * stays alive (no cudaDeviceReset, no release of the primary context between
 * calls).  All calls on a device share the array, so calls that overlap on the
 * GPU race. */
int slm_op_attend_noalloc(slm_ctx* ctx, float* y, const float* q, const float* k, const float* v,
                          const slm_attn* a);

/* ---------------------------------------------------------------------- */
/* Model level (src/model.rs, src/sample.rs).                              */
/* ---------------------------------------------------------------------- */

typedef struct slm_model_info {
  size_t vocab, d_model, heads, head_dim, kv_heads, hidden, window, max_loops, default_loops;
  size_t params; /* Model::params (src/model.rs:275-302) */
  char prelude[32], core[32], coda[32];
} slm_model_info;

/* Model::load (src/model.rs:226-269): `dir` holds config.json and model.safetensors (f32). */
int slm_model_load(slm_ctx* ctx, const char* dir, slm_model** out);
int slm_model_free(slm_model* model);
int slm_model_info_get(const slm_model* model, slm_model_info* out);

/* Model::session (src/model.rs:333-381); loops = 0 takes the default. */
int slm_session_new(slm_model* model, size_t loops, slm_session** out);
int slm_session_free(slm_session* se);
int slm_session_pos(const slm_session* se, size_t* out);
int slm_session_loops(const slm_session* se, size_t* out);
/* Model::feed (src/model.rs:658-667): chunks of at most `limit` (≤ 256). */
int slm_feed(slm_session* se, const uint32_t* ids, size_t n, size_t limit);
/* Model::step (src/model.rs:643-645). */
int slm_step(slm_session* se, uint32_t id);
/* Model::logits (src/model.rs:669-671): copies vocab floats, synchronises. */
int slm_logits(slm_session* se, float* out);
/* Model::state_bytes (src/model.rs:674-690). */
int slm_state_bytes(const slm_session* se, size_t* out);

/* ---- Session state transfer ------------------------------------------------
 * No counterpart in the reference, whose Session keeps its state private
 * (src/model.rs:210-223).  The recurrent state of a session as host arrays:
 * a snapshot to restore later, or a start at a chosen position without
 * reading a prompt first (the parity tests start the library and the CPU
 * oracle from the same state this way).  Arrays come in step order (the
 * prelude's blocks, then the core's blocks for loop 0, 1, …, then the coda's);
 * per block: window attention 'S' → k, v; GLA 'L' → s; global 'G' → k, v, p. */
typedef struct slm_state_array {
  char kind;     /* layer type of the block: 'S', 'L' or 'G' */
  char part;     /* 'k', 'v': cache [heads][cap][dh] (slot = position mod cap
                    for 'S'; positions in order for 'G'); 's': GLA state
                    [heads][dh][dh]; 'p': a G block's previous normalised
                    input (d floats, the shifted-key source) */
  size_t heads;  /* cache or state heads (1 for 'p') */
  size_t cap;    /* cache slots per head (0 for 's' and 'p') */
  size_t dh;     /* head size (d for 'p') */
  size_t floats; /* values in the array */
} slm_state_array;
int slm_session_state_count(const slm_session* se, size_t* out);
int slm_session_state_info(const slm_session* se, size_t i, slm_state_array* out);
/* Copies array i (info.floats values) to `out` on the host; synchronises. */
int slm_session_state_read(slm_session* se, size_t i, float* out);
/* Overwrites array i from the host.  A cache comes as [heads][cap][dh]: a
 * window cache at exactly its own capacity (ring slots depend on it); for a
 * global cache the first min(cap, info.cap) slots per head are copied and the
 * rest zeroed.  Synchronises. */
int slm_session_state_write(slm_session* se, size_t i, const float* in, size_t cap);
/* Puts the session at position `pos` (global caches grow to hold the next
 * step) without touching its arrays; write them before or after.  The next
 * step runs at `pos`.  Synchronises. */
int slm_session_set_pos(slm_session* se, size_t pos);

/* Sampling (src/sample.rs:3-15). */
typedef struct slm_sampling {
  float temperature;      /* 0 picks the most likely token */
  uint32_t top_k;         /* 0 keeps every token */
  float top_p;            /* 1 keeps them all */
  float repeat_penalty;   /* 1 disables the penalty */
  uint32_t repeat_window; /* how many recent tokens the penalty looks at */
} slm_sampling;

/* xorshift64* seeding, Rng::new (src/sample.rs:21-23). */
uint64_t slm_rng_seed(uint64_t seed);

/* pick (src/sample.rs:33-93) on the device, from the session's logits.
 * `recent` (host, n_recent ids) is the history the repeat penalty reads;
 * `rng_state` is read and advanced.  Candidates after top-k are kept in a
 * canonical order (logit descending, then id ascending).  Synchronises.
 * Greedy without a penalty, right after this session's slm_step on the
 * persistent kernel: returns the arg-max that step computed, as soon as the
 * step's mailbox (mapped pinned host memory) shows it, busy-waiting the
 * calling thread for the step (about one step's time, 0.2 ms at R = 4).
 * In such a greedy slm_step/slm_sample loop, slm_step also queues the next
 * persistent step behind the one it issues ("armed": it waits on the GPU,
 * for at most 20 ms, for the token the next slm_step writes to mapped
 * memory); any other call on the context cancels it, and one that times out
 * is replaced by a plain launch.  SLM_MEGA_ARM=0 in the environment turns
 * this off; so do CUDA_LAUNCH_BLOCKING=1 and any tool that makes launches
 * return only after the kernel ends (detected at the first armed launch). */
int slm_sample(slm_session* se, const slm_sampling* s, const uint32_t* recent, size_t n_recent,
               uint64_t* rng_state, uint32_t* out_id);

/* pick (src/sample.rs:33-93) on any device logits: `logits` holds at least
 * `vocab` floats; otherwise as slm_sample.  Synchronises. */
int slm_pick(slm_ctx* ctx, const slm_buf* logits, size_t vocab, const slm_sampling* s, const uint32_t* recent,
             size_t n_recent, uint64_t* rng_state, uint32_t* out_id);

/* n decode steps without leaving the device: feeds `first`, then each
 * sampled id, and writes the n sampled ids to `out` (host).  `recent` seeds
 * the penalty history; sampled ids join it.  Equivalent to n rounds of
 * slm_step + slm_sample.  Synchronises once at the end. */
int slm_decode(slm_session* se, uint32_t first, size_t n, const slm_sampling* s, const uint32_t* recent,
               size_t n_recent, uint64_t* rng_state, uint32_t* out);

/* Execution switches of a session (for tests and measurement):
 *   SLM_OPT_GRAPH    1 = replay the m = 1 step as a CUDA graph (default 1)
 *   SLM_OPT_MEGA     1 = run the m = 1 step as one persistent kernel (default
 *                    1 where the model allows it: head size 64, d_model
 *                    128·{1,2,3,4,6,8} up to 1024, damp 1, and global layers,
 *                    if any, with heads / kv_heads ≤ 3 that open neither the
 *                    prelude nor the loop; fails with SLM_ERR_INVALID
 *                    otherwise) */
#define SLM_OPT_GRAPH 1
#define SLM_OPT_MEGA 2
#define SLM_OPT_TRACE 3 /* 1 = record the per-phase timeline of each persistent step */
/* Test hook: 1 = the persistent step's first grid barrier waits for an arrival
 * that never comes, so its bounded wait (~2 s) expires and the step reports
 * SLM_ERR_DEVICE at the next synchronising call.  The session's state is then
 * undefined; the context stays usable. */
#define SLM_OPT_TEST_STALL 4
/* 1 = the persistent step streams bf16 copies of its matrices (rounded to
 * nearest once per model, on the first request) with f32 arithmetic, caches
 * and state: half the weight bytes per token.  Not a parity mode: logits
 * differ from f32 weights by the weights' rounding.  Needs the persistent
 * kernel with its fused phases and d_model a multiple of 256, at most 768;
 * SLM_ERR_INVALID otherwise.  No counterpart in the reference (its MLX
 * backend offers fp16 weights, src/mlx.rs:14-23). */
#define SLM_OPT_BF16 5
int slm_session_set(slm_session* se, int option, int64_t value);

/* Counters of a session:
 *   SLM_STAT_STEP_KERNELS  kernels one m = 1 step launches (graph nodes)
 *   SLM_STAT_GRAPHS        step graphs captured so far */
#define SLM_STAT_STEP_KERNELS 1
#define SLM_STAT_GRAPHS 2
#define SLM_STAT_MEGA 3    /* 1 when the persistent decode kernel is in use */
#define SLM_STAT_PHASES 4  /* phases (grid barriers + 1) of that kernel's step */
int slm_session_stat(const slm_session* se, int what, int64_t* out);

/* Timeline of the last persistent step (SLM_OPT_TRACE on): for each phase p
 * and CTA c, eight values at out[(p·grid + c)·8]: the globaltimer (ns) when
 * the CTA began the phase's work and when it reached the next grid barrier;
 * the ns it spent waiting for tiles, building the phase's input, on tile
 * arithmetic and in GEMV epilogues; the GEMV tiles it took; 0.
 * *n_out receives the count; nothing is copied when cap < count. */
int slm_session_trace(slm_session* se, uint64_t* out, size_t cap, size_t* n_out);

/* ---- Batched decode --------------------------------------------------------
 * No counterpart in the reference: its server runs one request at a time
 * (src/serve.rs:1-3) and Model::step advances one session.  A batch steps n
 * sessions of the same model together, one token each, reading the weights
 * once per step for all of them; each session keeps its own caches, GLA state
 * and position, so row i computes what slm_step would on session i (up to the
 * rounding of the linears, which run as one n-row product).  This serves many
 * independent sequences per GPU.
 *
 * The sessions must share the model and the loop count, appear once each,
 * and outlive the batch (slm_session_free fails while a session belongs to a
 * batch).  Global-attention caches grow per session (8192 positions, then
 * doubled, as slm_step grows them) before the step that needs the room.  Stepping a session on its own
 * between batch steps is allowed.  After batch steps a session's own logits
 * (slm_logits) are those of its last own step; read the batch's with
 * slm_batch_logits. */
int slm_batch_new(slm_session* const* sessions, size_t n, slm_batch** out);
int slm_batch_free(slm_batch* b);
int slm_batch_size(const slm_batch* b, size_t* out);
/* One step: feeds ids[i] (host, n ids) to session i.  Logits of every row are
 * kept in the batch. */
int slm_batch_step(slm_batch* b, const uint32_t* ids);
/* The last step's logits, out[i·vocab + j] (host, n·vocab floats).  Synchronises. */
int slm_batch_logits(slm_batch* b, float* out);
/* `steps` greedy decode steps of every session without leaving the device:
 * feeds first[i] to session i, then each picked id (first maximum, as pick
 * with temperature 0).  out[t·n + i] (host) receives session i's id of step t.
 * Synchronises once at the end. */
int slm_batch_decode(slm_batch* b, const uint32_t* first, size_t steps, uint32_t* out);
/* `steps` decode steps of every session with per-row sampling, pick
 * (src/sample.rs:33-93) on the device for each row, as a server that samples
 * each request with its own settings would: row i uses s[i], the history
 * recent[i] (n_recent[i] ids, host; null when n_recent is null or 0) for its
 * repeat penalty, to which its sampled ids are appended, and the xorshift64*
 * state rng_state[i] (read and advanced).  Feeds first[i] to session i, then
 * each sampled id; out[t·n + i] (host) receives row i's id of step t.
 * Candidates after top-k keep slm_sample's canonical order.  Synchronises
 * once at the end. */
int slm_batch_sample_decode(slm_batch* b, const uint32_t* first, size_t steps, const slm_sampling* s,
                            const uint32_t* const* recent, const size_t* n_recent, uint64_t* rng_state,
                            uint32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* SLM_B200_H */
