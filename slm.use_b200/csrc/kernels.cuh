// Host-side launchers of the sm_100a kernels (one .cu file per family).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace slm {

// y[i][r] = epi(W[r]·x[i]) for i < m; see common.cuh:Epi.
struct LinearArgs {
  const float* w = nullptr;
  int rows = 0, cols = 0;
  const float* x = nullptr;
  int ldx = 0, m = 0;
  float* y = nullptr;
  int ldy = 0;
  const float* res = nullptr;  // EPI_ADD
  int ldres = 0;
  int epi = 0;
  // Workspace for the tensor-core paths (see tc_linear_workspace); may be null.
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // The weights split into bf16 parts for the bf16x3 GEMM (gemm_bf16x3.cu), or null.
  const void* wplanes = nullptr;
  // x already split the same way (written by b3_rms_split), or null.
  const void* xplanes = nullptr;
  // Per-row-block arrival counters for the split GEMV (m ≤ 8), zero between
  // launches (the last CTA of a block resets its own), or null: no split.
  unsigned* cnt = nullptr;
};
// Workspace bytes of the m ≤ 8 GEMV's K slices for `a` (0: K is not split).
size_t gemv_workspace(const LinearArgs& a);
constexpr int kGemvCounters = 1 << 14;  // counters a context keeps for it
void linear(const LinearArgs& a, cudaStream_t st);
// SIMT path for 8 < m ≤ 64 tokens (skinny.cu): STORE/ADD epilogues, cols % 32
// == 0; needs skinny_workspace(a) bytes of a.ws (0 when K is not split).
void skinny_prepare();
bool skinny_ok(const LinearArgs& a);
size_t skinny_workspace(const LinearArgs& a);
void skinny_linear(const LinearArgs& a, void* ws, cudaStream_t st);
// bf16x3 tensor-core path for m > 64 with split weights (gemm_bf16x3.cu).
size_t b3_planes_bytes(size_t rows, size_t cols);
void b3_split_weights(const float* w, size_t rows, size_t cols, void* planes, cudaStream_t st);
bool b3_linear_ok(const LinearArgs& a);
size_t b3_linear_workspace(const LinearArgs& a);
void b3_linear(const LinearArgs& a, void* ws, cudaStream_t st);
// ew_rms without a base, also writing x's bf16x3 planes ([groups][6·size] bf16).
void b3_rms_split(float* y, void* planes, const float* x, const float* w, size_t groups, size_t size, float eps,
                  cudaStream_t st);
// Tensor-core (sm100 FastFP32) path for m > 8, gemm_tc.cu.
bool tc_linear_ok(const LinearArgs& a);
size_t tc_linear_workspace(const LinearArgs& a);
void tc_linear(const LinearArgs& a, void* workspace, cudaStream_t st);
void linear_prepare();

// Attention geometry (reference Attn, src/ops.rs:31-46).  reach 0 = unbounded.
struct AttnGeom {
  int m;
  long long reach, gap, cap;
  int heads, key_heads, dh;
  float scale;
  long long pos0 = 0;  // position of the first query when no device position pointer is given
  int* err = nullptr;  // device error word (bit 32: a bounded wait of the tensor-core pass expired)
};
// Per-row sequences of a batched decode step (device arrays of g.m entries).
struct AttnRows {
  float* const* k = nullptr;
  float* const* v = nullptr;
  long long* const* pos = nullptr;
  const long long* cap = nullptr;  // per-row capacities (global caches of different sizes), or null: g.cap
};
int attn_splits(const AttnGeom& g, long long max_span);
// Prefill slice pass on the tensor cores (head size 64, m > 8): on unless
// SLM_ATTN_TC=0 (read once); attn_splits and attention() follow it.
bool attention_tc_on();
void attention_tc(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g,
                  const long long* pos_ptr, int nsplit, float* part, cudaStream_t st);
size_t attn_part_floats(const AttnGeom& g, int nsplit);
// y[i][h·dh + e]; part holds attn_part_floats(g, nsplit) floats.  With cnt
// (heads·m counters, zero on entry and left zero) decode-sized calls merge
// their slices in the same launch: the last slice of each (query, head) does.
void attention(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g, const long long* pos_ptr,
               int nsplit, float* part, float* y, int ldy, cudaStream_t st, unsigned* cnt = nullptr);

struct GlaArgs {
  float* S;
  const float *q, *k, *v, *g, *dec, *bias, *hnw;
  int ldq, ldk, ldv, ldg, lddec;
  float eps;
  int m, heads, dh;
  float* out;
  int ldo;
  int fuse;  // 1: out = silu(g)·head_norm(y); 0: out = y (the bare Ops::gla)
};
void gla(const GlaArgs& a, cudaStream_t st);
// One token for each of a.m independent sequences: row i's state is S_rows[i]
// (a.S unused), its q/k/v/g/dec/out rows at i·ld.
void gla_rows(const GlaArgs& a, float* const* S_rows, cudaStream_t st);
// Attention of g.m single-token queries, each over its own cache and position.
void attention_rows(const float* q, int ldq, const AttnRows& rows, const AttnGeom& g, int nsplit, float* part,
                    float* y, int ldy, cudaStream_t st, unsigned* cnt = nullptr);

struct SampleArgs {
  const float* logits;
  float* work;  // 3·vocab words: logits after the penalty, sorted weights, sorted ids
  int vocab;
  float temperature, top_p, penalty;
  uint32_t top_k, window;
  const uint32_t* recent;  // device history
  long long nrecent;
  unsigned long long* rng;  // device xorshift64* state
  uint32_t* out;            // chosen id
  uint32_t* hist_out;       // optional: history array, written at [nrecent]
  uint32_t* next_id;        // optional: the next step's input id
  int* err;
};
void sample(const SampleArgs& a, cudaStream_t st);
// Batched: row i samples with rows[i] (a device array), its history count
// advanced by *step, its id written to outs[*step · m + i] (and next_id, hist_out).
void sample_rows(const SampleArgs* rows, size_t m, const unsigned* step, uint32_t* outs, cudaStream_t st);

// elementwise.cu
void ew_gather(float* y, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab, int* err,
               cudaStream_t st);
void ew_embed(float* e0, float* x, const float* w, const uint32_t* ids, size_t m, size_t d, size_t vocab, int* err,
              cudaStream_t st);
void ew_copy(float* y, const float* x, size_t n, cudaStream_t st);
void ew_shift(float* y, const float* first, const float* x, size_t m, size_t d, cudaStream_t st);
void ew_columns(float* y, const float* x, size_t m, size_t stride, size_t off, size_t len, cudaStream_t st);
void ew_add(float* y, const float* a, const float* b, size_t n, cudaStream_t st);
void ew_add_row(float* y, const float* x, const float* row, size_t m, size_t d, cudaStream_t st);
void ew_scale_rows(float* y, const float* x, const float* f, size_t m, size_t d, cudaStream_t st);
void ew_mix(float* y, const float* a, const float* b, size_t n, float t, cudaStream_t st);
void ew_transpose(float* dst, const float* src, size_t rows, size_t cols, cudaStream_t st);
// dst[i] = src[i] rounded to bf16 (nearest, ties to even).
void ew_to_bf16(void* dst, const float* src, size_t n, cudaStream_t st);
void ew_head_blocks(float* dst, const float* src, size_t rows, size_t heads, size_t dh, cudaStream_t st);
void ew_silu_mul(float* y, const float* g, const float* u, size_t n, cudaStream_t st);
void ew_loop_in(float* x, const float* s, const float* e, const float* row, size_t m, size_t d, cudaStream_t st);
void ew_rms(float* y, const float* x, const float* w, size_t groups, size_t size, float eps, const float* base,
            cudaStream_t st);
void ew_l2norm(float* y, size_t ldy, const float* x, size_t ldx, size_t rows, size_t heads, size_t dh,
               cudaStream_t st);
void ew_rope_table(float* c, float* s, const float* inv, long long pos, size_t m, size_t half, cudaStream_t st);
void ew_rope(float* y, const float* x, const float* c, const float* s, size_t m, size_t heads, size_t dh,
             cudaStream_t st);
void ew_store(float* cache, const float* src, size_t ldsrc, const long long* pos_ptr, long long pos, size_t m,
              size_t cap, size_t heads, size_t dh, cudaStream_t st);
void ew_rope_store(const float* mix, size_t ldmix, const float* inv, const long long* pos_ptr, size_t m,
                   size_t heads, size_t dh, size_t cap, float* qout, float* kc, float* vc, cudaStream_t st);
void ew_g_post(float* q, size_t d, size_t m, const long long* pos_ptr, float inv_log, int logn, const float* keys,
               size_t ldk, const float* vals, size_t ldv, size_t kd, size_t cap, size_t dh, float* kc, float* vc,
               cudaStream_t st);
void ew_silu_pair(float* mid, const float* up, size_t m, size_t F, cudaStream_t st);
void ew_advance_pos(long long* pos, long long m, cudaStream_t st);
// kc[h][*pos_ptr + off] = src[h·dh …] (h < kh), skipped past the capacity.
void ew_store_next(float* kc, const float* src, const long long* pos_ptr, long long off, size_t kh, size_t dh,
                   size_t cap, cudaStream_t st);
// Batched decode of m independent sequences (one token each; arrays of m).
void ew_rope_store_rows(const float* mix, size_t ldmix, const float* inv, long long* const* posr, size_t m,
                        size_t heads, size_t dh, size_t cap, float* qout, float* const* kr, float* const* vr,
                        cudaStream_t st);
// Batched global layers (row i: its session's position *posr[i], caches kr[i] /
// vr[i] of capr[i] slots per head, previous input rows src/dst[i]).
void ew_gather_rows(float* dst, float* const* src, size_t m, size_t d, cudaStream_t st);
void ew_scatter_rows(float* const* dst, const float* src, size_t m, size_t d, cudaStream_t st);
void ew_g_post_rows(float* q, size_t d, size_t m, long long* const* posr, float inv_log, int logn, const float* keys,
                    size_t ldk, const float* vals, size_t ldv, size_t kd, size_t dh, float* const* kr,
                    float* const* vr, const long long* capr, cudaStream_t st);
void ew_store_next_rows(float* const* kr, const float* src, long long* const* posr, long long off, size_t m, size_t kh,
                        size_t dh, const long long* capr, cudaStream_t st);
// *posr[i] += 1 for every row; *counter += 1 when counter is set.
void ew_advance_rows(long long* const* posr, size_t m, unsigned* counter, cudaStream_t st);
// Greedy pick per row of logits [m][vocab] (first maximum, NaN never wins):
// next[i] = id; outs[(*out_index)·m + i] = id when outs is set.
void argmax_rows(const float* logits, size_t vocab, size_t m, uint32_t* next, uint32_t* outs,
                 const unsigned* out_index, cudaStream_t st);

}  // namespace slm
