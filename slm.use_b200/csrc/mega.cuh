// Plan of the persistent decode kernel (decode_mega.cu): the m = 1 token step
// as a list of phases.  Each CTA runs them in order and waits only for the
// values it reads (counted fixed-point sums and tagged words); phases that read
// plain data other CTAs wrote in the step start after a grid barrier.  Built
// once per session on the host (model.cpp) and read by every CTA.
#pragma once

#include <stdint.h>

namespace slm {
namespace mega {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kStages = 4;
constexpr int kStageBytes = 48 * 1024;
constexpr int kMaxCols = 3072;       // widest GEMV input held on chip
constexpr int kMaxD = 1024;          // widest normalised (d_model) input
constexpr int kMaxItemOut = 256;     // logical outputs per GEMV item
constexpr int kDH = 64;              // head size of the kernel
constexpr int kAttnTile = 96;        // cache positions per attention tile (K + V = one stage)
constexpr int kMaxSplits = 16;       // attention splits per head
#ifndef SLM_LOOKAHEAD
#define SLM_LOOKAHEAD 0
#endif
constexpr int kLookahead = SLM_LOOKAHEAD;  // tiles prefetched into L2 ahead of the ring

enum PhaseKind : int { PH_GEMV = 0, PH_ATTN = 1, PH_GLA = 2 };

// How a GEMV phase forms its input vector.
enum InMode : int {
  IN_PLAIN = 0,      // v = a
  IN_RMS = 1,        // v = rms(a)·w
  IN_EMBED_RMS = 2,  // x = embed[ids[0]] (written to a and b), v = rms(x)·w
  IN_LOOP_RMS = 3,   // x = (a + b) + c, written to xout; v = rms(x)·w
  IN_ATTN = 4,       // v = the attention output, merged from the (head, split) partials in a
  IN_RMS_E = 5,      // G: v = rms(a)·w (+ rms(e0)·c when c is set); v written to xout (the next shift input)
};

// What a GEMV phase does with its dot products.
enum OutMode : int {
  OUT_STORE = 0,   // y[r] = acc
  OUT_ADD = 1,     // y[r] += acc (the residual)
  OUT_SILU = 2,    // pairs (j, j + n): y[j] = silu(acc_j)·acc_{j+n}
  OUT_ROPE = 3,    // S qkv: rotate q, k pairs (j, j+32) of each head, write q, store k, v in the ring
  OUT_LOGITS = 4,  // y[r] = acc and a per-item arg-max partial
  OUT_G = 5,       // G: segment 0 = q rows (× the logn factor) into q; segment 1 = kv rows: keys into
                   // the cache at pos (pos + 1 with kshift: the next position's shifted key), values at pos
  OUT_MLP = 6,     // the whole MLP: items are hidden units j; h_j = silu(gate_j)·up_j, then
                   // Σ_j h_j·downᵀ[j] (+ the residual on CTA 0) added into the fixed-point sum fx_out
};

// Fixed-point residual sums of fused phases (the MLP, and the mixer with o):
// one 64-bit word per value that carries its own completion count.  Each
// contributing CTA adds kFxOne + round(part · 2^30); the top 8 bits count the
// contributions, the low 56 bits hold the signed sum.  Integer adds are exact,
// so the result does not depend on the order in which CTAs arrive, and a
// reader knows the value is final when the count reaches the phase's number of
// contributors: no barrier and no second read.  Parts are bounded by 2^16, so
// 255 of them stay below 2^54 in magnitude; a part that is non-finite or
// larger is not added (its count is) and the step reports an error.  Word d of
// a slot counts the CTAs that have issued their adds (a hint: readers of an
// MLP's slot poll it before the values, so 148 readers do not poll 768 words
// while 148 writers add into them).
constexpr float kFxScale = 1073741824.0f;         // 2^30
constexpr float kFxInv = 1.0f / 1073741824.0f;    // 2^-30
constexpr float kFxMax = 65536.0f;                // 2^16
constexpr unsigned long long kFxOne = 1ull << 56;

// Values that one CTA writes and others read within a step (q, the current
// k and v, attention partials, GLA inputs, the inject output) are 64-bit
// words: the float in the low half, a tag (step epoch << 8 | producing phase)
// in the high half.  A reader polls until the tag is the one it expects.
constexpr int kTagPhaseBits = 8;  // phases per step < 256

struct Segment {
  const float* w;   // weight rows, row-major, `cols` wide
  int rows;         // logical outputs (pairs count for SILU / ROPE)
  int per_item;     // logical outputs per item
  int items;
  float* out;       // output (OUT_STORE/ADD/SILU/LOGITS)
  unsigned long long* tout;  // OUT_STORE, OUT_G q: tagged output (instead of out)
};

struct alignas(16) Phase {
  int kind;
  int sync;     // a grid barrier before this phase: it reads plain data other CTAs wrote in this step
  int fx_cnt;   // contributions per value of fx_in when it is final
  int fx_arrive;  // CTAs that announce their adds in word d of fx_in (0: poll the values only)
  int tag_in;   // the phase whose tagged outputs this phase reads (tq, tmix, tpart, tin_b)
  // Tagged buffers: q | k | v of this position (3 × d: OUT_ROPE writes, ATTN reads; OUT_G writes q),
  // attention partials [head][split][dh + 2], GLA inputs (q|k|v|g rows, 4 × d, and decay, heads),
  // and the loop input's inject term.
  unsigned long long *tq, *tpart, *tmix, *tdec;
  unsigned long long* tkv;  // ATTN: tagged k | v of this position (d each), or null: read them from the cache
  const unsigned long long* tin_b;
  // GEMV
  int cols;
  int in_mode, out_mode;
  int res_smem;  // OUT_ADD: the residual is the x of the last normalising prologue (kept on chip)
  const float *in_a, *in_b, *in_c, *norm_w;
  float* xout;
  int nseg;
  Segment seg[2];
  // OUT_ROPE / OUT_G / ATTN / GLA
  float *q, *kc, *vc;  // q buffer and the layer's cache (ATTN, ROPE, G)
  long long cap, window;  // window 0: unbounded reach (G)
  long long gap;          // ATTN: the query at p sees positions up to p - gap
  int qg;                 // ATTN: query heads per cache head (items are cache heads × splits)
  int kshift;             // OUT_G
  float inv_log;          // OUT_G: 1/ln(logn), 0 for no logn scaling
  const float* inv_freq;
  // OUT_MLP: downᵀ ([F][d], row j = column j of down) and the slot its sums go to
  const float* wt;
  unsigned long long* fx_out;
  // Inputs: when set, the `a` input is this fixed-point slot instead of in_a
  const unsigned long long* fx_in;
  // ATTN with o (S blocks): the o matrix as per-head column blocks [heads][d][dh];
  // split s multiplies rows s·orows … of its head's block, after the head's
  // `splits` partials have arrived (per-head counters `cnt`, zeroed each step),
  // and adds them into fx_out (head 0's CTAs also add the residual in_a/fx_in).
  const float* wo;
  int orows;
  unsigned long long* cnt;
  int l2keep;  // the phase's weight tiles are read again within the step (loop blocks): keep them in L2
  // ATTN: heads × splits items; partials and per-head arrival counters
  int heads, splits;
  float* part;
  unsigned* counters;
  float* y;
  float scale;
  // GLA: state [heads][64][64], raw q|k|v|g rows in `mix`, decay in `dec`
  float* state;
  const float *mix, *dec, *bias, *hnw;
  // items of the phase (all kinds)
  int items;
};

struct Plan {
  int nphases;
  Phase* phases;       // device array
  int d, heads, vocab;
  float eps;
  const float* embed;
  const float* inv_freq;  // rope frequencies (dh/2), staged in shared memory at entry
  const uint32_t* ids;  // ids[0]: the token of this step
  float *e0, *x0;       // embedding outputs
  long long* pos;       // position of this step (advanced at the end)
  unsigned* arg_count;  // arrival counter of the logits arg-max
  unsigned long long* arg_part;  // per-item arg-max partials
  int greedy;           // 1: write the arg-max to next_id / out
  uint32_t* next_id;
  uint32_t* out_ids;    // out_ids[*out_index] = id, then ++*out_index
  unsigned* out_index;
  uint32_t* argmax;     // every step: the arg-max of its logits (first maximum; NaN never wins)
  uint32_t* argmax2;    // the same id, beside the context's error word (one copy reads both)
  uint32_t* hist;       // optional history array (same index as out + hist_base)
  unsigned long long hist_base;
  unsigned* bar;        // grid barrier: [0] arrivals (monotonic in a step), [1] CTAs done
  int* err;             // error word: 8 = a bounded wait expired, 16 = a residual part out of range
  long long spin_limit;
  // Optional timeline, per phase and CTA, eight words at (phase·grid + cta)·8:
  // globaltimer (ns) when the CTA starts the phase's work and when it reaches
  // the next barrier, then the ns it spent waiting for tiles, building the
  // input vector, on tile arithmetic and in GEMV epilogues, the GEMV tiles it
  // took, and a spare zero.
  unsigned long long* trace;
  // Test hook: when set, the first grid barrier waits for one arrival more
  // than the grid has, so its bounded wait runs out (failure-path test).
  int test_stall;
  int global;  // the plan has global-attention layers (selects the kernel built for them)
  long long host_id;  // ≥ 0: this step's token, passed with the launch; < 0: read ids[0]
  // Fixed-point slots of fused phases and per-head counters: two sets of
  // fx_words words, fx_stride apart; a step uses set (epoch & 1) and zeroes
  // the other one for the next step.  Phase descriptors point into set 0.
  unsigned long long* fx;
  int fx_words;
  long long fx_stride;
  unsigned* epoch;  // step counter of the session (tags, fixed-point set parity)
  int all_sync;     // a grid barrier before every phase (the unfused variants)
  int mlp_cta;    // 1: fused MLP tiles split by rows with a CTA barrier per tile (always for d > 768)
  // L2 priority of the bulk copies: 0 none; 1 weights of phases marked l2keep
  // evict_last, every other tile evict_first; 2 the same with the others normal.
  int l2mode;
  // Bytes of one weight value in the GEMV, MLP and o tiles: 4 (f32) or 2
  // (bf16 copies of the same matrices; caches and arithmetic stay f32).
  int wbytes;
  // Most tiles a producer keeps in flight (issued, not landed); 1 … kStages.
  int inflight;
  // Steps of one launch (greedy decode): step s + 1 takes the arg-max of step
  // s, passed between CTAs as a tagged word; 1 for a single step.
  int nsteps;
  unsigned long long* next_tagged;
  // The phase after which every CTA has finished the previous step, so the
  // fixed-point set the next step uses may be zeroed (see run()).
  int zero_phase;
  // Optional mailbox in mapped pinned host memory (single steps launched by
  // slm_step): once every CTA has finished the step, the last one writes
  // host_mbox[1] = arg-max | error word << 32, then host_mbox[0] = host_seq
  // after a system-scope fence; the host polls word 0 instead of copying the
  // arg-max back and synchronising the stream.
  unsigned long long* host_mbox;
  unsigned long long host_seq;
  // Optional gate (an armed launch, queued before the host knows the step's
  // token): CTA 0 polls host_gate (mapped pinned memory) for a word
  // (gate_seq << 32 | token), bounded by kArmNs; the token 0xFFFFFFFF, or no
  // word in time, cancels the step (the kernel then writes host_mbox[2] =
  // gate_seq and ends without touching the session's state).  The decision
  // reaches the other CTAs through next_tagged, tagged with gate_seq (bit 31
  // clear, so it never matches a step's arg-max tag).
  const volatile unsigned long long* host_gate;
  unsigned long long gate_seq;
};
constexpr unsigned long long kArmNs = 20000000ull;  // 20 ms without a token: the armed step cancels itself

}  // namespace mega
}  // namespace slm
