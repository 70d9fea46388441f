// Token selection on the device (reference pick, src/sample.rs:33-93, and the
// xorshift64* Rng, src/sample.rs:18-31), so a decode step hands back 4 bytes
// instead of the vocab-sized logits the reference reads back every token
// (src/main.rs:208-223).
//
// One CTA of 1024 threads:
//   1. copy the logits to a work buffer and apply the repeat penalty once per
//      distinct id of the last `window` history entries (sample.rs:34-47);
//   2. temperature ≤ 0: arg-max, first index on ties (sample.rs:48-53);
//   3. top-k and/or top-p: candidates come out in rounds of up to 2048, each
//      round the next-largest by (logit in f32 total order, then smaller id) —
//      the canonical order that stands in for select_nth_unstable's
//      unspecified one — found by an MSB-first radix select over that 64-bit
//      composite key and bitonic-sorted in shared memory.  Weights
//      e^((l - top)/T), the top-p cut on the running sum, then the cumulative
//      walk with r = u·Σw (sample.rs:54-92), sequentially in candidate order
//      on one thread as the reference does;
//   4. no top-k and no top-p: every id in id order (the reference leaves the
//      ids unsorted), with a block scan in place of the sequential walk.
#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

constexpr int ST = 1024;    // threads
constexpr int MAXC = 2048;  // candidates per round, in shared memory

__device__ __forceinline__ uint32_t total_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Larger composite = earlier in the canonical order.
__device__ __forceinline__ unsigned long long composite(float f, uint32_t id) {
  return ((unsigned long long)total_key(f) << 32) | (0xFFFFFFFFu - id);
}

__device__ __forceinline__ uint32_t comp_id(unsigned long long c) { return 0xFFFFFFFFu - (uint32_t)(c & 0xFFFFFFFFu); }

__device__ __forceinline__ float rng_next(unsigned long long* st) {
  unsigned long long x = *st;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *st = x;
  return (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / (float)(1ull << 24);
}

__device__ float block_max(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
  return warp_max(t);
}

struct Shared {
  uint32_t hist[256];
  unsigned long long cand[MAXC];
  float wts[MAXC];
  float red[32];
  float wpre[32];
  unsigned long long best, prefix, thresh;
  uint32_t remaining, count, found, nsorted;
  float s_sum, s_r;
};

// The c largest composites below `bound` (all when bound == 0): sets
// sh.thresh so that exactly c composites c satisfy thresh ≤ c < bound.
__device__ void select_round(const float* work, int V, unsigned long long bound, uint32_t c, Shared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid == 0) {
    sh.prefix = 0;
    sh.remaining = c;
    sh.found = 0;
  }
  unsigned long long mask = 0;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += ST) sh.hist[b] = 0;
    if (tid == 0) sh.count = 0;
    __syncthreads();
    if (sh.found) break;
    const unsigned long long prefix = sh.prefix;
    for (int base = 0; base < V; base += ST) {
      int i = base + tid;
      bool act = false;
      uint32_t digit = 0;
      if (i < V) {
        unsigned long long k = composite(work[i], (uint32_t)i);
        act = (!bound || k < bound) && (k & mask) == prefix;
        digit = (uint32_t)(k >> shift) & 0xFFu;
      }
      unsigned am = __ballot_sync(0xffffffffu, act);
      if (act) {
        unsigned peers = __match_any_sync(am, digit);
        if (lane == __ffs(peers) - 1) atomicAdd(&sh.hist[digit], (uint32_t)__popc(peers));
      }
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = sh.remaining, cum = 0;
      int b = 255;
      for (; b >= 0; b--) {
        if (cum + sh.hist[b] >= rem) break;
        cum += sh.hist[b];
      }
      if (b < 0) b = 0;
      sh.remaining = rem - cum;
      sh.prefix = prefix | ((unsigned long long)b << shift);
      // Every composite under the new prefix is taken: stop here.
      if (sh.hist[b] == sh.remaining || shift == 0) sh.found = 1;
    }
    mask |= 0xFFull << shift;
    __syncthreads();
  }
  if (tid == 0) sh.thresh = sh.prefix;  // low bits zero: the smallest composite under the prefix
  __syncthreads();
}

// Collects the selected composites and sorts them, descending.
__device__ void gather_sort(const float* work, int V, unsigned long long bound, uint32_t c, Shared& sh) {
  const int tid = threadIdx.x;
  if (tid == 0) sh.count = 0;
  __syncthreads();
  const unsigned long long th = sh.thresh;
  for (int i = tid; i < V; i += ST) {
    unsigned long long k = composite(work[i], (uint32_t)i);
    if (k >= th && (!bound || k < bound)) {
      uint32_t slot = atomicAdd(&sh.count, 1u);
      if (slot < (uint32_t)MAXC) sh.cand[slot] = k;
    }
  }
  __syncthreads();
  uint32_t P = 1;
  while (P < c) P <<= 1;
  for (uint32_t i = c + tid; i < P; i += ST) sh.cand[i] = 0;
  __syncthreads();
  for (uint32_t size = 2; size <= P; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = tid; i < P; i += ST) {
        uint32_t j = i ^ stride;
        if (j > i) {
          bool desc = (i & size) == 0;
          unsigned long long x = sh.cand[i], y = sh.cand[j];
          if (desc ? (x < y) : (x > y)) sh.cand[i] = y, sh.cand[j] = x;
        }
      }
      __syncthreads();
    }
  }
}

__device__ void finish(const SampleArgs& a, uint32_t chosen) {
  a.out[0] = chosen;
  if (a.hist_out) a.hist_out[a.nrecent] = chosen;
  if (a.next_id) a.next_id[0] = chosen;
}

__device__ void sample_body(const SampleArgs& a, Shared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  float* work = a.work;
  float* sw = a.work + V;                                    // sorted weights (multi-round)
  uint32_t* sid = reinterpret_cast<uint32_t*>(a.work + 2 * (size_t)V);  // their ids

  for (int i = tid; i < V; i += ST) work[i] = a.logits[i];
  __syncthreads();
  if (a.penalty != 1.0f && a.nrecent > 0) {
    long long start = a.nrecent > (long long)a.window ? a.nrecent - a.window : 0;
    for (long long j = start + tid; j < a.nrecent; j += ST) {
      uint32_t id = a.recent[j];
      if (id >= (uint32_t)V) continue;
      bool first = true;
      for (long long e = start; e < j; e++)
        if (a.recent[e] == id) {
          first = false;
          break;
        }
      if (first) {
        float l = work[id];
        work[id] = l > 0.0f ? l / a.penalty : l * a.penalty;
      }
    }
  }
  __syncthreads();

  if (a.temperature <= 0.0f) {
    unsigned long long best = 0;
    for (int i = tid; i < V; i += ST) {
      float v = work[i];
      if (v != v) continue;  // NaN never wins a `>` comparison
      unsigned long long c = composite(v, (uint32_t)i);
      if (c > best) best = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      if (other > best) best = other;
    }
    if (tid == 0) sh.best = 0;
    __syncthreads();
    if (lane == 0 && best) atomicMax(&sh.best, best);
    __syncthreads();
    if (tid == 0) {
      uint32_t chosen = sh.best ? comp_id(sh.best) : 0;
      float bv = work[chosen];
      // -0.0 and +0.0 compare equal under the reference's `>`: keep the first.
      if (bv == 0.0f)
        for (uint32_t i = 0; i < chosen; i++)
          if (work[i] == bv) {
            chosen = i;
            break;
          }
      finish(a, chosen);
    }
    return;
  }

  const bool use_k = a.top_k > 0 && a.top_k < (uint32_t)V;
  float top = -INFINITY;
  for (int i = tid; i < V; i += ST) top = fmaxf(top, work[i]);
  top = block_max(top, sh.red);
  const float invT = a.temperature;

  if (!use_k && !(a.top_p < 1.0f)) {
    // Every id, in id order.  Contiguous slices per thread keep the order.
    int per = (V + ST - 1) / ST, lo = tid * per, hi = min(V, lo + per);
    float part = 0.0f;
    for (int i = lo; i < hi; i++) part += expf((work[i] - top) / invT);
    float x = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) sh.red[warp] = x;
    __syncthreads();
    if (warp == 0) {
      float t = sh.red[lane], s = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      sh.wpre[lane] = s - t;
      if (lane == 31) sh.s_sum = s;
    }
    __syncthreads();
    float before = sh.wpre[warp] + x - part;
    if (tid == 0) {
      unsigned long long st = *a.rng;
      sh.s_r = rng_next(&st) * sh.s_sum;
      *a.rng = st;
      sh.count = 0xFFFFFFFFu;
    }
    __syncthreads();
    float r = sh.s_r - before;
    if (r > 0.0f && r <= part) {
      for (int i = lo; i < hi; i++) {
        r -= expf((work[i] - top) / invT);
        if (r <= 0.0f) {
          atomicMin(&sh.count, (uint32_t)i);
          break;
        }
      }
    }
    __syncthreads();
    if (tid == 0) finish(a, sh.count == 0xFFFFFFFFu ? (uint32_t)(V - 1) : sh.count);
    return;
  }

  // Sorted candidates, in rounds.  Without top-k every id is sorted, so the
  // top-p total is the sequential sum in sorted order, as the reference
  // computes it (sample.rs:61-73).
  const uint32_t K = use_k ? a.top_k : (uint32_t)V;
  const bool multi = K > (uint32_t)MAXC;
  if (tid == 0) sh.nsorted = 0;
  __syncthreads();
  unsigned long long bound = 0;
  while (true) {
    const uint32_t done = sh.nsorted;
    if (done >= K) break;
    const uint32_t c = min((uint32_t)MAXC, K - done);
    select_round(work, V, bound, c, sh);
    gather_sort(work, V, bound, c, sh);
    for (uint32_t i = tid; i < c; i += ST) {
      uint32_t id = comp_id(sh.cand[i]);
      float w = expf((work[id] - top) / invT);
      sh.wts[i] = w;
      if (multi) {
        sw[done + i] = w;
        sid[done + i] = id;
      }
    }
    __syncthreads();
    if (tid == 0) sh.nsorted = done + c;
    bound = sh.cand[c - 1];
    __syncthreads();
  }
  if (tid == 0) {
    auto W = [&](uint32_t i) { return multi ? sw[i] : sh.wts[i]; };
    auto ID = [&](uint32_t i) { return multi ? sid[i] : comp_id(sh.cand[i]); };
    uint32_t keep = K;
    if (a.top_p < 1.0f) {
      float total = 0.0f;
      for (uint32_t i = 0; i < K; i++) total += W(i);
      float enough = a.top_p * total, held = 0.0f;
      for (uint32_t i = 0; i < K; i++) {
        held += W(i);
        if (held >= enough) {
          keep = i + 1;
          break;
        }
      }
    }
    float total = 0.0f;
    for (uint32_t i = 0; i < keep; i++) total += W(i);
    unsigned long long st = *a.rng;
    float r = rng_next(&st) * total;
    *a.rng = st;
    uint32_t pick = keep - 1;
    for (uint32_t i = 0; i < keep; i++) {
      r -= W(i);
      if (r <= 0.0f) {
        pick = i;
        break;
      }
    }
    finish(a, ID(pick));
  }
}

}  // namespace

__global__ void __launch_bounds__(ST) k_sample(SampleArgs a) {
  __shared__ Shared sh;
  sample_body(a, sh);
}

// One CTA per row of a batched step: row i's settings, history, RNG state and
// work space come from rows[i]; its history and outputs are offset by the
// steps the batch has taken so far (*step).
__global__ void __launch_bounds__(ST) k_sample_rows(const SampleArgs* rows, const unsigned* step, uint32_t* outs,
                                                    size_t m) {
  __shared__ Shared sh;
  SampleArgs a = rows[blockIdx.x];
  const unsigned t = *step;
  a.nrecent += t;
  a.out = outs + (size_t)t * m + blockIdx.x;
  sample_body(a, sh);
}

namespace {

// One CTA per row: the largest composite key (logit, then the smaller id);
// -0.0 and +0.0 share a key, so the first of them wins, as under `>`.
__device__ __forceinline__ void argmax_take(unsigned long long& best, float v, uint32_t i) {
  if (v != v) return;  // NaN never wins a `>` comparison
  const unsigned long long c = composite(v + 0.0f, i);
  if (c > best) best = c;
}

__global__ void __launch_bounds__(1024)
    k_argmax_rows(const float* __restrict__ logits, size_t V, uint32_t* next, uint32_t* outs,
                  const unsigned* out_index, size_t m) {
  __shared__ unsigned long long best_w[32];
  const size_t row = blockIdx.x;
  const float* l = logits + row * V;
  unsigned long long best = 0;
  if (V % 4 == 0 && ((uintptr_t)l & 15) == 0) {
    const float4* l4 = reinterpret_cast<const float4*>(l);
    for (size_t i = threadIdx.x; i < V / 4; i += blockDim.x) {
      const float4 v = l4[i];
      argmax_take(best, v.x, (uint32_t)(4 * i));
      argmax_take(best, v.y, (uint32_t)(4 * i + 1));
      argmax_take(best, v.z, (uint32_t)(4 * i + 2));
      argmax_take(best, v.w, (uint32_t)(4 * i + 3));
    }
  } else {
    for (size_t i = threadIdx.x; i < V; i += blockDim.x) argmax_take(best, l[i], (uint32_t)i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    if (other > best) best = other;
  }
  if ((threadIdx.x & 31) == 0) best_w[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (best_w[w] > best_w[0]) best_w[0] = best_w[w];
    const uint32_t id = best_w[0] ? comp_id(best_w[0]) : 0u;
    next[row] = id;
    if (outs) outs[(size_t)(*out_index) * m + row] = id;
  }
}

}  // namespace

void argmax_rows(const float* logits, size_t vocab, size_t m, uint32_t* next, uint32_t* outs,
                 const unsigned* out_index, cudaStream_t st) {
  if (!m) return;
  k_argmax_rows<<<(unsigned)m, 1024, 0, st>>>(logits, vocab, next, outs, out_index, m);
  SLM_LAUNCHED("k_argmax_rows");
}

void sample(const SampleArgs& a, cudaStream_t st) {
  k_sample<<<1, ST, 0, st>>>(a);
  SLM_LAUNCHED("k_sample");
}

void sample_rows(const SampleArgs* rows, size_t m, const unsigned* step, uint32_t* outs, cudaStream_t st) {
  if (!m) return;
  k_sample_rows<<<(unsigned)m, ST, 0, st>>>(rows, step, outs, m);
  SLM_LAUNCHED("k_sample_rows");
}

}  // namespace slm
