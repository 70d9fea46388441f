// Token selection on the device (reference pick, src/sample.rs:33-93, and the
// xorshift64* Rng, src/sample.rs:18-31), so a decode step hands back 4 bytes
// instead of the vocab-sized logits the reference reads back every token
// (src/main.rs:208-223).
//
// One CTA of 1024 threads:
//   1. copy the logits to a work buffer and apply the repeat penalty once per
//      distinct id of the last `window` history entries;
//   2. temperature ≤ 0: arg-max, first index on ties (sample.rs:48-53);
//   3. otherwise top-k by an MSB-first radix select over the total order of
//      f32 (Rust's total_cmp), ties at the threshold broken by smaller id; the
//      k candidates are bitonic-sorted (logit descending, then id ascending —
//      the canonical order that stands in for select_nth_unstable's
//      unspecified one); weights e^((l - top)/T), top-p cut on the running
//      sum, then the cumulative walk with r = u·Σw (sample.rs:61-92).
// Sequential sums and the walk run in candidate order on one thread, as the
// reference does, whenever the candidate set is a sorted list (≤ 2048).
#include "common.cuh"
#include "kernels.cuh"

namespace slm {

namespace {

constexpr int ST = 1024;      // threads
constexpr int MAXC = 2048;    // candidates kept in shared memory

__device__ __forceinline__ uint32_t total_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

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

// Exclusive block scan of one uint per thread (ST threads).
__device__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_tot, uint32_t* total) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  if (w == 0) {
    uint32_t t = warp_tot[lane];
    uint32_t s = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_tot[lane] = s - t;
    if (lane == 31) *total = s;
  }
  __syncthreads();
  return warp_tot[w] + x - v;
}

__global__ void __launch_bounds__(ST) k_sample(SampleArgs a) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t s_total, s_count, s_prefix, s_remaining;
  __shared__ unsigned long long cand[MAXC];
  __shared__ float wts[MAXC];
  __shared__ float redf[32];
  __shared__ unsigned long long s_best;
  const int tid = threadIdx.x;
  const int V = a.vocab;
  float* work = a.work;

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

  uint32_t chosen = 0;
  if (a.temperature <= 0.0f) {
    // Arg-max; (key, ~index) packs "larger value, then smaller index".
    unsigned long long best = 0;
    bool have = false;
    for (int i = tid; i < V; i += ST) {
      float v = work[i];
      if (v != v) continue;  // NaN never wins a `>` comparison
      unsigned long long c = ((unsigned long long)total_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)i);
      if (!have || c > best) best = c, have = true;
    }
    if (tid == 0) s_best = 0;
    __syncthreads();
    if (have) atomicMax(&s_best, best);
    __syncthreads();
    chosen = s_best ? 0xFFFFFFFFu - (uint32_t)(s_best & 0xFFFFFFFFu) : 0;
    if (tid == 0) {
      // -0.0 and +0.0 compare equal in the reference's `>`: keep the first.
      float bv = work[chosen];
      if (bv == 0.0f)
        for (uint32_t i = 0; i < chosen; i++)
          if (work[i] == bv) {
            chosen = i;
            break;
          }
      a.out[0] = chosen;
      if (a.hist_out) a.hist_out[a.nrecent] = chosen;
      if (a.next_id) a.next_id[0] = chosen;
    }
    return;
  }

  const bool use_k = a.top_k > 0 && a.top_k < (uint32_t)V;
  const bool sorted = use_k || a.top_p < 1.0f;
  if (!sorted) {
    // Every id, in id order: weights, a block sum, then the walk.
    float top = -INFINITY;
    for (int i = tid; i < V; i += ST) top = fmaxf(top, work[i]);
    top = block_max(top, redf);
    // Contiguous slices per thread keep the walk in id order.
    int per = (V + ST - 1) / ST, lo = tid * per, hi = min(V, lo + per);
    float part = 0.0f;
    for (int i = lo; i < hi; i++) part += expf((work[i] - top) / a.temperature);
    __syncthreads();
    // Exclusive scan of the float partials (via warp shuffles + shared).
    float x = part;
    int lane = tid & 31, w = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) redf[w] = x;
    __syncthreads();
    __shared__ float wpre[32];
    __shared__ float s_sum, s_r;
    if (w == 0) {
      float t = redf[lane], s = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      wpre[lane] = s - t;
      if (lane == 31) s_sum = s;
    }
    __syncthreads();
    float before = wpre[w] + x - part;
    if (tid == 0) {
      unsigned long long st = *a.rng;
      s_r = rng_next(&st) * s_sum;
      *a.rng = st;
      s_count = 0xFFFFFFFFu;
    }
    __syncthreads();
    float r = s_r - before;
    if (r > 0.0f && r <= part) {
      for (int i = lo; i < hi; i++) {
        r -= expf((work[i] - top) / a.temperature);
        if (r <= 0.0f) {
          atomicMin(&s_count, (uint32_t)i);
          break;
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      chosen = s_count == 0xFFFFFFFFu ? (uint32_t)(V - 1) : s_count;
      a.out[0] = chosen;
      if (a.hist_out) a.hist_out[a.nrecent] = chosen;
      if (a.next_id) a.next_id[0] = chosen;
    }
    return;
  }

  // Candidate set: the K largest by total order (K ≤ MAXC).
  const uint32_t K = use_k ? a.top_k : (uint32_t)min(V, MAXC);
  if (K > (uint32_t)MAXC) {
    if (tid == 0 && a.err) atomicOr(a.err, 2);
    return;
  }
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = K;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += ST) hist[b] = 0;
    __syncthreads();
    uint32_t prefix = s_prefix;
    for (int i = tid; i < V; i += ST) {
      uint32_t k = total_key(work[i]);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = s_remaining, cum = 0;
      int b = 255;
      for (; b >= 0; b--) {
        if (cum + hist[b] >= rem) break;
        cum += hist[b];
      }
      if (b < 0) b = 0;
      s_remaining = rem - cum;
      s_prefix = prefix | ((uint32_t)b << shift);
    }
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix, need_eq = s_remaining;
  if (tid == 0) s_count = 0;
  __syncthreads();
  // Above the threshold: any order (sorted below).
  for (int i = tid; i < V; i += ST) {
    uint32_t k = total_key(work[i]);
    if (k > T) {
      uint32_t slot = atomicAdd(&s_count, 1u);
      if (slot < (uint32_t)MAXC) cand[slot] = ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)i);
    }
  }
  __syncthreads();
  const uint32_t n_gt = s_count;
  // At the threshold: the need_eq smallest ids.
  {
    int per = (V + ST - 1) / ST, lo = tid * per, hi = min(V, lo + per);
    uint32_t c = 0;
    for (int i = lo; i < hi; i++) c += total_key(work[i]) == T;
    uint32_t rank = block_excl_scan(c, warp_tot, &s_total);
    for (int i = lo; i < hi && rank < need_eq; i++) {
      if (total_key(work[i]) == T) {
        uint32_t slot = n_gt + rank;
        if (slot < (uint32_t)MAXC) cand[slot] = ((unsigned long long)T << 32) | (0xFFFFFFFFu - (uint32_t)i);
        rank++;
      }
    }
  }
  __syncthreads();
  // Bitonic sort, descending, over the next power of two.
  uint32_t P = 1;
  while (P < K) P <<= 1;
  for (uint32_t i = K + tid; i < P; i += ST) cand[i] = 0;
  __syncthreads();
  for (uint32_t size = 2; size <= P; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = tid; i < P; i += ST) {
        uint32_t j = i ^ stride;
        if (j > i) {
          bool desc = (i & size) == 0;
          unsigned long long x = cand[i], y = cand[j];
          if (desc ? (x < y) : (x > y)) cand[i] = y, cand[j] = x;
        }
      }
      __syncthreads();
    }
  }
  // Weights in candidate order.
  const float top = work[0xFFFFFFFFu - (uint32_t)(cand[0] & 0xFFFFFFFFu)];
  for (uint32_t i = tid; i < K; i += ST) {
    uint32_t id = 0xFFFFFFFFu - (uint32_t)(cand[i] & 0xFFFFFFFFu);
    wts[i] = expf((work[id] - top) / a.temperature);
  }
  // Without top-k the top-p cut needs Σ over every id.
  float all_sum = 0.0f;
  if (!use_k) {
    float part = 0.0f;
    for (int i = tid; i < V; i += ST) part += expf((work[i] - top) / a.temperature);
    all_sum = block_sum(part, redf);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t keep = K;
    if (a.top_p < 1.0f) {
      float total = 0.0f;
      if (use_k)
        for (uint32_t i = 0; i < K; i++) total += wts[i];
      else
        total = all_sum;
      float enough = a.top_p * total, held = 0.0f;
      keep = 0;
      for (uint32_t i = 0; i < K; i++) {
        held += wts[i];
        if (held >= enough) {
          keep = i + 1;
          break;
        }
      }
      if (keep == 0) {
        if (use_k) {
          keep = K;
        } else {
          if (a.err) atomicOr(a.err, 4);  // top-p set larger than the candidates held on chip
          keep = K;
        }
      }
    }
    float total = 0.0f;
    for (uint32_t i = 0; i < keep; i++) total += wts[i];
    unsigned long long st = *a.rng;
    float r = rng_next(&st) * total;
    *a.rng = st;
    uint32_t pick = keep - 1;
    for (uint32_t i = 0; i < keep; i++) {
      r -= wts[i];
      if (r <= 0.0f) {
        pick = i;
        break;
      }
    }
    chosen = 0xFFFFFFFFu - (uint32_t)(cand[pick] & 0xFFFFFFFFu);
    a.out[0] = chosen;
    if (a.hist_out) a.hist_out[a.nrecent] = chosen;
    if (a.next_id) a.next_id[0] = chosen;
  }
}

}  // namespace

void sample(const SampleArgs& a, cudaStream_t st) {
  k_sample<<<1, ST, 0, st>>>(a);
  SLM_LAUNCHED("k_sample");
}

}  // namespace slm
