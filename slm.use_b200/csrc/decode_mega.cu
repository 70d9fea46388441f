// The m = 1 token step as one persistent, warp-specialised kernel.
//
// Everything a decode step reads from HBM — the weights, the old entries of
// the sliding-window rings and the recurrent GLA state — is fixed for the
// whole step; only small activation vectors (x, q, y, mid: a few KB) flow
// from phase to phase.  So one producer thread per CTA walks the step's
// static tiles in order:
//   * a ring cursor streams them into a 4-stage shared-memory ring with
//     cp.async.bulk (TMA bulk copies, mbarrier completion), never waiting for
//     the grid barriers that separate phases;
//   * a lookahead cursor, kLookahead tiles further on, issues
//     cp.async.bulk.prefetch.L2 for the same tiles, so HBM keeps streaming
//     while the ring is full and the consumers sit at a barrier.
// Eight consumer warps wait at each barrier, rebuild the phase's input vector
// on chip (RMSNorm, loop input, embedding) and consume the tiles.
//
// Phases follow the reference's block (src/model.rs:400-560) and advance
// (src/model.rs:563-640) for one token:
//   S block: [norm1 + qkv + rope + ring store] [window attention, split over
//            positions, merged by the last arriving CTA of each head]
//            [o + residual] [norm2 + up + silu] [down + residual]
//   L block: [norm1 + qkvg + decay] [GLA: l2norm, state update, q·S,
//            head_norm, silu gate] [o + residual] [norm2 + up] [down]
//   glue:    embedding in the first prologue, inject after the prelude, the
//            loop input (s + e + loop_embed[r]) in the first core prologue,
//            norm_f + tied logits + greedy arg-max at the end.
// Every wait (mbarrier, grid barrier) is bounded: past ~2 s the kernel sets
// bit 8 of the error word and returns.
#include "common.cuh"
#include "kernels.cuh"
#include "mega.cuh"

namespace slm {
namespace mega {

namespace {

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Explicit shared-window load (the ring is reached through pointers the
// compiler cannot prove to be shared, which would make it emit generic loads).
__device__ __forceinline__ float4 lds4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds1(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
// 16 bytes of weights in shared memory as floats: 4 f32, or 8 bf16 (a bf16
// value is the top half of an f32, so widening is exact).
template <int WB>
__device__ __forceinline__ void widen(const float4 x, float (&v)[16 / WB]) {
  if constexpr (WB == 4) {
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  } else {
    const uint32_t u[4] = {__float_as_uint(x.x), __float_as_uint(x.y), __float_as_uint(x.z), __float_as_uint(x.w)};
#pragma unroll
    for (int i = 0; i < 4; i++) v[2 * i] = __uint_as_float(u[i] << 16), v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}
template <int WB>
__device__ __forceinline__ void wchunk(uint32_t a, float (&v)[16 / WB]) {
  widen<WB>(lds4(a), v);
}
template <int E>
__device__ __forceinline__ float dotn(const float (&w)[E], const float (&x)[E], float acc) {
#pragma unroll
  for (int e = 0; e < E; e++) acc = fmaf(w[e], x[e], acc);
  return acc;
}

__device__ __forceinline__ void st_release_cta_shared(unsigned* p, unsigned v) {
  asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(saddr(p)), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta_shared(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr(p)) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_u64(long long* p, long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *(const volatile int*)p; }
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Barrier of the 256 consumer threads that also ANDs a flag over them, so a
// failed wait in any thread is seen by all of them at the same point.
__device__ __forceinline__ int consumers_and(int v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.s32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(v)
      : "memory");
  return r;
}

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait


// Bounded wait on an mbarrier phase; false (and the error bit) on expiry or
// when another CTA has already failed.
__device__ bool wait_mbar(uint64_t* b, unsigned parity, int* err) {
  if (mbar_try_wait(b, parity)) return true;
  unsigned long long t0 = now_ns();
  for (unsigned it = 1;; it++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63) == 0) {
      if (ld_volatile(err) & 8) return false;
      if (now_ns() - t0 > kWaitNs) {
        atomicOr(err, 8);
        return false;
      }
    }
  }
}

// Bounded wait for a copy this CTA issued itself.  Such a copy completes
// whatever other CTAs did, so the error word is not consulted: only the time
// limit ends the wait (and then sets the error bit).  The producer's drain
// uses it so that the CTA never exits with bulk copies into its shared memory
// still in flight.
__device__ bool wait_mbar_own(uint64_t* b, unsigned parity, int* err) {
  if (mbar_try_wait(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (unsigned it = 1;; it++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63) == 0 && now_ns() - t0 > kWaitNs) {
      atomicOr(err, 8);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t total_key(float f) {
  uint32_t u = __float_as_uint(f + 0.0f);  // -0 → +0: equal values compare equal
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ ulonglong2 ld_relaxed_u64x2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
// A word the host writes (mapped pinned memory): system scope.
__device__ __forceinline__ unsigned long long ld_sys_u64(const volatile unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_fx(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// A bounded spin: again() is false once the wait has run past kWaitNs (the
// error bit is set here) or another CTA has given up (error bit 8 seen).
struct Spin {
  unsigned it = 0;
  unsigned long long t0 = 0;
  __device__ __forceinline__ bool again(int* err) {
    if ((++it & 15) != 0) return true;
    if (ld_volatile(err) & 8) return false;
    const unsigned long long t = now_ns();
    if (!t0) {
      t0 = t;
    } else if (t - t0 > kWaitNs) {
      atomicOr(err, 8);
      return false;
    }
    return true;
  }
};

// Fixed-point words: contributions so far, and the value they sum to.
__device__ __forceinline__ unsigned fx_count(unsigned long long w) {
  return (unsigned)((w + (1ull << 55)) >> 56);
}
__device__ __forceinline__ float fx_value(unsigned long long w) {
  const long long v = (long long)(w - ((unsigned long long)fx_count(w) << 56));
  return __ll2float_rn(v) * kFxInv;
}
// The word one CTA adds for a part: one count and the part in units of 2^-30
// (a part out of range adds only the count, and *bad is set).
__device__ __forceinline__ unsigned long long fx_word(float v, bool* bad) {
  if (!(fabsf(v) < kFxMax)) {  // NaN included
    *bad = true;
    return kFxOne;
  }
  return kFxOne + (unsigned long long)__float2ll_rn(v * kFxScale);
}

// Four values i4·4 … of a fixed-point slot once all `cnt` parts of each have
// landed (one load round per poll).  False when the wait gave up.
__device__ __forceinline__ bool fx_poll4(const unsigned long long* fx, int i4, unsigned cnt, int* err, float4* out) {
  const unsigned long long* f = fx + 4 * i4;
  Spin sp;
  do {
    const ulonglong2 a = ld_relaxed_u64x2(f), b = ld_relaxed_u64x2(f + 2);
    if (fx_count(a.x) == cnt && fx_count(a.y) == cnt && fx_count(b.x) == cnt && fx_count(b.y) == cnt) {
      *out = make_float4(fx_value(a.x), fx_value(a.y), fx_value(b.x), fx_value(b.y));
      return true;
    }
  } while (sp.again(err));
  *out = make_float4(0.f, 0.f, 0.f, 0.f);
  return false;
}

// One read of the same four values: true when every one is final.
__device__ __forceinline__ bool fx_try4(const unsigned long long* fx, int i4, unsigned cnt, float4* out) {
  const unsigned long long* f = fx + 4 * i4;
  const ulonglong2 a = ld_relaxed_u64x2(f), b = ld_relaxed_u64x2(f + 2);
  *out = make_float4(fx_value(a.x), fx_value(a.y), fx_value(b.x), fx_value(b.y));
  return fx_count(a.x) == cnt && fx_count(a.y) == cnt && fx_count(b.x) == cnt && fx_count(b.y) == cnt;
}

// Tagged words: the float in the low half, the producer's tag in the high half.
__device__ __forceinline__ unsigned long long tagged(float v, unsigned tag) {
  return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void put_tagged(unsigned long long* p, float v, unsigned tag) {
  st_relaxed_u64(p, tagged(v, tag));
}
// N tagged values p[i·stride] once each carries `tag`.  False when the wait gave up.
template <int N>
__device__ __forceinline__ bool poll_tagged(const unsigned long long* p, int stride, unsigned tag, int* err,
                                            float (&out)[N]) {
  Spin sp;
  do {
    unsigned long long w[N];
#pragma unroll
    for (int i = 0; i < N; i++) w[i] = ld_relaxed_u64(p + (size_t)i * stride);
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; i++) all &= (unsigned)(w[i] >> 32) == tag;
    if (all) {
#pragma unroll
      for (int i = 0; i < N; i++) out[i] = __uint_as_float((unsigned)w[i]);
      return true;
    }
  } while (sp.again(err));
#pragma unroll
  for (int i = 0; i < N; i++) out[i] = 0.0f;
  return false;
}
// One read of four consecutive tagged values: true when all carry `tag`.
__device__ __forceinline__ bool try_tagged4(const unsigned long long* p, unsigned tag, float4* out) {
  const ulonglong2 a = ld_relaxed_u64x2(p), b = ld_relaxed_u64x2(p + 2);
  *out = make_float4(__uint_as_float((unsigned)a.x), __uint_as_float((unsigned)a.y), __uint_as_float((unsigned)b.x),
                     __uint_as_float((unsigned)b.y));
  return (unsigned)(a.x >> 32) == tag && (unsigned)(a.y >> 32) == tag && (unsigned)(b.x >> 32) == tag &&
         (unsigned)(b.y >> 32) == tag;
}

// ---------------------------------------------------------------------------
// Tile geometry shared by the producer and the consumers
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool is_pair(const Phase& ph) {
  return ph.out_mode == OUT_SILU || ph.out_mode == OUT_ROPE || ph.out_mode == OUT_MLP;
}

// Logical outputs per tile of a GEMV phase (a fused MLP unit takes three rows:
// gate, up and downᵀ).
__device__ __forceinline__ int tile_outs(const Phase& ph, int wb) {
  int rows = kStageBytes / (ph.cols * wb);
  const int most = wb == 2 ? 32 : 16;  // two (f32) or four (bf16) rows per consumer warp
  if (rows > most) rows = most;
  if (ph.out_mode == OUT_MLP) return rows / 3;
  return is_pair(ph) ? rows / 2 : rows;
}

// First weight row of logical output o (and its partner).
__device__ __forceinline__ void out_rows(const Phase& ph, const Segment& sg, int o, int d, int* r0, int* r1) {
  if (ph.out_mode == OUT_ROPE) {
    int sec = o / (d / 2), rem = o % (d / 2), h = rem / 32, j = rem % 32;
    *r0 = sec * d + h * kDH + j;
    *r1 = *r0 + 32;
  } else if (ph.out_mode == OUT_SILU || ph.out_mode == OUT_MLP) {
    *r0 = o;
    *r1 = o + sg.rows;
  } else {
    *r0 = o;
    *r1 = -1;
  }
}

// Item i of a GEMV phase → segment and logical output range.
__device__ __forceinline__ void gemv_item(const Phase& ph, int i, int* seg, int* o0, int* o1) {
  int s = 0;
  if (ph.nseg > 1 && i >= ph.seg[0].items) {
    i -= ph.seg[0].items;
    s = 1;
  }
  const Segment& sg = ph.seg[s];
  *seg = s;
  *o0 = i * sg.per_item;
  *o1 = min(sg.rows, *o0 + sg.per_item);
}

// The step's query sees positions lo .. pos - gap (lo = 0 for an unbounded
// window).  With gap 0, split s takes a slice of the old positions lo..pos-1
// and the last split also takes `pos` itself, from the cache the projection
// phase just wrote; with gap ≥ 1 the slices cover lo..pos-gap.
template <bool GL = true>
__device__ __forceinline__ void attn_slice(const Phase& ph, long long pos, int s, long long* a, long long* b) {
  long long lo = ph.window > 0 && pos > ph.window - 1 ? pos - (ph.window - 1) : 0;
  long long hi = GL && ph.gap > 0 ? pos + 1 - ph.gap : pos;  // exclusive
  long long count = hi > lo ? hi - lo : 0;
  long long chunk = (count + ph.splits - 1) / ph.splits;
  *a = lo + (long long)s * chunk;
  *b = min(hi, *a + chunk);
  if (*b < *a) *b = *a;
}

struct Tile {
  int n;
  const void* src[4];
  unsigned bytes[4];
  unsigned off[4];
  unsigned total;
  int keep;  // weights read again within the step
  int step;  // step of the launch the tile belongs to
  int mut;   // cache or state written by earlier steps (not weights)
};

// Resumable walk over this CTA's tiles, phase by phase (the order in which
// the consumers take them).
struct Walker {
  const Plan* P;
  long long pos;
  int me, G;
  int p = 0, i = -1, seg = 0;
  long long t = 0, tend = 0;
  int extra = 0;  // ATTN with o: the o tile follows the item's K/V tiles
  int step = 0;   // step of the launch

  __device__ Walker(const Plan* pl, long long ps) : P(pl), pos(ps) {
    me = blockIdx.x;
    G = gridDim.x;
  }

  __device__ void start_item(const Phase& ph) {
    if (ph.kind == PH_GEMV) {
      int o0, o1;
      gemv_item(ph, i, &seg, &o0, &o1);
      t = o0, tend = o1;
    } else if (ph.kind == PH_ATTN) {
      attn_slice(ph, pos, i % ph.splits, &t, &tend);
    } else {
      t = 0, tend = 1;  // with o: every split of the head reads the state
    }
    extra = ph.wo ? 1 : 0;
  }

  __device__ bool next(Tile& T) {
    for (;;) {
      if (p >= P->nphases) {  // the next step of the launch, one position on
        if (step + 1 >= P->nsteps) return false;
        step++, pos++, p = 0, i = -1;
      }
      const Phase& ph = P->phases[p];
      if (i < 0) {
        i = me;
        if (i >= ph.items) {
          p++, i = -1;
          continue;
        }
        start_item(ph);
      }
      if (t < tend) {
        make(ph, T);
        return true;
      }
      if (extra) {  // rows s·orows … of head h's o block
        const int h = i / ph.splits, s = i % ph.splits;
        T.n = 1;
        T.keep = ph.l2keep;
        T.step = step, T.mut = 0;
        T.src[0] = reinterpret_cast<const char*>(ph.wo) + ((size_t)h * P->d + (size_t)s * ph.orows) * kDH * P->wbytes;
        T.bytes[0] = T.total = (unsigned)ph.orows * kDH * P->wbytes;
        T.off[0] = 0;
        extra = 0;
        return true;
      }
      i += G;
      if (i >= ph.items) {
        p++, i = -1;
        continue;
      }
      start_item(ph);
    }
  }

  __device__ void make(const Phase& ph, Tile& T) {
    T.n = 0;
    T.keep = ph.kind == PH_GEMV ? ph.l2keep : 0;  // K/V and GLA state tiles stream
    T.step = step, T.mut = ph.kind != PH_GEMV;
    if (ph.kind == PH_GEMV) {
      const Segment& sg = ph.seg[seg];
      const int Tn = tile_outs(ph, P->wbytes);
      int n = (int)min((long long)Tn, tend - t);
      int r0, r1;
      out_rows(ph, sg, (int)t, P->d, &r0, &r1);
      const unsigned rowb = (unsigned)ph.cols * P->wbytes;
      const char* wb = reinterpret_cast<const char*>(sg.w);
      T.src[0] = wb + (size_t)r0 * rowb, T.bytes[0] = n * rowb, T.off[0] = 0, T.n = 1;
      if (is_pair(ph)) T.src[1] = wb + (size_t)r1 * rowb, T.bytes[1] = n * rowb, T.off[1] = n * rowb, T.n = 2;
      if (ph.out_mode == OUT_MLP)  // [gate n][up n][downᵀ n]
        T.src[2] = reinterpret_cast<const char*>(ph.wt) + (size_t)t * rowb, T.bytes[2] = n * rowb,
        T.off[2] = 2 * n * rowb, T.n = 3;
      t += n;
    } else if (ph.kind == PH_ATTN) {
      const int h = i / ph.splits;
      const float* kb = ph.kc + (size_t)h * ph.cap * kDH;
      const float* vb = ph.vc + (size_t)h * ph.cap * kDH;
      int n = (int)min((long long)kAttnTile, tend - t);
      long long slot = t % ph.cap;
      int n1 = (int)min((long long)n, ph.cap - slot);
      const unsigned vo = kAttnTile * kDH * 4;
      T.src[0] = kb + slot * kDH, T.bytes[0] = n1 * kDH * 4, T.off[0] = 0;
      T.src[1] = vb + slot * kDH, T.bytes[1] = n1 * kDH * 4, T.off[1] = vo;
      T.n = 2;
      if (n1 < n) {
        T.src[2] = kb, T.bytes[2] = (n - n1) * kDH * 4, T.off[2] = n1 * kDH * 4;
        T.src[3] = vb, T.bytes[3] = (n - n1) * kDH * 4, T.off[3] = vo + n1 * kDH * 4;
        T.n = 4;
      }
      t += n;
    } else {
      const int h = ph.wo ? i / ph.splits : i;
      T.src[0] = ph.state + (size_t)h * kDH * kDH, T.bytes[0] = kDH * kDH * 4, T.off[0] = 0, T.n = 1;
      t += 1;
    }
    T.total = 0;
    for (int j = 0; j < T.n; j++) T.total += T.bytes[j];
  }
};

struct Smem {
  uint64_t full[kStages], empty[kStages];
  Phase ph[2];  // descriptors of this phase and the next, staged with cp.async
  float xin[kMaxCols];
  float xraw[kMaxD];
  float acc[2][2][kMaxItemOut];  // [column half][pair half][output]
  float red[32];
  float wsm[kConsumerWarps][kDH + 2];
  float cmb[kMaxSplits][kDH + 2];
  float vec[4][kDH];
  float yp[4][kDH];
  float inv_freq[kDH / 2];
  unsigned long long best;
  int flag;
  uint32_t cur_id;   // the token of the running step (steps after the first: the previous arg-max)
  unsigned step_ok;  // steps whose start the consumers have seen (the producer may read caches after it)
  unsigned gate;     // armed launch: 0 undecided, 1 go, 2 cancelled
};

// ---------------------------------------------------------------------------
// Producer: one thread, two cursors over the same tile sequence.
// ---------------------------------------------------------------------------
__device__ void producer(const Plan& P, Smem& sm, char* ring, long long pos) {
  // The lookahead cursor starts where the ring's first fill ends and is only
  // advanced after a ring copy has been issued, so prefetches never queue
  // ahead of data the consumers are about to wait for.
  Walker ring_w(&P, pos), ahead(&P, pos);
  Tile T, A;
  uint64_t pol_keep = 0, pol_other = 0;
  if (P.l2mode) {
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
    if (P.l2mode == 1)
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_other));
    else
      asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol_other));
  }
  for (int j = 0; j < kStages; j++)
    if (!ahead.next(A)) break;
  unsigned k = 0;
  const unsigned inflight = P.inflight >= 1 && P.inflight < kStages ? (unsigned)P.inflight : (unsigned)kStages;
  int ready = 0;  // the last step whose caches and states this thread may read
  bool gated = P.host_gate == nullptr;
  while (ring_w.next(T)) {
    if (!gated && k == (unsigned)kStages) {
      // Armed launch: the first ring of tiles is in flight; issue more only
      // once the consumers know the step goes ahead (drain and end if not).
      Spin sp;
      unsigned g = 0;
      while ((g = ld_acquire_cta_shared(&sm.gate)) == 0)
        if (!sp.again(P.err)) break;
      if (g != 1) break;
      gated = true;
    }
    if (T.mut && T.step > ready) {
      // K/V and GLA state of step s were written by step s - 1: wait until
      // the consumers have seen that step end (their acquire of its arg-max),
      // then order those writes before this thread's bulk copies.
      Spin sp;
      bool good = true;
      while ((int)ld_acquire_cta_shared(&sm.step_ok) < T.step)
        if (!sp.again(P.err)) {
          good = false;
          break;
        }
      if (!good) break;
      ready = T.step;
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    const int s = k % kStages;
    if (k >= (unsigned)kStages && !wait_mbar(&sm.empty[s], ((k / kStages) - 1) & 1, P.err)) break;
    // Tile k - inflight must have landed first: fewer bytes queued in the
    // memory system keep its round trips (the CTAs' exchanges) short.
    if (inflight < (unsigned)kStages && k >= inflight) {
      const unsigned j = k - inflight;
      if (!wait_mbar(&sm.full[j % kStages], (j / kStages) & 1, P.err)) break;
    }
    mbar_expect_tx(&sm.full[s], T.total);
    char* dst = ring + (size_t)s * kStageBytes;
    if (P.l2mode) {
      const uint64_t pol = T.keep ? pol_keep : pol_other;
      for (int j = 0; j < T.n; j++) bulk_g2s_hint(dst + T.off[j], T.src[j], T.bytes[j], &sm.full[s], pol);
    } else {
      for (int j = 0; j < T.n; j++) bulk_g2s(dst + T.off[j], T.src[j], T.bytes[j], &sm.full[s]);
    }
    k++;
    if (kLookahead > 0 && k >= (unsigned)kStages) {
      // One more tile of lookahead per tile issued, up to kLookahead beyond the ring.
      int burst = k == (unsigned)kStages ? kLookahead : 1;
      for (int b = 0; b < burst; b++) {
        if (!ahead.next(A)) break;
        for (int j = 0; j < A.n; j++) prefetch_l2(A.src[j], A.bytes[j]);
      }
    }
  }
  // Drain: every copy issued must land before the CTA may exit, also when the
  // step is being abandoned because some CTA's wait ran out.
  unsigned first = k > (unsigned)kStages ? k - kStages : 0;
  for (unsigned j = first; j < k; j++) wait_mbar_own(&sm.full[j % kStages], (j / kStages) & 1, P.err);
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------

// GL: the plan has global-attention layers (G projection, GQA items, gap);
// the kernel without them keeps the smaller code of the S/L path.
template <bool GL, int WB>
struct Cons {
  const Plan& P;
  Smem& sm;
  char* ring;
  unsigned k = 0;         // tiles consumed
  unsigned barriers = 0;  // grid barriers passed in this step
  bool ok = true;
  int tid, warp, lane;
  long long pos;
  unsigned ep;   // the session's step counter at entry
  int cur = 0;   // index of the running phase

  __device__ Cons(const Plan& p, Smem& s, char* r, long long ps, unsigned e)
      : P(p), sm(s), ring(r), pos(ps), ep(e) {
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
  }

  // Tag of phase q's outputs in this step (never 0: zeroed buffers match no tag).
  __device__ __forceinline__ unsigned tag_of(int q) const {
    return (((ep & 0x7fffffu) | 0x800000u) << kTagPhaseBits) | (unsigned)q;
  }
  // A fixed-point slot or counter of this step's parity set.
  template <class T>
  __device__ __forceinline__ T* fxp(T* base) const {
    return base + (ep & 1) * P.fx_stride;
  }
  // Contributions a fixed-point input needs; the stall test asks for one that never comes.
  __device__ __forceinline__ unsigned fx_need(const Phase& ph) const {
    return (unsigned)ph.fx_cnt + (P.test_stall ? 1u : 0u);
  }
  // Before reading a fixed-point input whose writers announce their adds:
  // one thread polls the arrival word, the others wait at a consumers barrier.
  __device__ __forceinline__ void fx_wait_arrivals(const Phase& ph) {
    if (!ph.fx_in || !ph.fx_arrive) return;
    if (tid == 0) {
      const unsigned long long ta = P.trace ? now_ns() : 0;
      const unsigned long long* a = fxp(ph.fx_in) + P.d;
      const unsigned long long want = (unsigned long long)ph.fx_arrive + (P.test_stall ? 1u : 0u);
      Spin sp;
      while (ld_relaxed_u64(a) < want)
        if (!sp.again(P.err)) {
          ok = false;
          break;
        }
      if (ta) xwait += now_ns() - ta;
    }
    all_ok();
  }
  // One tagged value (bounded wait; clears ok when it gives up).
  __device__ __forceinline__ float tval(const unsigned long long* p, unsigned tag) {
    float v[1];
    if (!poll_tagged<1>(p, 1, tag, P.err, v)) ok = false;
    return v[0];
  }

  // Starts copying phase q's descriptor into sm.ph[slot]; it lands by the
  // next consumers barrier after stage_wait().  Reading descriptors from
  // shared memory keeps them off the critical path of the phase start.
  __device__ void stage_phase(int slot, int q) {
    constexpr int chunks = sizeof(Phase) / 16;
    if (q < P.nphases && tid < chunks)
      cp_async16(reinterpret_cast<char*>(&sm.ph[slot]) + tid * 16,
                 reinterpret_cast<const char*>(P.phases + q) + tid * 16);
  }
  __device__ void stage_wait() { cp_async_wait_all(); }

  unsigned long long waited = 0, pro_ns = 0, comp_ns = 0, epi_ns = 0, ntiles = 0, xwait = 0;  // for the timeline

  __device__ const float* take() {
    int s = k % kStages;
    unsigned long long t0 = P.trace && tid == 0 ? now_ns() : 0;
    int got = wait_mbar(&sm.full[s], (k / kStages) & 1, P.err) ? 1 : 0;
    if (t0) waited += now_ns() - t0;
    if (!consumers_and(got)) {
      ok = false;
      return nullptr;
    }
    return reinterpret_cast<const float*>(ring + (size_t)s * kStageBytes);
  }
  // Per-warp variant: no CTA barrier, so warps overlap their tile work; a
  // failed wait only clears `ok`, and items end with a uniform check.
  __device__ const float* take_warp() {
    int s = k % kStages;
    unsigned long long t0 = P.trace && tid == 0 ? now_ns() : 0;
    if (!wait_mbar(&sm.full[s], (k / kStages) & 1, P.err)) ok = false;
    if (t0) waited += now_ns() - t0;
    return reinterpret_cast<const float*>(ring + (size_t)s * kStageBytes);
  }
  // Consumers barrier that also makes `ok` uniform; false when any failed.
  __device__ bool all_ok() {
    if (!consumers_and(ok ? 1 : 0)) ok = false;
    return ok;
  }

  __device__ void release() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[k % kStages]);
    k++;
  }

  // Grid barrier: a monotonic arrival count (reset at the end of the step);
  // barrier b of the step completes when the count reaches b · grid.
  __device__ void grid_sync() {
    consumers_sync();
    barriers++;
    if (tid == 0) {
      unsigned* cnt = P.bar;
      const unsigned target = barriers * gridDim.x + (P.test_stall && barriers == 1 ? 1u : 0u);
      red_release_add(cnt, 1u);  // release: covers the CTA's writes ordered by the barrier above
      unsigned long long t0 = 0;
      for (unsigned it = 0; ld_acquire(cnt) < target; it++) {
        if ((it & 15) == 15) {
          if (ld_volatile(P.err) & 8) {
            sm.flag = 1;
            break;
          }
          if (!t0) {
            t0 = now_ns();
          } else if (now_ns() - t0 > kWaitNs) {
            atomicOr(P.err, 8);
            sm.flag = 1;
            break;
          }
        }
      }
    }
    consumers_sync();
    if (sm.flag == 1) ok = false;
  }

  // Float4 i4 of a phase's `a` input: the fixed-point slot of the fused phase
  // that produced it, once final, or the float buffer (after a grid barrier).
  __device__ __forceinline__ float4 in4(const Phase& ph, int i4) {
    if (ph.fx_in) {
      float4 v;
      if (!fx_poll4(fxp(ph.fx_in), i4, fx_need(ph), P.err, &v)) ok = false;
      return v;
    }
    return __ldcg(reinterpret_cast<const float4*>(ph.in_a) + i4);
  }

  // Input vector of a GEMV phase into sm.xin (and the raw x into sm.xraw).
  // Every load of a thread is issued before any is used.
  __device__ void prologue(const Phase& ph) {
    const int n4 = ph.cols / 4;
    if (ph.in_mode == IN_ATTN) {
      attn_merge(ph);
      return;
    }
    if (ph.in_mode == IN_PLAIN) {
      fx_wait_arrivals(ph);
      if (!ok) return;
      constexpr int J = kMaxCols / 4 / 256;
      float4 v[J];
      const float4* a4 = reinterpret_cast<const float4*>(ph.in_a);
#pragma unroll
      for (int j = 0; j < J; j++)
        if (tid + j * 256 < n4) v[j] = ph.fx_in ? in4(ph, tid + j * 256) : __ldcg(a4 + tid + j * 256);
#pragma unroll
      for (int j = 0; j < J; j++)
        if (tid + j * 256 < n4) reinterpret_cast<float4*>(sm.xin)[tid + j * 256] = v[j];
      all_ok();
      return;
    }
    if (GL && ph.in_mode == IN_RMS_E) {
      // G: v = rms(x)·w (+ rms(e0)·w_e), as two normalisations and one add.
      fx_wait_arrivals(ph);
      if (!ok) return;
      const bool own = tid < n4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f), e = x, w = x, we = x;
      if (own) {
        w = __ldg(reinterpret_cast<const float4*>(ph.norm_w) + tid);
        x = in4(ph, tid);
        if (ph.in_c) {  // e0: this step's embedding row, read from the weights
          const uint32_t id = sm.cur_id;
          we = __ldg(reinterpret_cast<const float4*>(ph.in_c) + tid);
          e = __ldg(reinterpret_cast<const float4*>(P.embed + (size_t)id * ph.cols) + tid);
        }
        reinterpret_cast<float4*>(sm.xraw)[tid] = x;
      }
      float s1 = x.x * x.x, s2 = e.x * e.x;
      s1 = fmaf(x.y, x.y, s1), s2 = fmaf(e.y, e.y, s2);
      s1 = fmaf(x.z, x.z, s1), s2 = fmaf(e.z, e.z, s2);
      s1 = fmaf(x.w, x.w, s1), s2 = fmaf(e.w, e.w, s2);
      s1 = warp_sum(s1), s2 = warp_sum(s2);
      if (lane == 0) sm.red[warp] = s1, sm.red[kConsumerWarps + warp] = s2;
      if (!all_ok()) return;
      float t1 = 0.0f, t2 = 0.0f;
#pragma unroll
      for (int q = 0; q < kConsumerWarps; q++) t1 += sm.red[q], t2 += sm.red[kConsumerWarps + q];
      const float r1 = 1.0f / sqrtf(t1 / (float)ph.cols + P.eps), r2 = 1.0f / sqrtf(t2 / (float)ph.cols + P.eps);
      if (own) {
        float4 v = make_float4(x.x * r1 * w.x, x.y * r1 * w.y, x.z * r1 * w.z, x.w * r1 * w.w);
        if (ph.in_c) {
          v.x = v.x + e.x * r2 * we.x, v.y = v.y + e.y * r2 * we.y;
          v.z = v.z + e.z * r2 * we.z, v.w = v.w + e.w * r2 * we.w;
        }
        reinterpret_cast<float4*>(sm.xin)[tid] = v;
        if (blockIdx.x == 0 && ph.xout) reinterpret_cast<float4*>(ph.xout)[tid] = v;
      }
      consumers_sync();
      return;
    }
    rms_prologue(ph);
  }

  // Normalised input (IN_RMS, IN_EMBED_RMS, IN_LOOP_RMS): d ≤ kMaxD, at most
  // one float4 per thread.
  __device__ __forceinline__ void rms_prologue(const Phase& ph) {
    fx_wait_arrivals(ph);
    if (!ok) return;
    const int n4 = ph.cols / 4;
    const bool own = tid < n4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f), w = x;
    if (own) {
      w = __ldg(reinterpret_cast<const float4*>(ph.norm_w) + tid);
      if (ph.in_mode == IN_EMBED_RMS) {
        const uint32_t id = sm.cur_id;
        x = __ldg(reinterpret_cast<const float4*>(P.embed + (size_t)id * ph.cols) + tid);
        if (blockIdx.x == 0) {
          reinterpret_cast<float4*>(P.e0)[tid] = x;
          reinterpret_cast<float4*>(P.x0)[tid] = x;
        }
      } else if (ph.in_mode == IN_LOOP_RMS) {
        // All three terms in one round of loads per poll (the loop
        // embedding row, the slot's values and the tagged inject term), so
        // their latencies overlap.
        const float4 c = __ldg(reinterpret_cast<const float4*>(ph.in_c) + tid);
        float4 a, b;
        Spin sp;
        bool done;
        do {
          bool ga = true, gb = true;
          if (ph.fx_in)
            ga = fx_try4(fxp(ph.fx_in), tid, fx_need(ph), &a);
          else
            a = __ldcg(reinterpret_cast<const float4*>(ph.in_a) + tid);
          if (ph.tin_b)  // the inject output, tagged by its phase
            gb = try_tagged4(ph.tin_b + 4 * tid, tag_of(ph.tag_in), &b);
          else
            b = __ldcg(reinterpret_cast<const float4*>(ph.in_b) + tid);
          done = ga && gb;
        } while (!done && sp.again(P.err));
        if (!done) ok = false;
        x = make_float4((a.x + b.x) + c.x, (a.y + b.y) + c.y, (a.z + b.z) + c.z, (a.w + b.w) + c.w);
        if (blockIdx.x == 0) reinterpret_cast<float4*>(ph.xout)[tid] = x;
      } else {
        x = in4(ph, tid);
      }
      reinterpret_cast<float4*>(sm.xraw)[tid] = x;
    }
    float ss = x.x * x.x;
    ss = fmaf(x.y, x.y, ss);
    ss = fmaf(x.z, x.z, ss);
    ss = fmaf(x.w, x.w, ss);
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
    if (!all_ok()) return;  // every input final (or the step is being abandoned)
    float tsum = 0.0f;
#pragma unroll
    for (int q = 0; q < kConsumerWarps; q++) tsum += sm.red[q];
    const float r = 1.0f / sqrtf(tsum / (float)ph.cols + P.eps);
    if (own)
      reinterpret_cast<float4*>(sm.xin)[tid] =
          make_float4(x.x * r * w.x, x.y * r * w.y, x.z * r * w.z, x.w * r * w.w);
    consumers_sync();
  }

  // Merge of the attention partials for one GEMV input (see attn_merge).
  template <int Q, int S>
  __device__ void attn_merge_t(const Phase& ph, int d, int s_rt) {
    const int H = ph.heads, Srt = S > 0 ? S : s_rt;
    constexpr int QQ = Q > 0 ? Q : 1, SS = S > 0 ? S : 1;
    float* ml = &sm.cmb[0][0];          // [H·S][2]: m, l; then c = e^{m − M_h}
    float* Lh = &sm.cmb[kMaxSplits / 2][0];  // [H]: Σ_s c·l (after the H·S·2 ≤ 512 floats above)
    const unsigned tg = tag_of(ph.tag_in);  // partials of the attention phase
    for (int i = tid; i < H * Srt; i += 256) {
      ml[2 * i] = tval(ph.tpart + (size_t)i * (kDH + 2) + kDH, tg);
      ml[2 * i + 1] = tval(ph.tpart + (size_t)i * (kDH + 2) + kDH + 1, tg);
    }
    float av[QQ][SS];
    if (Q > 0 && S > 0) {
#pragma unroll
      for (int q = 0; q < QQ; q++) {
        const int o = tid + 256 * q;
        if (o >= d) break;
        const unsigned long long* src = ph.tpart + (size_t)(o / kDH) * S * (kDH + 2) + (o % kDH);
#pragma unroll
        for (int j = 0; j < SS; j++) av[q][j] = tval(src + (size_t)j * (kDH + 2), tg);
      }
    }
    if (!all_ok()) return;
    if (tid < H) {  // per head: the split weights, in split order
      float* m = ml + 2 * tid * Srt;
      float M = -INFINITY;
      for (int j = 0; j < Srt; j++) M = fmaxf(M, m[2 * j]);
      float L = 0.0f;
      for (int j = 0; j < Srt; j++) {
        float c = (M == -INFINITY || m[2 * j] == -INFINITY) ? 0.0f : expf(m[2 * j] - M);
        L += m[2 * j + 1] * c;
        m[2 * j] = c;
      }
      Lh[tid] = L;
    }
    consumers_sync();
    for (int q = 0; q < (d + 255) / 256; q++) {
      const int o = tid + 256 * q;
      if (o >= d) break;
      const float* c = ml + 2 * (o / kDH) * Srt;
      const unsigned long long* src = ph.tpart + (size_t)(o / kDH) * Srt * (kDH + 2) + (o % kDH);
      float A = 0.0f;
#pragma unroll
      for (int j = 0; j < (S > 0 ? S : kMaxSplits); j++) {
        if (j >= Srt) break;
        float a;
        if (Q > 0 && S > 0) {
          a = 0.0f;
#pragma unroll
          for (int qq = 0; qq < QQ; qq++)
            if (qq == q) a = av[qq][j];
        } else {
          a = tval(src + (size_t)j * (kDH + 2), tg);
        }
        A = fmaf(a, c[2 * j], A);
      }
      const float L = Lh[o / kDH];
      sm.xin[o] = L > 0.0f ? A / L : 0.0f;
    }
    all_ok();
  }

  // Attention output y = Σ_s e^{m_s−M}·acc_s / Σ_s e^{m_s−M}·l_s per (head, dim)
  // from the partials of the previous phase ([head][split][dh | m | l]),
  // merged in split order on every CTA: one round of loads, no last-arriver
  // step in the attention phase.
  __device__ void attn_merge(const Phase& ph) {
    const int d = ph.cols;
    if (d == 768 && ph.splits == 12)
      attn_merge_t<3, 12>(ph, d, 12);
    else
      attn_merge_t<0, 0>(ph, d, ph.splits);
  }

  // GEMV phase with K float4 of x per lane held in registers.  A row of
  // `cols` is split over S = 1 or 2 warps (S = 2 above 1536 columns); each
  // warp walks the rows of a tile two at a time (two independent chains).
  // Partial sums land in sm.acc[column half][pair half][output] and are
  // combined, in a fixed order, in the epilogue.
  // NC 16-byte weight chunks per lane per row half (WB bytes a weight).
  template <int NC>
  __device__ void gemv_phase_k(const Phase& ph) {
    constexpr int E = 16 / WB;
    const int G = gridDim.x;
    const int S = ph.cols > 1536 ? 2 : 1;
    const int span = ph.cols / S;
    const int sgi = warp % S, rowslot = warp / S, rstride = kConsumerWarps / S;
    float xr[NC][E];
    {
      const float* xin = sm.xin + sgi * span + lane * E;
#pragma unroll
      for (int c = 0; c < NC; c++)
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          const float4 v = *reinterpret_cast<const float4*>(xin + 32 * E * c + e);
          xr[c][e] = v.x, xr[c][e + 1] = v.y, xr[c][e + 2] = v.z, xr[c][e + 3] = v.w;
        }
    }
    const int T = tile_outs(ph, WB);
    const bool pair = is_pair(ph);
    for (int i = blockIdx.x; i < ph.items && ok; i += G) {
      int s, o0, o1;
      gemv_item(ph, i, &s, &o0, &o1);
      const Segment& sg = ph.seg[s];
      for (int t0 = o0; t0 < o1; t0 += T) {
        const int n = min(T, o1 - t0);
        const int rows = pair ? 2 * n : n;
        const char* w = reinterpret_cast<const char*>(take_warp());
        unsigned long long c0 = P.trace && tid == 0 ? now_ns() : 0;
        for (int r = rowslot; r < rows; r += 2 * rstride) {
          const int r2 = r + rstride;
          const bool two = r2 < rows;
          const uint32_t w0 = saddr(w + ((size_t)r * ph.cols + sgi * span) * WB) + lane * 16;
          const uint32_t w1 = saddr(w + ((size_t)(two ? r2 : r) * ph.cols + sgi * span) * WB) + lane * 16;
          float a0 = 0.0f, b0 = 0.0f, a1 = 0.0f, b1 = 0.0f;
#pragma unroll
          for (int c = 0; c < NC; c++) {
            float u[E], v[E];
            wchunk<WB>(w0 + 512 * c, u);
            wchunk<WB>(w1 + 512 * c, v);
            if (c & 1) {
              b0 = dotn(u, xr[c], b0);
              b1 = dotn(v, xr[c], b1);
            } else {
              a0 = dotn(u, xr[c], a0);
              a1 = dotn(v, xr[c], a1);
            }
          }
          a0 += b0;
          a1 += b1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
          }
          if (lane == 0) {
            const int base = t0 - o0;
            sm.acc[sgi][pair ? r / n : 0][base + (pair ? r % n : r)] = a0;
            if (two) sm.acc[sgi][pair ? r2 / n : 0][base + (pair ? r2 % n : r2)] = a1;
          }
        }
        release();
        if (c0) comp_ns += now_ns() - c0, ntiles++;
      }
      if (!all_ok()) return;  // every partial of the item written
      unsigned long long e0 = P.trace && tid == 0 ? now_ns() : 0;
      if (S == 2)
        for (int t = tid; t < o1 - o0; t += 256) {
          sm.acc[0][0][t] += sm.acc[1][0][t];
          if (pair) sm.acc[0][1][t] += sm.acc[1][1][t];
        }
      if (S == 2) consumers_sync();
      epilogue(ph, sg, o0, o1, i);
      consumers_sync();
      if (e0) epi_ns += now_ns() - e0;
    }
  }

  // Fused MLP items: hidden units j in tiles of n = tile_outs units, laid out
  // [gate rows n][up rows n][downᵀ rows n].  The 2n dot products of a tile go
  // to sm.acc[tile parity] (a warp may start the next tile's products while
  // another still reads this tile's), then every thread adds h_j·downᵀ[j][c]
  // for its columns c = tid + 256·q into y, in unit order.
  template <int K>
  __device__ __forceinline__ void mlp_items(const Phase& ph, float (&y)[kMaxD / 256]) {
    const int G = gridDim.x, d = ph.cols;
    float4 xr[K];
    {
      const float4* xin4 = reinterpret_cast<const float4*>(sm.xin) + lane;
#pragma unroll
      for (int k = 0; k < K; k++) xr[k] = xin4[32 * k];
    }
    const int T = tile_outs(ph, 4);  // f32 weights only (bf16 plans use mlp_items_w)
    unsigned tile = 0;
    for (int i = blockIdx.x; i < ph.items && ok; i += G) {
      int s, o0, o1;
      gemv_item(ph, i, &s, &o0, &o1);
      for (int t0 = o0; t0 < o1; t0 += T, tile++) {
        const int n = min(T, o1 - t0), rows = 2 * n;
        const float* w = take_warp();
        unsigned long long c0 = P.trace && tid == 0 ? now_ns() : 0;
        float(*acc)[kMaxItemOut] = sm.acc[tile & 1];
        for (int r = warp; r < rows; r += 2 * kConsumerWarps) {
          const int r2 = r + kConsumerWarps;
          const bool two = r2 < rows;
          const uint32_t w0 = saddr(w + (size_t)r * d) + lane * 16;
          const uint32_t w1 = saddr(w + (size_t)(two ? r2 : r) * d) + lane * 16;
          float a0 = 0.0f, b0 = 0.0f, a1 = 0.0f, b1 = 0.0f;
#pragma unroll
          for (int k = 0; k < K; k++) {
            float4 u = lds4(w0 + 512 * k), v = lds4(w1 + 512 * k);
            if (k & 1) {
              b0 = dot4(u, xr[k], b0);
              b1 = dot4(v, xr[k], b1);
            } else {
              a0 = dot4(u, xr[k], a0);
              a1 = dot4(v, xr[k], a1);
            }
          }
          a0 += b0;
          a1 += b1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
          }
          if (lane == 0) {
            acc[r / n][r % n] = a0;
            if (two) acc[r2 / n][r2 % n] = a1;
          }
        }
        consumers_sync();  // every gate and up product of the tile
        const uint32_t dt = saddr(w + (size_t)2 * n * d) + tid * 4;
        for (int j = 0; j < n; j++) {
          const float h = silu_mul(acc[0][j], acc[1][j]);
#pragma unroll
          for (int q = 0; q < kMaxD / 256; q++)
            if (tid + 256 * q < d) y[q] = fmaf(h, lds1(dt + (uint32_t)(j * d + 256 * q) * 4), y[q]);
        }
        release();
        if (c0) comp_ns += now_ns() - c0, ntiles++;
      }
      if (!all_ok()) return;
    }
  }

  // Fused MLP items, a warp per hidden unit: unit u of this CTA (counted over
  // its tiles) belongs to warp u mod 8, which forms gate·n and up·n (two
  // chains), h = silu(gate)·up, and adds h·downᵀ[u] into its own partial
  // (columns 4·lane + 128·k).  No CTA barrier per tile; the eight partials are
  // summed once at the end, in a fixed order (needs 4·d ≤ kMaxCols floats of
  // sm.xin).
  template <int NC>
  __device__ __forceinline__ void mlp_items_w(const Phase& ph, float (&y)[kMaxD / 256]) {
    constexpr int E = 16 / WB;
    const int G = gridDim.x, d = ph.cols;
    // Lane `lane` owns columns (lane + 32·c)·E … + E − 1 of x and of its partial.
    float xr[NC][E], yv[NC][E];
    {
      const bool res = blockIdx.x == 0 && warp == 0;  // the residual, once per slot
#pragma unroll
      for (int c = 0; c < NC; c++)
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          const int col = (lane + 32 * c) * E + e;
          const float4 v = *reinterpret_cast<const float4*>(sm.xin + col);
          const float4 r = res ? *reinterpret_cast<const float4*>(sm.xraw + col) : make_float4(0.f, 0.f, 0.f, 0.f);
          xr[c][e] = v.x, xr[c][e + 1] = v.y, xr[c][e + 2] = v.z, xr[c][e + 3] = v.w;
          yv[c][e] = r.x, yv[c][e + 1] = r.y, yv[c][e + 2] = r.z, yv[c][e + 3] = r.w;
        }
    }
    const int T = tile_outs(ph, WB);
    const size_t rowb = (size_t)d * WB;
    int u = 0;  // units of this CTA before the current tile
    for (int i = blockIdx.x; i < ph.items && ok; i += G) {
      int s, o0, o1;
      gemv_item(ph, i, &s, &o0, &o1);
      for (int t0 = o0; t0 < o1; t0 += T) {
        const int n = min(T, o1 - t0);
        const char* w = reinterpret_cast<const char*>(take_warp());
        unsigned long long c0 = P.trace && tid == 0 ? now_ns() : 0;
        for (int j = (warp - u % kConsumerWarps + kConsumerWarps) % kConsumerWarps; j < n; j += kConsumerWarps) {
          const uint32_t g0 = saddr(w + (size_t)j * rowb) + lane * 16;
          const uint32_t u0 = saddr(w + (size_t)(n + j) * rowb) + lane * 16;
          const uint32_t r0 = saddr(w + (size_t)(2 * n + j) * rowb) + lane * 16;
          // Every load of the unit (gate, up and its down column) is issued
          // before the first product, so their latencies overlap; bf16
          // chunks stay packed until they are used.
          float4 gr[NC], ur[NC], dr[NC];
#pragma unroll
          for (int c = 0; c < NC; c++) gr[c] = lds4(g0 + 512 * c), ur[c] = lds4(u0 + 512 * c);
#pragma unroll
          for (int c = 0; c < NC; c++) dr[c] = lds4(r0 + 512 * c);
          float a0 = 0.0f, b0 = 0.0f, a1 = 0.0f, b1 = 0.0f;
#pragma unroll
          for (int c = 0; c < NC; c++) {
            float gq[E], uq[E];
            widen<WB>(gr[c], gq);
            widen<WB>(ur[c], uq);
            if (c & 1) {
              b0 = dotn(gq, xr[c], b0);
              b1 = dotn(uq, xr[c], b1);
            } else {
              a0 = dotn(gq, xr[c], a0);
              a1 = dotn(uq, xr[c], a1);
            }
          }
          a0 += b0;
          a1 += b1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
          }
          const float h = silu_mul(a0, a1);
#pragma unroll
          for (int c = 0; c < NC; c++) {
            float dq[E];
            widen<WB>(dr[c], dq);
#pragma unroll
            for (int e = 0; e < E; e++) yv[c][e] = fmaf(h, dq[e], yv[c][e]);
          }
        }
        release();
        u += n;
        if (c0) comp_ns += now_ns() - c0, ntiles++;
      }
      if (!all_ok()) return;
    }
    // ((w0 + w4) + (w1 + w5)) + ((w2 + w6) + (w3 + w7)) per column, through sm.xin.
    float* buf = sm.xin;  // [4][d]
    consumers_sync();  // every warp has read its x from sm.xin
    if (warp >= 4)
#pragma unroll
      for (int c = 0; c < NC; c++)
#pragma unroll
        for (int e = 0; e < E; e += 4)
          *reinterpret_cast<float4*>(buf + (warp - 4) * d + (lane + 32 * c) * E + e) =
              make_float4(yv[c][e], yv[c][e + 1], yv[c][e + 2], yv[c][e + 3]);
    consumers_sync();
    if (warp < 4)
#pragma unroll
      for (int c = 0; c < NC; c++)
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          float4& o = *reinterpret_cast<float4*>(buf + warp * d + (lane + 32 * c) * E + e);
          const float4 v = o;
          o = make_float4(yv[c][e] + v.x, yv[c][e + 1] + v.y, yv[c][e + 2] + v.z, yv[c][e + 3] + v.w);
        }
    consumers_sync();
    const float* b = sm.xin;
#pragma unroll
    for (int q = 0; q < kMaxD / 256; q++) {
      const int c = tid + 256 * q;
      if (c < d) y[q] = (b[c] + b[d + c]) + (b[2 * d + c] + b[3 * d + c]);
    }
  }

  // The whole MLP of a block as one phase: x' = x + down·(silu(gate·n)·(up·n))
  // with n = rms(x)·w.  Each CTA sums its hidden units' down columns on chip
  // and adds them, as int64 fixed point, into the phase's slot; CTA 0 also adds
  // the residual x.  The next phase reads x' from the slot.
  __device__ __forceinline__ void mlp_phase(const Phase& ph) {
    unsigned long long t0 = P.trace && tid == 0 ? now_ns() : 0;
    rms_prologue(ph);  // the plan gives fused MLPs IN_RMS inputs
    if (t0) pro_ns += now_ns() - t0;
    if (!ok) return;
    const int d = ph.cols;
    if (blockIdx.x >= ph.items) {  // no hidden units here: count in, so readers know the sum is final
      for (int c = tid; c < d; c += 256) red_add_fx(fxp(ph.fx_out) + c, kFxOne);
      consumers_sync();
      if (tid == 0) red_add_fx(fxp(ph.fx_out) + d, 1ull);  // this CTA's adds are issued
      return;
    }
    float y[kMaxD / 256];
#pragma unroll
    for (int q = 0; q < kMaxD / 256; q++) y[q] = 0.0f;
    if (!P.mlp_cta) {
      switch (d / (512 / WB)) {  // 16-byte chunks per lane
        case 1: mlp_items_w<1>(ph, y); break;
        case 2: mlp_items_w<2>(ph, y); break;
        case 3: mlp_items_w<3>(ph, y); break;
        case 4: mlp_items_w<4>(ph, y); break;
        case 6: mlp_items_w<6>(ph, y); break;
        default: break;  // d > 768 takes the per-tile CTA split (mlp_cta set by the plan)
      }
    } else if constexpr (WB == 4) {  // the row-split variant reads f32 tiles only
#pragma unroll
      for (int q = 0; q < kMaxD / 256; q++) {
        const int c = tid + 256 * q;
        y[q] = blockIdx.x == 0 && c < d ? sm.xraw[c] : 0.0f;
      }
      switch (d / 128) {
        case 1: mlp_items<1>(ph, y); break;
        case 2: mlp_items<2>(ph, y); break;
        case 3: mlp_items<3>(ph, y); break;
        case 4: mlp_items<4>(ph, y); break;
        case 6: mlp_items<6>(ph, y); break;
        case 8: mlp_items<8>(ph, y); break;
        default: break;  // excluded when the plan is built
      }
    }
    if (!ok) return;
    unsigned long long e0 = P.trace && tid == 0 ? now_ns() : 0;
    bool bad = false;
    unsigned long long* fo = fxp(ph.fx_out);
#pragma unroll
    for (int q = 0; q < kMaxD / 256; q++) {
      const int c = tid + 256 * q;
      if (c < d) red_add_fx(fo + c, fx_word(y[q], &bad));
    }
    if (bad) atomicOr(P.err, 16);
    consumers_sync();
    if (tid == 0) red_add_fx(fo + d, 1ull);  // this CTA's adds are issued
    if (e0) epi_ns += now_ns() - e0;
  }

  __device__ void gemv_phase(const Phase& ph) {
    if (ph.out_mode == OUT_MLP) {
      mlp_phase(ph);
      return;
    }
    // Normalising prologues run everywhere: they also refresh sm.xraw, the
    // residual of the phases that follow.
    if (blockIdx.x >= ph.items && ph.in_mode == IN_PLAIN) return;
    unsigned long long t0 = P.trace && tid == 0 ? now_ns() : 0;
    prologue(ph);
    if (t0) pro_ns += now_ns() - t0;
    if (!ok || blockIdx.x >= ph.items) return;
    const int K = ph.cols / (ph.cols > 1536 ? 2 : 1) / (512 / WB);  // 16-byte chunks per lane and row half
    switch (K) {
      case 1: gemv_phase_k<1>(ph); break;
      case 2: gemv_phase_k<2>(ph); break;
      case 3: gemv_phase_k<3>(ph); break;
      case 4: gemv_phase_k<4>(ph); break;
      case 6: gemv_phase_k<6>(ph); break;
      case 8: gemv_phase_k<8>(ph); break;
      case 12: gemv_phase_k<12>(ph); break;
      default: break;  // excluded when the plan is built
    }
  }

  __device__ void epilogue(const Phase& ph, const Segment& sg, int o0, int o1, int item) {
    const int n = o1 - o0;
    if (GL && ph.out_mode == OUT_G) {
      if (&sg == &ph.seg[0]) {  // q rows, scaled as the graph path does (k_g_post)
        const float f = ph.inv_log > 0.0f ? log1pf((float)pos) * ph.inv_log : 1.0f;
        const unsigned tg = tag_of(cur);
        for (int t = tid; t < n; t += 256) {
          const float a = sm.acc[0][0][t];
          const float v = ph.inv_log > 0.0f ? a * f : a;
          if (sg.tout)
            put_tagged(sg.tout + o0 + t, v, tg);
          else
            sg.out[o0 + t] = v;
        }
      } else {  // kv rows: [keys (heads · dh) | values (heads · dh)]
        const int kd = ph.heads * kDH;
        for (int t = tid; t < n; t += 256) {
          const int o = o0 + t;
          const float a = sm.acc[0][0][t];
          if (o < kd) {
            const long long slot = ph.kshift ? pos + 1 : pos;
            ph.kc[((size_t)(o / kDH) * ph.cap + (size_t)slot) * kDH + o % kDH] = a;
          } else {
            const int u = o - kd;
            ph.vc[((size_t)(u / kDH) * ph.cap + (size_t)pos) * kDH + u % kDH] = a;
          }
        }
      }
      return;
    }
    if (ph.out_mode == OUT_ROPE) {
      // q, k, v of this position: tagged into tq ([q | k | v], d each) for
      // the attention phase; k and v also into the ring (later steps).
      const int d = P.d;
      const size_t slot = (size_t)(pos % ph.cap);
      const unsigned tg = tag_of(cur);
      for (int t = tid; t < n; t += 256) {
        int o = o0 + t;
        int sec = o / (d / 2), rem = o % (d / 2), h = rem / 32, j = rem % 32;
        float a = sm.acc[0][0][t], b = sm.acc[0][1][t];
        float u = a, v = b;
        if (sec < 2) {
          float ang = (float)pos * sm.inv_freq[j];
          float sn, cs;
          sincosf(ang, &sn, &cs);
          u = a * cs - b * sn, v = a * sn + b * cs;
        }
        if (sec > 0) {
          float* r = (sec == 1 ? ph.kc : ph.vc) + ((size_t)h * ph.cap + slot) * kDH;
          r[j] = u;
          r[32 + j] = v;
        }
        unsigned long long* tq = ph.tq + (size_t)sec * d + h * kDH;
        put_tagged(tq + j, u, tg);
        put_tagged(tq + 32 + j, v, tg);
      }
      return;
    }
    for (int t = tid; t < n; t += 256) {
      int o = o0 + t;
      float a = sm.acc[0][0][t];
      if (ph.out_mode == OUT_ADD)
        sg.out[o] = (ph.res_smem ? sm.xraw[o] : __ldcg(sg.out + o)) + a;
      else if (ph.out_mode == OUT_SILU)
        sg.out[o] = silu_mul(a, sm.acc[0][1][t]);
      else if (sg.tout)
        put_tagged(sg.tout + o, a, tag_of(cur));
      else
        sg.out[o] = a;
    }
    if (ph.out_mode == OUT_LOGITS) logits_argmax(o0, n, item, ph.items);
  }

  __device__ void logits_argmax(int o0, int n, int item, int items) {
    unsigned long long best = 0;
    for (int t = tid; t < n; t += 256) {
      float v = sm.acc[0][0][t];
      if (v != v) continue;
      unsigned long long c = ((unsigned long long)total_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)(o0 + t));
      if (c > best) best = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      if (other > best) best = other;
    }
    if (tid == 0) sm.best = 0;
    consumers_sync();
    if (lane == 0 && best) atomicMax(&sm.best, best);
    consumers_sync();
    if (tid == 0) {
      P.arg_part[item] = sm.best;
      __threadfence();
      unsigned prev = atomicAdd(P.arg_count, 1u);
      sm.flag = prev == (unsigned)items - 1 ? 2 : 0;
    }
    consumers_sync();
    if (sm.flag == 2) {
      __threadfence();
      unsigned long long b = 0;
      for (int j = tid; j < items; j += 256) {
        unsigned long long c = __ldcg(P.arg_part + j);
        if (c > b) b = c;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
        if (other > b) b = other;
      }
      consumers_sync();
      if (tid == 0) sm.best = 0;
      consumers_sync();
      if (lane == 0 && b) atomicMax(&sm.best, b);
      consumers_sync();
      if (tid == 0) {
        uint32_t id = sm.best ? 0xFFFFFFFFu - (uint32_t)(sm.best & 0xFFFFFFFFu) : 0;
        *P.argmax = id;
        if (P.argmax2) *P.argmax2 = id;
        if (P.greedy) {
          P.next_id[0] = id;
          const unsigned at = atomicAdd(P.out_index, 1u);
          if (P.out_ids) P.out_ids[at] = id;
          if (P.hist) P.hist[P.hist_base + at] = id;
        }
        *P.arg_count = 0;
        P.pos[0] = pos + 1;  // every CTA read the position at entry
        if (P.nsteps > 1) {  // the next step's token, once the count above is reset
          __threadfence();
          st_relaxed_u64(P.next_tagged, ((unsigned long long)tag_of(cur) << 32) | id);
        }
        sm.flag = 0;
      }
      consumers_sync();
    }
  }

  // Attention of the step's query for cache head c, split s: the QG query
  // heads c·QG … that share the head (GQA) walk the same K/V tiles (one HBM
  // read); each writes its (head, split) partial (acc, m, l).
  template <int QG>
  __device__ void attn_item_t(const Phase& ph, int item) {
    const int c = item / ph.splits, s = item % ph.splits;
    const int sub = lane & 7, grp = lane >> 3;
    // Lane `sub` of a group owns dims sub*4 .. sub*4+3 and 32+sub*4 .. 32+sub*4+3,
    // so a group reads each cached row as two contiguous 128-byte runs.
    const int d0 = sub * 4, d1 = 32 + sub * 4;
    float qv[QG][8], mx[QG], l[QG], acc[QG][8];
    const unsigned tg_in = tag_of(ph.tag_in);  // q (and k, v) of the projection phase
    const unsigned long long tq0 = P.trace && tid == 0 ? now_ns() : 0;
#pragma unroll
    for (int g = 0; g < QG; g++) {
      const unsigned long long* qp = ph.tq + (c * QG + g) * kDH;
      float a[4], b[4];
      if (!poll_tagged<4>(qp + d0, 1, tg_in, P.err, a)) ok = false;
      if (!poll_tagged<4>(qp + d1, 1, tg_in, P.err, b)) ok = false;
#pragma unroll
      for (int e = 0; e < 4; e++) qv[g][e] = a[e], qv[g][4 + e] = b[e];
      mx[g] = -INFINITY, l[g] = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; e++) acc[g][e] = 0.0f;
    }
    long long a, b;
    attn_slice<GL>(ph, pos, s, &a, &b);
    unsigned long long c0 = P.trace && tid == 0 ? now_ns() : 0;
    if (tq0) pro_ns += c0 - tq0;
    for (long long t0 = a; t0 < b; t0 += kAttnTile) {
      const int n = (int)min((long long)kAttnTile, b - t0);
      const float* tile = take_warp();
      const float* Kt = tile;
      const float* Vt = tile + kAttnTile * kDH;
      constexpr int J = kAttnTile / 32;
#pragma unroll
      for (int g = 0; g < QG; g++) {
        float sc[J];
#pragma unroll
        for (int j = 0; j < J; j++) {
          const int r = grp + 4 * warp + 32 * j;
          const uint32_t ka = saddr(Kt + (r < n ? r : 0) * kDH);
          float4 k0 = lds4(ka + d0 * 4), k1 = lds4(ka + d1 * 4);
          float x = qv[g][0] * k0.x + qv[g][1] * k0.y + qv[g][2] * k0.z + qv[g][3] * k0.w + qv[g][4] * k1.x +
                    qv[g][5] * k1.y + qv[g][6] * k1.z + qv[g][7] * k1.w;
          x += __shfl_xor_sync(0xffffffffu, x, 1);
          x += __shfl_xor_sync(0xffffffffu, x, 2);
          x += __shfl_xor_sync(0xffffffffu, x, 4);
          sc[j] = r < n ? x * ph.scale : -INFINITY;
        }
        float M = mx[g];
#pragma unroll
        for (int j = 0; j < J; j++) M = fmaxf(M, sc[j]);
        if (M != -INFINITY) {
          const float corr = mx[g] == -INFINITY ? 0.0f : expf(mx[g] - M);
          l[g] *= corr;
#pragma unroll
          for (int e = 0; e < 8; e++) acc[g][e] *= corr;
#pragma unroll
          for (int j = 0; j < J; j++) {
            const int r = grp + 4 * warp + 32 * j;
            if (r >= n) continue;
            const float pe = expf(sc[j] - M);
            l[g] += pe;
            const uint32_t va = saddr(Vt + r * kDH);
            float4 v0 = lds4(va + d0 * 4), v1 = lds4(va + d1 * 4);
            acc[g][0] = fmaf(pe, v0.x, acc[g][0]), acc[g][1] = fmaf(pe, v0.y, acc[g][1]);
            acc[g][2] = fmaf(pe, v0.z, acc[g][2]), acc[g][3] = fmaf(pe, v0.w, acc[g][3]);
            acc[g][4] = fmaf(pe, v1.x, acc[g][4]), acc[g][5] = fmaf(pe, v1.y, acc[g][5]);
            acc[g][6] = fmaf(pe, v1.z, acc[g][6]), acc[g][7] = fmaf(pe, v1.w, acc[g][7]);
          }
          mx[g] = M;
        }
      }
      release();
    }
    unsigned long long e0 = 0;
    if (c0) {
      e0 = now_ns();
      comp_ns += e0 - c0;
      ntiles++;
    }
    if ((!GL || ph.gap == 0) && s == ph.splits - 1 && warp == 0 && grp == 0) {
      // The step's own position: tagged by the projection phase, or (after a
      // grid barrier) in the cache where it stored them.
      float kk[8], vv[8];
      if (ph.tkv) {
        const unsigned long long* kr = ph.tkv + c * kDH;
        const unsigned long long* vr = kr + P.d;
        float a[4], b[4], e4[4], f4[4];
        if (!poll_tagged<4>(kr + d0, 1, tg_in, P.err, a)) ok = false;
        if (!poll_tagged<4>(kr + d1, 1, tg_in, P.err, b)) ok = false;
        if (!poll_tagged<4>(vr + d0, 1, tg_in, P.err, e4)) ok = false;
        if (!poll_tagged<4>(vr + d1, 1, tg_in, P.err, f4)) ok = false;
#pragma unroll
        for (int e = 0; e < 4; e++) kk[e] = a[e], kk[4 + e] = b[e], vv[e] = e4[e], vv[4 + e] = f4[e];
      } else {
        const size_t slot = (size_t)(pos % ph.cap);
        const float* kr = ph.kc + ((size_t)c * ph.cap + slot) * kDH;
        const float* vr = ph.vc + ((size_t)c * ph.cap + slot) * kDH;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          kk[e] = __ldcg(kr + d0 + e), kk[4 + e] = __ldcg(kr + d1 + e);
          vv[e] = __ldcg(vr + d0 + e), vv[4 + e] = __ldcg(vr + d1 + e);
        }
      }
#pragma unroll
      for (int g = 0; g < QG; g++) {
        float sc = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) sc += qv[g][e] * kk[e];
        sc += __shfl_xor_sync(0x000000ffu, sc, 1);
        sc += __shfl_xor_sync(0x000000ffu, sc, 2);
        sc += __shfl_xor_sync(0x000000ffu, sc, 4);
        sc *= ph.scale;
        const float M = fmaxf(mx[g], sc);
        const float corr = mx[g] == -INFINITY ? 0.0f : expf(mx[g] - M);
        const float pe = expf(sc - M);
        l[g] = l[g] * corr + pe;
#pragma unroll
        for (int e = 0; e < 8; e++) acc[g][e] = acc[g][e] * corr + pe * vv[e];
        mx[g] = M;
      }
    }
#pragma unroll
    for (int g = 0; g < QG; g++) {
      // Merge the four lane groups of each warp, then the warps.
#pragma unroll
      for (int o = 8; o < 32; o <<= 1) {
        float om = __shfl_xor_sync(0xffffffffu, mx[g], o), ol = __shfl_xor_sync(0xffffffffu, l[g], o);
        float M = fmaxf(mx[g], om);
        float ca = mx[g] == -INFINITY ? 0.0f : expf(mx[g] - M), cb = om == -INFINITY ? 0.0f : expf(om - M);
        l[g] = l[g] * ca + ol * cb;
#pragma unroll
        for (int e = 0; e < 8; e++) acc[g][e] = acc[g][e] * ca + __shfl_xor_sync(0xffffffffu, acc[g][e], o) * cb;
        mx[g] = M;
      }
      if (grp == 0) {
#pragma unroll
        for (int e = 0; e < 4; e++) sm.wsm[warp][d0 + e] = acc[g][e], sm.wsm[warp][d1 + e] = acc[g][4 + e];
        if (sub == 0) sm.wsm[warp][kDH] = mx[g], sm.wsm[warp][kDH + 1] = l[g];
      }
      if (!all_ok()) return;
      unsigned long long* out = ph.tpart + ((size_t)(c * QG + g) * ph.splits + s) * (kDH + 2);
      if (tid < kDH + 2) {
        const int e = tid < kDH ? tid : 0;
        float m0 = sm.wsm[0][kDH], l0 = sm.wsm[0][kDH + 1], a0 = sm.wsm[0][e];
        for (int w = 1; w < kConsumerWarps; w++) {
          float om = sm.wsm[w][kDH], ol = sm.wsm[w][kDH + 1];
          float M = fmaxf(m0, om);
          float ca = m0 == -INFINITY ? 0.0f : expf(m0 - M), cb = om == -INFINITY ? 0.0f : expf(om - M);
          l0 = l0 * ca + ol * cb;
          a0 = a0 * ca + sm.wsm[w][e] * cb;
          m0 = M;
        }
        put_tagged(out + tid, tid < kDH ? a0 : (tid == kDH ? m0 : l0), tag_of(cur));
      }
      consumers_sync();  // sm.wsm is free for the next head / item
    }
    if (e0) epi_ns += now_ns() - e0;
  }

  // Attention + o (S blocks).  The CTA of (head h, split s) has written its
  // partial; it counts itself in for h and waits (bounded) for the head's
  // other splits, merges the partials in split order (as the o prologue's
  // merge does), multiplies rows s·R … s·R + R − 1 of h's o block (one tile;
  // four threads per row) and adds them into the fixed-point slot; head 0's
  // CTAs add the residual rows.  Every output row gets one part per head.
  // The residual rows and the tile are fetched before the wait.
  __device__ __forceinline__ void attn_o_tail(const Phase& ph, int h, int s) { mixer_o_tail(ph, h, s, false); }

  // The same for L blocks: every split of head h ran the GLA itself (gla_item)
  // and holds y_h in sm.vec[0], so there is nothing to wait for or merge.
  __device__ __forceinline__ void mixer_o_tail(const Phase& ph, int h, int s, bool gla) {
    constexpr int RQ = kMaxItemOut / 64;  // rows per thread: r = tid / 4 + 64·k
    const int R = ph.orows, q4 = tid & 3;
    const unsigned long long to0 = P.trace && tid == 0 ? now_ns() : 0;
    float res[RQ];  // the block's input x, which this CTA's own prologue left in sm.xraw
#pragma unroll
    for (int k = 0; k < RQ; k++) {
      const int r = (tid >> 2) + 64 * k;
      res[k] = h == 0 && q4 == 0 && r < R ? sm.xraw[s * R + r] : 0.0f;
    }
    const float* w = take_warp();
    // The merge, in split order: the head's partials ([split][acc | m | l]),
    // polled by all threads into sm.cmb until every split has tagged its own
    // (one load round per poll); the split weights c_j = e^(m_j − M) once per
    // split, in sm.red.
    if (!gla) {
      const unsigned long long* pp = ph.tpart + (size_t)h * ph.splits * (kDH + 2);
      const unsigned tg = tag_of(cur);
      constexpr int NV = (kMaxSplits * (kDH + 2) + 255) / 256;
      const int nv = ph.splits * (kDH + 2);
      Spin sp;
      const unsigned long long tw0 = to0 ? now_ns() : 0;
      for (;;) {
        unsigned long long wv[NV];
#pragma unroll
        for (int k = 0; k < NV; k++)
          if (tid + 256 * k < nv) wv[k] = ld_relaxed_u64(pp + tid + 256 * k);
        bool all = true;
#pragma unroll
        for (int k = 0; k < NV; k++)
          if (tid + 256 * k < nv) {
            const int i = tid + 256 * k;
            all &= (unsigned)(wv[k] >> 32) == tg;
            sm.cmb[i / (kDH + 2)][i % (kDH + 2)] = __uint_as_float((unsigned)wv[k]);
          }
        if (all) break;
        if (!sp.again(P.err)) {
          ok = false;
          break;
        }
      }
      if (tw0) xwait += now_ns() - tw0;
      all_ok();
      if (ok && tid < ph.splits) {
        float M = -INFINITY;
        for (int j = 0; j < ph.splits; j++) M = fmaxf(M, sm.cmb[j][kDH]);
        const float m = sm.cmb[tid][kDH];
        sm.red[tid] = (M == -INFINITY || m == -INFINITY) ? 0.0f : expf(m - M);
      }
      consumers_sync();
      if (ok && tid < kDH) {
        float A = 0.0f, L = 0.0f;
        for (int j = 0; j < ph.splits; j++) {
          const float c = sm.red[j];
          L += sm.cmb[j][kDH + 1] * c;
          A = fmaf(sm.cmb[j][tid], c, A);
        }
        sm.vec[0][tid] = L > 0.0f ? A / L : 0.0f;
      }
    }
    consumers_sync();
    // Row r = tid / 4 (+ 64·k): thread q4 takes the 16-byte chunks q4 + 4·i
    // of the row (E columns each).
    bool bad = false;
    if (ok) {
      constexpr int E = 16 / WB, CPT = kDH / E / 4;
      float yq[CPT][E];
#pragma unroll
      for (int i = 0; i < CPT; i++)
#pragma unroll
        for (int e = 0; e < E; e++) yq[i][e] = sm.vec[0][(q4 + 4 * i) * E + e];
#pragma unroll
      for (int k = 0; k < RQ; k++) {
        const int r = (tid >> 2) + 64 * k;
        if (64 * k >= R) break;  // uniform
        float v = 0.0f;
        if (r < R) {
          const uint32_t a = saddr(reinterpret_cast<const char*>(w) + (size_t)r * kDH * WB) + q4 * 16;
#pragma unroll
          for (int i = 0; i < CPT; i++) {
            float wq[E];
            wchunk<WB>(a + 64 * i, wq);
            v = dotn(wq, yq[i], v);
          }
        }
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (q4 == 0 && r < R) red_add_fx(fxp(ph.fx_out) + s * R + r, fx_word(v + res[k], &bad));
      }
    }
    release();
    if (bad) atomicOr(P.err, 16);
    all_ok();  // sm.cmb and sm.vec are free; ok uniform
    if (to0) epi_ns += now_ns() - to0;
  }

  __device__ void attn_item(const Phase& ph, int item) {
    if (!GL) {
      attn_item_t<1>(ph, item);
      return;
    }
    switch (ph.qg) {
      case 2: attn_item_t<2>(ph, item); break;
      case 3: attn_item_t<3>(ph, item); break;
      default: attn_item_t<1>(ph, item); break;  // the plan allows 1..3
    }
  }

  // GLA for head h: l2norm q, k; S = d·S + kᵀv; y = q·S; head_norm; silu gate.
  // With o in the phase (ph.wo) every split s of the head runs it on its own
  // copy of the state and keeps y_h in sm.vec[0]; splits other than 0 report
  // that their copy has landed, and split 0 writes the new state back only
  // after all of them have.
  __device__ void gla_item(const Phase& ph, int h, int s = 0) {
    const int d = P.d;
    // The layer's constants first, so their loads overlap the polls below.
    const float bias = __ldg(ph.bias + h);
    const float hn = warp < 2 ? __ldg(ph.hnw + tid) : 0.0f;
    // [q | k | v | g] rows (each d wide) and the decay, tagged by the projection phase.
    const unsigned tg = tag_of(ph.tag_in);
    if (tid < kDH) {
      float v[4];
      if (!poll_tagged<4>(ph.tmix + h * kDH + tid, d, tg, P.err, v)) ok = false;
#pragma unroll
      for (int k = 0; k < 4; k++) sm.vec[k][tid] = v[k];
    }
    const float dcy = 1.0f / (1.0f + expf(tval(ph.tdec + h, tg) + bias));
    if (!all_ok()) return;
    if (warp < 2) {  // warp 0: |q|, warp 1: |k|
      float a = sm.vec[warp][lane], b = sm.vec[warp][lane + 32];
      float ss = warp_sum(a * a + b * b);
      float r = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
      sm.vec[warp][lane] = a * r;
      sm.vec[warp][lane + 32] = b * r;
    }
    float* tile = const_cast<float*>(take());  // (its barrier also orders the l2norm above)
    if (!tile) return;
    unsigned long long* cnt = ph.wo ? fxp(ph.cnt) + h : nullptr;
    if (ph.wo && s != 0 && tid == 0) red_release_add_u64(cnt, 1ull);  // the old state is read
    const int b = tid & 63, qa = tid >> 6;
    const float vb = sm.vec[2][b];
    float yp = 0.0f;
#pragma unroll
    for (int a = qa * 16; a < qa * 16 + 16; a++) {
      float s = dcy * tile[a * kDH + b] + sm.vec[1][a] * vb;
      tile[a * kDH + b] = s;
      yp = fmaf(sm.vec[0][a], s, yp);
    }
    sm.yp[qa][b] = yp;
    consumers_sync();
    // The gated, normalised output, then the state back to HBM (coalesced).
    if (warp < 2) {
      int bb = tid;
      float y = ((sm.yp[0][bb] + sm.yp[1][bb]) + sm.yp[2][bb]) + sm.yp[3][bb];
      float ss = warp_sum(y * y);
      if (lane == 0) sm.red[warp] = ss;
      asm volatile("bar.sync 2, 64;" ::: "memory");
      float tot = sm.red[0] + sm.red[1];
      float r = 1.0f / sqrtf(tot / (float)kDH + P.eps);
      const float o = silu_mul(sm.vec[3][bb], y * r * hn);
      if (ph.wo)
        sm.vec[0][bb] = o;  // q is no longer read: every thread passed the barrier above
      else
        ph.y[h * kDH + bb] = o;
    }
    if (ph.wo && s != 0) {
      consumers_sync();
      release();
      return;
    }
    if (ph.wo && tid == 0) {  // split 0: every other split's copy of the old state has landed
      unsigned long long t0 = 0;
      for (unsigned it = 0; ld_acquire_u64(cnt) < (unsigned long long)(ph.splits - 1); it++) {
        if ((it & 15) == 15) {
          if (ld_volatile(P.err) & 8) {
            sm.flag = 1;
            break;
          }
          if (!t0) {
            t0 = now_ns();
          } else if (now_ns() - t0 > kWaitNs) {
            atomicOr(P.err, 8);
            sm.flag = 1;
            break;
          }
        }
      }
    }
    if (ph.wo) {
      consumers_sync();
      if (sm.flag == 1) ok = false;
    }
    float* Sg = ph.state + (size_t)h * kDH * kDH;
    if (ok)
      for (int e = tid; e < kDH * kDH; e += 256) Sg[e] = tile[e];
    consumers_sync();
    release();
  }

  __device__ void stamp(int p, int which) {
    if (P.trace && tid == 0) {
      unsigned long long* t = P.trace + ((size_t)p * gridDim.x + blockIdx.x) * 8;
      t[which] = now_ns();
      if (which == 1) {
        t[2] = waited, t[3] = pro_ns, t[4] = comp_ns, t[5] = epi_ns, t[6] = ntiles, t[7] = xwait;
        waited = pro_ns = comp_ns = epi_ns = ntiles = xwait = 0;
      }
    }
  }

  // Zeroes the fixed-point set the next step adds into.  Its last readers
  // were in the previous step; the caller guarantees every CTA is past them.
  __device__ void zero_next_set() {
    unsigned long long* nx = P.fx + ((ep + 1) & 1) * P.fx_stride;
    for (int e = blockIdx.x * 256 + tid; e < P.fx_words; e += gridDim.x * 256) nx[e] = 0;
  }

  __device__ void run_phase(const Phase& ph) {
    if (ph.kind == PH_GEMV) {
      gemv_phase(ph);
    } else if (ph.kind == PH_ATTN) {
      for (int i = blockIdx.x; i < ph.items && ok; i += gridDim.x) attn_item(ph, i);
      // S blocks with o: one item per CTA (items ≤ grid), QG = 1 (the cache head is the head).
      if (ph.wo && blockIdx.x < ph.items && ok) attn_o_tail(ph, blockIdx.x / ph.splits, blockIdx.x % ph.splits);
    } else {
      if (!ph.wo) {
        for (int i = blockIdx.x; i < ph.items && ok; i += gridDim.x) gla_item(ph, i);
      } else if (blockIdx.x < ph.items) {  // L blocks with o: items are heads × splits, one per CTA
        const int h = blockIdx.x / ph.splits, s = blockIdx.x % ph.splits;
        gla_item(ph, h, s);
        if (ok) mixer_o_tail(ph, h, s, true);
      }
    }
  }

  // Armed launch: wait for the host's token (see Plan::host_gate).  True when
  // the step goes ahead (its token in sm.cur_id); false when it was
  // cancelled, which every CTA learns before any state is touched.
  __device__ bool gate() {
    const unsigned gtag = (unsigned)(P.gate_seq & 0x7fffffffu);
    if (tid == 0) {
      unsigned id = 0xffffffffu;
      if (blockIdx.x == 0) {
        const unsigned long long t0 = now_ns();
        for (unsigned it = 0;; it++) {
          const unsigned long long w = ld_sys_u64(P.host_gate);
          if ((unsigned)(w >> 32) == (unsigned)P.gate_seq) {
            id = (unsigned)w;
            break;
          }
          if ((it & 15) == 15 && now_ns() - t0 > kArmNs) break;  // no token in time: cancel
        }
        st_relaxed_u64(P.next_tagged, ((unsigned long long)gtag << 32) | id);
      }
      // Every CTA takes the decision from CTA 0 (bounded like every other wait;
      // CTA 0's own wait is far shorter).
      Spin sp;
      unsigned long long w = 0;
      bool got = true;
      while (((w = ld_relaxed_u64(P.next_tagged)) >> 32) != gtag)
        if (!sp.again(P.err)) {
          got = false;
          break;
        }
      id = got ? (unsigned)w : 0xffffffffu;
      if (id != 0xffffffffu) sm.cur_id = id;
      sm.flag = id != 0xffffffffu ? 1 : 2;
      st_release_cta_shared(&sm.gate, id != 0xffffffffu ? 1u : 2u);  // the producer may go on, or drain
    }
    consumers_sync();
    const bool go = sm.flag == 1;
    consumers_sync();  // sm.flag is reused by the step's waits
    if (tid == 0) sm.flag = 0;
    if (!go && blockIdx.x == 0 && tid == 0) {
      // Tell the host this launch ended without running its step.
      *(volatile unsigned long long*)(P.host_mbox + 2) = P.gate_seq;
      __threadfence_system();
    }
    return go;
  }

  __device__ void run() {
    if (tid < kDH / 2 && P.inv_freq) sm.inv_freq[tid] = __ldg(P.inv_freq + tid);
    if (tid == 0) sm.cur_id = P.host_id >= 0 ? (uint32_t)P.host_id : P.ids[0];
    if (P.host_gate && !gate()) return;  // an armed launch whose step was cancelled
    const int np = P.nphases;
    stage_phase(0, 0);
    stage_wait();
    consumers_sync();
    long long g = 0;  // phases run in this launch (descriptor buffer parity)
    for (int st = 0; st < P.nsteps && ok; st++) {
      if (st > 0) {
        // The previous step's arg-max is this step's token: tagged by its
        // logits phase once every CTA had finished that step.
        if (tid == 0) {
          const unsigned want = tag_of(np - 1);
          unsigned long long w = 0;
          Spin sp;
          while (((w = ld_relaxed_u64(P.next_tagged)) >> 32) != want)
            if (!sp.again(P.err)) {
              ok = false;
              break;
            }
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          sm.cur_id = (uint32_t)w;
          st_release_cta_shared(&sm.step_ok, (unsigned)st);  // the producer may read this step's caches
        }
        if (!all_ok()) return;
        pos++, ep++;
      }
      // Single steps (no zero point) zero the next set at their start: the
      // previous step ended with its launch.
      if (P.zero_phase < 0) zero_next_set();
      for (int p = 0; p < np && ok; p++, g++) {
        if (g > 0) {
          stamp(p > 0 ? p - 1 : np - 1, 1);
          stage_wait();  // phase p's descriptor, requested one phase ago
          if (!consumers_and(ok ? 1 : 0)) {
            ok = false;
            return;
          }
          if (P.all_sync || sm.ph[g & 1].sync) {
            grid_sync();
            if (!ok) return;
          }
        }
        // Past the zero point every CTA has finished the previous step.
        if (p == P.zero_phase + 1) zero_next_set();
        cur = p;
        stamp(p, 0);
        if (g + 1 < (long long)np * P.nsteps) stage_phase((int)((g + 1) & 1), (p + 1) % np);
        run_phase(sm.ph[g & 1]);
      }
    }
    consumers_sync();
    stamp(np - 1, 1);
    if (tid == 0 && ok) {
      // The last CTA to finish resets the barrier count for the next launch
      // and advances the step counter: every CTA has passed every barrier and
      // read the counter by then.
      __threadfence();
      unsigned prev = atomicAdd(P.bar + 1, 1u);
      if (prev == gridDim.x - 1) {
        atomicExch(P.bar, 0u);
        atomicExch(P.bar + 1, 0u);
        atomicExch(P.epoch, ep + 1u);
        if (P.host_mbox) {
          // Every CTA has finished the step (each fenced its writes before its
          // count above): hand the arg-max and the error word to the host.
          __threadfence();
          const unsigned am = *(const volatile unsigned*)P.argmax;
          const unsigned ew = (unsigned)ld_volatile(P.err);
          *(volatile unsigned long long*)(P.host_mbox + 1) = ((unsigned long long)ew << 32) | am;
          __threadfence_system();
          *(volatile unsigned long long*)P.host_mbox = P.host_seq;
        }
      }
    }
  }
};

template <bool GL, int WB>
__global__ void __launch_bounds__(kThreads, 1) k_decode_mega(const __grid_constant__ Plan P) {
  extern __shared__ __align__(1024) char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  char* ring = smem_raw + ((sizeof(Smem) + 1023) / 1024) * 1024;
  const long long pos = P.pos[0];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.flag = 0;
    sm.step_ok = 0;
    sm.gate = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerWarps * 32) {
    if (threadIdx.x == kConsumerWarps * 32) producer(P, sm, ring, pos);
    return;
  }
  Cons<GL, WB> c(P, sm, ring, pos, *P.epoch);
  c.run();
}

}  // namespace

size_t smem_bytes() { return ((sizeof(Smem) + 1023) / 1024) * 1024 + (size_t)kStages * kStageBytes; }
static_assert(((sizeof(Smem) + 1023) / 1024) * 1024 + (size_t)kStages * kStageBytes <= 227 * 1024,
              "decode kernel shared memory above the 227 KB an sm_100 CTA may use");

void prepare() {
  for (auto f : {k_decode_mega<false, 4>, k_decode_mega<true, 4>, k_decode_mega<false, 2>, k_decode_mega<true, 2>})
    SLM_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes()));
}

int blocks_per_sm() {
  int least = 1 << 30;
  for (auto f : {k_decode_mega<false, 4>, k_decode_mega<true, 4>, k_decode_mega<false, 2>, k_decode_mega<true, 2>}) {
    int a = 0;
    SLM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, f, kThreads, smem_bytes()));
    least = a < least ? a : least;
  }
  return least;
}

void launch(const Plan& plan, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool bf = plan.wbytes == 2;
  if (plan.global)
    SLM_CUDA(cudaLaunchKernelEx(&cfg, bf ? k_decode_mega<true, 2> : k_decode_mega<true, 4>, plan));
  else
    SLM_CUDA(cudaLaunchKernelEx(&cfg, bf ? k_decode_mega<false, 2> : k_decode_mega<false, 4>, plan));
}

}  // namespace mega
}  // namespace slm
