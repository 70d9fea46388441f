// Prefill attention on the tensor cores, head size 64: the slice pass of
// attention.cu for 128-query tiles with QKᵀ and P·V as tcgen05 MMAs
// (reference Ops::attend, src/ops.rs:218-227; CPU arithmetic
// src/cpu.rs:352-403).
//
// Precision.  Every fp32 operand x is split into a bf16 pair x = hi + lo
// (hi = bf16(x), lo = bf16(x − hi); |x − hi − lo| ≤ 2^-18 |x|) and each
// product is taken as hi·hi + hi·lo + lo·hi, accumulated in fp32 in tensor
// memory: three kind::f16 MMAs per k-step, the dropped lo·lo term below
// 2^-16 of the product.  The softmax itself (mask, max, exp, sums) stays in
// fp32 registers.
//
// One CTA = 128 queries of one head × one slice of their key range
// (grid (nsplit, ceil(m/128), heads)), 320 threads, one CTA per SM:
//  * warp 8 (one thread) fetches each 64-position tile's fp32 K and V rows
//    from the ring with bulk copies into one of four shared buffers, as soon
//    as the MMAs of the tile four back are done with it;
//  * warps 4–7 split each landed tile in place into the layout the MMA reads;
//  * warp 9 (one thread) issues the MMAs: QKᵀ two tiles ahead into two score
//    buffers, P·V accumulating into one output, all in tensor memory;
//  * warps 0–3 own one query row per thread (tensor-memory lane = row).  Each
//    writes its row of Q (split) into tensor memory once; per tile it reads
//    its row of scores, masks it to its window, runs the online softmax and
//    writes its row of P (split) into one of two tensor-memory buffers.  P is
//    taken against a reference max that trails the running max by at most
//    2^8, so the output in tensor memory is rescaled (read, scaled, written
//    back) only in the rare tiles where a row's max grows past that.
// Q and P are the A operands of their MMAs straight from tensor memory (one
// row per lane, two bf16 of K per 32-bit column): the tensor core reads only
// K and V from shared memory.  K/V tiles are [key][dh] bf16 rows of 128 bytes
// in the 128-byte swizzled layout (8-key atoms of 1024 bytes, the 16-byte
// chunk c of key r at chunk c ^ (r % 8)): K is the K-major B operand of QKᵀ,
// V the MN-major B operand of P·V (K = key), with no transposition.
// Partials have the layout of the other slice passes (acc[64], max, sum per
// (slice, query, head)) and are merged by the same combine.
//
// Every wait is bounded (2 s): past it the CTA sets bit 32 of the context's
// error word, stops, waits (bounded) for the MMAs it issued, frees its
// tensor memory and returns.
#include <cuda_bf16.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "window.cuh"

namespace slm {

namespace {

constexpr int TQ = 128, TK = 64, TDH = 64;
constexpr uint32_t kHalf = 8192;           // one [64][64] bf16 tile
constexpr int kBufs = 4;                   // K/V tile buffers
constexpr uint32_t kKV = 0;                // buffers of Kh, Kl, Vh, Vl
constexpr uint32_t kKVBuf = 4 * kHalf;
constexpr uint32_t kBars = kKV + kBufs * kKVBuf;  // mbarriers, tensor-memory address, abort flag
constexpr size_t kTcSmem = kBars + 192 + 1024;     // + slack to align the base to 1024
// Tensor-memory columns: two score buffers, the output, Q split (bf16 pairs,
// two per column), two buffers of P split.
constexpr uint32_t kColS = 0, kColO = 128, kColQ = 192, kColP = 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kLazy = 8.0f;              // rescale a row's output only when its max rises by more (log2 units)
constexpr unsigned long long kTcWaitNs = 2000000000ull;

// kind::f16 instruction descriptors: bf16 A and B, fp32 D, M = 128, N = 64;
// A K-major, B K-major (QKᵀ) or MN-major (P·V, bit 16).
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(64 >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescO = kIdescS | (1u << 16);
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long tc_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Byte offset of the 16-byte chunk c (elements 8c .. 8c + 7) of row r of a
// [64][64] bf16 tile in the 128-byte swizzled layout: rows of 128 bytes, 8-row
// atoms of 1024 bytes, chunk c of row r stored at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Shared-memory matrix descriptor, 128-byte swizzle: start address, leading
// and stride byte offsets, descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t mdesc(uint32_t a, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// An MMA with A in tensor memory (one row per lane, two bf16 of K per column).
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// d (+)= ah·bh + ah·bl + al·bh over K = 64 in four k-steps of 16, A in tensor
// memory at columns ah, al (8 columns a step); B from a swizzled [key][dh]
// tile: K-major for QKᵀ (a step is 32 bytes along the 128-byte rows; 8-key
// atoms 1024 bytes apart) or MN-major for P·V (a step is two 8-key atoms,
// 2048 bytes; the 64 dims are one atom wide, so the leading offset is unused).
template <bool kBmn>
__device__ __forceinline__ void umma3t(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl,
                                       bool accumulate = false) {
  constexpr uint32_t idesc = kBmn ? kIdescO : kIdescS;
  constexpr uint32_t bstep = kBmn ? 2048 : 32, blbo = kBmn ? 8192 : 16, bsbo = 1024;
#pragma unroll
  for (int k = 0; k < 4; k++) umma_ts(d, ah + 8 * k, mdesc(bh + bstep * k, blbo, bsbo), idesc, accumulate || k > 0);
#pragma unroll
  for (int k = 0; k < 4; k++) umma_ts(d, ah + 8 * k, mdesc(bl + bstep * k, blbo, bsbo), idesc, 1);
#pragma unroll
  for (int k = 0; k < 4; k++) umma_ts(d, al + 8 * k, mdesc(bh + bstep * k, blbo, bsbo), idesc, 1);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void bar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}

// Bounded wait on an mbarrier phase.  False when the CTA has stopped (the
// flag another thread set) or the wait expired (then this thread sets it).
__device__ bool tc_wait(uint64_t* b, unsigned parity, volatile int* abort, int* err) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = tc_now();
  for (unsigned it = 1;; it++) {
    if (bar_try(b, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort) return false;
      if (tc_now() - t0 > kTcWaitNs) {
        *abort = 1;
        if (err) atomicOr(err, 32);
        return false;
      }
    }
  }
}

// 32 columns of this warp's 32 lanes (one row per thread), waited for.
__device__ __forceinline__ void tmem_ld32(uint32_t a, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Store 32 columns of this warp's lanes, waited for.
__device__ __forceinline__ void tmem_st32(uint32_t a, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(a),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

// Store 32 columns of 32-bit words (bf16 pairs) for this warp's lanes, waited for.
__device__ __forceinline__ void tmem_st32u(uint32_t a, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(a),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// 64 floats as 32 bf16 pairs of high parts and 32 of low parts.
__device__ __forceinline__ void split64(const float* x, uint32_t* hi, uint32_t* lo) {
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 af = __bfloat1622float2(a);
    const __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * i] - af.x, x[2 * i + 1] - af.y);
    hi[i] = *reinterpret_cast<const uint32_t*>(&a);
    lo[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
}

// Eight floats as 16 bytes of bf16 high parts and 16 bytes of low parts
// (pairs converted together).
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 af = __bfloat1622float2(a);
    const __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * i] - af.x, x[2 * i + 1] - af.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&a);
    l[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void st16(char* base, uint32_t off, uint4 v) {
  *reinterpret_cast<uint4*>(base + off) = v;
}

// One bar.sync over four warps (barrier 1: warps 0–3, 2: warps 4–7) that
// also ORs a flag across them.
template <int kBar>
__device__ __forceinline__ bool warps4_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kBar)
      : "memory");
  return r != 0;
}

// Fetch one tile's fp32 K and V rows (positions base .. min(base + 64, end)
// - 1, ring slots from slot0, wrapping at cap) into a tile buffer as
// [key][dh] rows (K at 0, V at 16 KB) with bulk copies completing on `bar`.
__device__ __forceinline__ void fetch_tile(char* buf, uint64_t* bar, const float* Kb, const float* Vb, long long base,
                                           long long end, long long slot0, long long cap) {
  const int rows = (int)(end - base < TK ? end - base : TK);
  bar_expect_tx(bar, 2u * rows * TDH * sizeof(float));
  long long sl = slot0;
  for (int r = 0; r < rows;) {
    const int n = (int)(cap - sl < rows - r ? cap - sl : rows - r);
    const unsigned bytes = (unsigned)n * TDH * sizeof(float);
    bulk_g2s(buf + (size_t)r * TDH * sizeof(float), Kb + (size_t)sl * TDH, bytes, bar);
    bulk_g2s(buf + 2 * kHalf + (size_t)r * TDH * sizeof(float), Vb + (size_t)sl * TDH, bytes, bar);
    r += n;
    sl = 0;
  }
}

// Split a landed tile in place into the MMA layout (Kh, Kl, Vh, Vl at 0, 8,
// 16, 24 KB; rows at or past `end` as zeros).  Loader thread lt (0..127)
// takes, for e = lt + 128 i (i < 4), key e / 8 and dims 8·(e % 8) .. + 7 of K
// and of V: eight lanes read one fp32 row and write the eight swizzled chunks
// of its bf16 rows, both without bank conflicts; every loader reads before
// any writes (barrier 2).  False when the CTA has stopped.
__device__ __forceinline__ bool split_tile(char* buf, long long base, long long end, int lt, bool ok,
                                           volatile int* abort) {
  float4 ka[4][2], va[4][2];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int e = lt + 128 * i, key = e >> 3, c = 8 * (e & 7);
    if (ok && base + key < end) {
      const float4* ks = reinterpret_cast<const float4*>(buf + (size_t)key * TDH * sizeof(float) + c * 4);
      const float4* vs = reinterpret_cast<const float4*>(buf + 2 * kHalf + (size_t)key * TDH * sizeof(float) + c * 4);
      ka[i][0] = ks[0];
      ka[i][1] = ks[1];
      va[i][0] = vs[0];
      va[i][1] = vs[1];
    } else {
      ka[i][0] = ka[i][1] = va[i][0] = va[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncwarp();  // bar.red is warp-aligned: thread 128 may come from its own waits
  if (warps4_any<2>(!ok || *abort)) return false;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int e = lt + 128 * i, key = e >> 3;
    const uint32_t off = sw_off(key, e & 7);
    uint4 hi, lo;
    const float xk[8] = {ka[i][0].x, ka[i][0].y, ka[i][0].z, ka[i][0].w,
                         ka[i][1].x, ka[i][1].y, ka[i][1].z, ka[i][1].w};
    split8(xk, hi, lo);
    st16(buf, off, hi);
    st16(buf + kHalf, off, lo);
    const float xv[8] = {va[i][0].x, va[i][0].y, va[i][0].z, va[i][0].w,
                         va[i][1].x, va[i][1].y, va[i][1].z, va[i][1].w};
    split8(xv, hi, lo);
    st16(buf + 2 * kHalf, off, hi);
    st16(buf + 3 * kHalf, off, lo);
  }
  return true;
}

__global__ void __launch_bounds__(320, 1)
    k_attn_tc(const float* __restrict__ q, int ldq, const float* __restrict__ K, const float* __restrict__ V,
              AttnGeom g, const long long* __restrict__ pos_ptr, int nsplit, float* __restrict__ part) {
  extern __shared__ uint8_t tc_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kBars);
  uint64_t* kv_full = bars;           // [kBufs]: the 128 loader threads stored the tile
  uint64_t* kv_empty = bars + kBufs;  // [kBufs]: the tile's MMAs are done with the buffer
  uint64_t* s_done = bars + 2 * kBufs;  // [2]: scores of tile j in score buffer j % 2
  uint64_t* o_done = s_done + 2;        // [2]: P·V of tile j (P buffer j % 2) folded into the output
  uint64_t* fin = s_done + 4;           // drain after a stop
  uint64_t* landed = fin + 1;           // [kBufs]: a tile's fp32 rows arrived (bulk copies)
  uint64_t* p_full = landed + kBufs;    // [2]: the 128 rows wrote P of tile j (P buffer j % 2)
  uint64_t* q_full = p_full + 2;        // the 128 rows wrote Q
  uint32_t* tmem_word = reinterpret_cast<uint32_t*>(sm + kBars + 160);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + kBars + 164);

  const int s = blockIdx.x, i0 = blockIdx.y * TQ, h = blockIdx.z, t = threadIdx.x, warp = t >> 5;
  const long long pos = pos_ptr ? pos_ptr[0] : g.pos0;
  const int kvh = h / (g.heads / g.key_heads);
  const float* Kb = K + (size_t)kvh * g.cap * TDH;
  const float* Vb = V + (size_t)kvh * g.cap * TDH;
  const int ilast = min(i0 + TQ, g.m) - 1;
  const Range r0 = visible(pos + i0, g.reach, g.gap), r1 = visible(pos + ilast, g.reach, g.gap);
  const long long ulo = r0.lo, uhi = max(r1.hi, r0.hi);
  const long long count = uhi - ulo, chunk = (count + nsplit - 1) / nsplit;
  const long long start = ulo + (long long)s * chunk, end = min(uhi, start + chunk);
  const int ntiles = start < end ? (int)((end - start + TK - 1) / TK) : 0;
  const int i = i0 + t;  // the query row of threads 0..127

  if (ntiles == 0) {  // an empty slice: the partial of a query that sees nothing
    if (t < TQ && i < g.m) {
      float* out = part + (((size_t)s * g.m + i) * g.heads + h) * (TDH + 2);
      for (int e = 0; e < TDH; e++) out[e] = 0.0f;
      out[TDH] = -INFINITY;
      out[TDH + 1] = 0.0f;
    }
    return;
  }

  // Thread 256 (the fetcher) initialises the barriers and starts the first
  // kBufs tiles' copies at once; tile j goes into buffer j % kBufs, the later
  // ones once the P·V of tile j - kBufs is done (below).
  long long fslot = start % g.cap;
  int fetched = 0;
  auto fetch = [&](int b) {
    fetch_tile(sm + kKV + b * kKVBuf, &landed[b], Kb, Vb, start + (long long)fetched * TK, end, fslot, g.cap);
    fslot = (fslot + TK) % g.cap;
    fetched++;
  };
  if (t == 256) {
    for (int b = 0; b < kBufs; b++) {
      bar_init(&kv_full[b], 128);
      bar_init(&kv_empty[b], 1);
      bar_init(&landed[b], 1);
    }
    for (int b = 0; b < 2; b++) {
      bar_init(&s_done[b], 1);
      bar_init(&o_done[b], 1);
      bar_init(&p_full[b], 128);
    }
    bar_init(q_full, 128);
    bar_init(fin, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int b = 0; b < kBufs && b < ntiles; b++) fetch(b);
  }
  __syncwarp();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_word)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_async_smem();
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_word;
  const uint32_t tO = tmem + kColO;

  if (warp == 9) {  // MMA issuer (thread 288)
    if (t == 288) {
      const uint32_t qh = tmem + kColQ, ql = tmem + kColQ + 32;
      bool ok = tc_wait(q_full, 0, abort, g.err);
      for (int j = 0; j < 2 && j < ntiles && ok; j++) {  // the scores of the first two tiles
        ok = tc_wait(&kv_full[j], 0, abort, g.err);
        if (ok) {
          tc_after();
          const uint32_t kb = saddr(sm + kKV + j * kKVBuf);
          umma3t<false>(tmem + kColS + 64 * j, qh, ql, kb, kb + kHalf);
          umma_commit(&s_done[j]);
        }
      }
      for (int j = 0, b = 0; ok && j < ntiles; j++) {
        const int sb = j & 1;
        if (!tc_wait(&p_full[sb], (j >> 1) & 1, abort, g.err)) break;
        tc_after();
        const uint32_t kb = saddr(sm + kKV + b * kKVBuf), pa = tmem + kColP + 64 * sb;
        umma3t<true>(tO, pa, pa + 32, kb + 2 * kHalf, kb + 3 * kHalf, j > 0);
        umma_commit(&o_done[sb]);
        umma_commit(&kv_empty[b]);
        // The scores of tile j + 2 into this score buffer (its rows have read it).
        const int b2 = b + 2 >= kBufs ? b + 2 - kBufs : b + 2;
        if (j + 2 < ntiles) {
          if (!tc_wait(&kv_full[b2], ((j + 2) / kBufs) & 1, abort, g.err)) break;
          tc_after();
          const uint32_t kn = saddr(sm + kKV + b2 * kKVBuf);
          umma3t<false>(tmem + kColS + 64 * sb, qh, ql, kn, kn + kHalf);
          umma_commit(&s_done[sb]);
        }
        b = b + 1 == kBufs ? 0 : b + 1;
      }
      // After a stop, every MMA issued completes before the tensor memory is freed.
      if (*abort) {
        umma_commit(fin);
        const unsigned long long t0 = tc_now();
        while (!bar_try(fin, 0) && tc_now() - t0 < kTcWaitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 8) {  // fetcher
    if (t == 256) {
      for (int b = fetched % kBufs; fetched < ntiles; b = b + 1 == kBufs ? 0 : b + 1)
        if (!tc_wait(&kv_empty[b], ((fetched / kBufs) - 1) & 1, abort, g.err)) break;
        else fetch(b);
      // The last copy into each buffer lands before the CTA exits (earlier
      // ones have: their tiles were split before the buffer was reused).
      for (int j = fetched > kBufs ? fetched - kBufs : 0; j < fetched; j++) {
        const unsigned long long t0 = tc_now();
        while (!bar_try(&landed[j % kBufs], (j / kBufs) & 1) && tc_now() - t0 < kTcWaitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {  // splitters
    const int lt = t - 128;
    for (int j = 0, b = 0; j < ntiles; j++) {
      const bool ok = tc_wait(&landed[b], (j / kBufs) & 1, abort, g.err);
      if (!split_tile(sm + kKV + b * kKVBuf, start + (long long)j * TK, end, lt, ok, abort)) break;
      fence_async_smem();
      bar_arrive(&kv_full[b]);
      b = b + 1 == kBufs ? 0 : b + 1;
    }
  } else {  // rows
    long long qlo = 0, qhi = 0;
    if (i < g.m) {
      const Range rr = visible(pos + i, g.reach, g.gap);
      qlo = rr.lo;
      qhi = rr.hi;
    }
    // The row's softmax state in log2 units: mu is the reference its P values
    // are taken against (within kLazy of the running max), l their sum.
    float mu = -INFINITY, l = 0.0f;
    const uint32_t lanes = tmem + ((uint32_t)(warp * 32) << 16);
    {  // this row of Q, split, into tensor memory (rows past m as zeros)
      float x[TDH];
      const float* src = q + (size_t)i * ldq + (size_t)h * TDH;
#pragma unroll
      for (int c = 0; c < TDH; c += 4) {
        const float4 v = i < g.m ? *reinterpret_cast<const float4*>(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        x[c] = v.x, x[c + 1] = v.y, x[c + 2] = v.z, x[c + 3] = v.w;
      }
      uint32_t hi[32], lo[32];
      split64(x, hi, lo);
      tmem_st32u(lanes + kColQ, hi);
      tmem_st32u(lanes + kColQ + 32, lo);
      tc_before();
      bar_arrive(q_full);
    }
    const float k2 = g.scale * kLog2e;  // scores in log2 units: exp(x) = exp2(x · log2 e)
    for (int j = 0; j < ntiles; j++) {
      const long long base = start + (long long)j * TK;
      const int sb = j & 1;
      bool ok = tc_wait(&s_done[sb], (j >> 1) & 1, abort, g.err);
      // P buffer sb was last read by the P·V of tile j - 2.
      if (ok && j >= 2) ok = tc_wait(&o_done[sb], ((j - 2) >> 1) & 1, abort, g.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_after();
      float sc[TK];
      tmem_ld32(lanes + kColS + 64 * sb, sc);
      tmem_ld32(lanes + kColS + 64 * sb + 32, sc + 32);
      // This row's visible columns of the tile: [c0, c1).
      const long long lo_p = qlo > base ? qlo : base, hi_p = min(min(qhi, end), base + TK);
      const long long d0 = lo_p - base;
      const int c0 = d0 < TK ? (int)d0 : TK, c1 = hi_p > lo_p ? (int)(hi_p - base) : c0;
      if (c0 == 0 && c1 == TK) {
#pragma unroll
        for (int c = 0; c < TK; c++) sc[c] *= k2;
      } else {
#pragma unroll
        for (int c = 0; c < TK; c++) sc[c] = c >= c0 && c < c1 ? sc[c] * k2 : -INFINITY;
      }
      float mq[4] = {sc[0], sc[1], sc[2], sc[3]};
#pragma unroll
      for (int c = 4; c < TK; c++) mq[c & 3] = fmaxf(mq[c & 3], sc[c]);
      const float T = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      // A new reference when the tile's max exceeds the old one by more than
      // kLazy; the output so far (in tensor memory) and l are then scaled by
      // 2^(old − new) (by 0 when there was none: both are 0).
      float f = 1.0f;
      bool grow = false;
      if (T > mu + kLazy) {
        grow = mu != -INFINITY;
        f = exp2f(mu - T);
        mu = T;
      }
      if (__any_sync(0xffffffffu, grow)) {
        // The output holds the P·V of tiles 0 .. j - 1: wait for the last.
        const bool ok3 = tc_wait(&o_done[sb ^ 1], ((j - 1) >> 1) & 1, abort, g.err);
        __syncwarp();
        if (__all_sync(0xffffffffu, ok3)) {
          tc_after();
          float ov[32];
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            tmem_ld32(lanes + kColO + 32 * hh, ov);
#pragma unroll
            for (int e = 0; e < 32; e++) ov[e] *= f;
            tmem_st32(lanes + kColO + 32 * hh, ov);
          }
        }
      }
      const float ms = mu == -INFINITY ? 0.0f : mu;  // a row that has seen nothing: every p is 0
      float rq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < TK; c++) {
        sc[c] = exp2f(sc[c] - ms);
        rq[c & 3] += sc[c];
      }
      l = l * f + ((rq[0] + rq[1]) + (rq[2] + rq[3]));
      {
        uint32_t hi[32], lo[32];
        split64(sc, hi, lo);
        tmem_st32u(lanes + kColP + 64 * sb, hi);
        tmem_st32u(lanes + kColP + 64 * sb + 32, lo);
      }
      tc_before();
      bar_arrive(&p_full[sb]);
    }
    // The output: wait for the last two tiles' P·V (each barrier is at most
    // one phase short of them), read this row, and stage it in shared memory
    // (the tile buffers, free now) so the partial rows go out coalesced.
    bool ok = true;
    for (int j = ntiles - 2; j < ntiles; j++)
      if (j >= 0 && ok) ok = tc_wait(&o_done[j & 1], (j >> 1) & 1, abort, g.err);
    __syncwarp();
    float o[TDH];
    if (__all_sync(0xffffffffu, ok)) {
      tc_after();
      tmem_ld32(lanes + kColO, o);
      tmem_ld32(lanes + kColO + 32, o + 32);
    } else {
#pragma unroll
      for (int e = 0; e < TDH; e++) o[e] = 0.0f;
    }
    float2* row = reinterpret_cast<float2*>(sm + kKV + (size_t)t * (TDH + 2) * sizeof(float));
#pragma unroll
    for (int e = 0; e < TDH / 2; e++) row[e] = make_float2(o[2 * e], o[2 * e + 1]);
    row[TDH / 2] = make_float2(mu == -INFINITY ? mu : mu / kLog2e, l);  // max back to natural-log units
    __syncwarp();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const int lane = t & 31;
    for (int r = warp; r < TQ && i0 + r < g.m; r += 4) {
      const float* src = reinterpret_cast<const float*>(sm + kKV + (size_t)r * (TDH + 2) * sizeof(float));
      float* out = part + (((size_t)s * g.m + i0 + r) * g.heads + h) * (TDH + 2);
      out[lane] = src[lane];
      out[32 + lane] = src[32 + lane];
      if (lane < 2) out[64 + lane] = src[64 + lane];
    }
  }

  tc_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

bool attention_tc_on() {
  static const bool on = [] {
    const char* e = std::getenv("SLM_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

void attention_tc(const float* q, int ldq, const float* K, const float* V, const AttnGeom& g,
                  const long long* pos_ptr, int nsplit, float* part, cudaStream_t st) {
  // The shared-memory limit is a per-device function attribute: set it on
  // the first launch on each device (a process may drive several).
  constexpr int kDevices = 64;
  static std::once_flag once[kDevices];
  int dev = 0;
  SLM_CUDA(cudaGetDevice(&dev));
  auto set = [] {
    SLM_CUDA(cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
  };
  if (dev >= 0 && dev < kDevices)
    std::call_once(once[dev], set);
  else
    set();
  k_attn_tc<<<dim3(nsplit, (g.m + TQ - 1) / TQ, g.heads), 320, kTcSmem, st>>>(q, ldq, K, V, g, pos_ptr, nsplit,
                                                                              part);
  SLM_LAUNCHED("k_attn_tc");
}

}  // namespace slm
