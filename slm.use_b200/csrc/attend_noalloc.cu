// Softmax attention (the Ops::attend operation) for callers that must not
// allocate device memory.
//
// slm_op_attend grows a caller-visible scratch buffer with cudaMalloc when it
// is too small, and cudaMalloc/cudaFree may synchronise the whole device.
// Some callers cannot accept that: code that runs between kernels of a
// latency-critical decode loop, or a process whose device memory is fully
// reserved up front by its own allocator (a serving framework's memory pool)
// and whose budget a stray allocation would break.  This entry point takes
// raw device pointers for its inputs and output and keeps its scratch (the
// per-split softmax partials and the query position) in one file-scope
// __device__ array, so it calls no allocating routine at all.
//
// The array is kNoAllocFloats floats (4 MiB) per device.  Every GPU that loads
// this library holds it until the process exits.  All calls on a device share
// it and each call overwrites what the previous one left; nothing in it has to
// start at zero (every partial a call reads, that call wrote first).  Calls
// whose work overlaps on the GPU (different streams or contexts on one device)
// race on the array and must be serialised by the caller.
#include <mutex>
#include <string>
#include <vector>

#include "capi.hpp"
#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocFloats = size_t(1) << 20;  // 4 MiB
constexpr size_t kPartOffset = 64;                  // floats before the partials (256-byte aligned)

static __device__ __align__(256) float g_attend_scratch[kNoAllocFloats];

// Device address of g_attend_scratch, per device.  In host code the symbol
// is only a host-side stand-in; a kernel must be given this address instead.
// It is looked up once per device and kept: valid while the device's primary
// context lives (a cudaDeviceReset would make it stale).
std::mutex g_mutex;
std::vector<float*> g_scratch;

float* scratch_on(int device) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if ((int)g_scratch.size() <= device) g_scratch.resize(device + 1, nullptr);
  if (!g_scratch[device]) {
    float* p = nullptr;
    slm::check_cuda(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_attend_scratch),
                    "cudaGetSymbolAddress(g_attend_scratch)");
    g_scratch[device] = p;
  }
  return g_scratch[device];
}

__global__ void k_put_pos(long long* dst, long long pos) { dst[0] = pos; }

}  // namespace

using namespace slm;

extern "C" int slm_op_attend_noalloc(slm_ctx* c, float* y, const float* q, const float* k, const float* v,
                                     const slm_attn* at) {
  return guard([&] {
    SLM_REQUIRE(c && at && y && q && k && v, "attend_noalloc: null argument");
    SLM_REQUIRE(at->dh <= 256, "attend_noalloc: head size above 256");
    SLM_REQUIRE(at->key_heads > 0 && at->heads % at->key_heads == 0 && at->cap > 0 && at->reach > 0,
                "attend_noalloc: bad geometry");
    SLM_REQUIRE(at->m < (1u << 31) && at->heads < (1u << 31), "attend_noalloc: shape too large");
    // The kernels read q, k and v in 16-byte vectors.
    SLM_REQUIRE((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) == 0,
                "attend_noalloc: q, k and v must be 16-byte aligned");
    if (!at->m) return;
    AttnGeom g;
    g.m = (int)at->m;
    g.reach = at->reach == SIZE_MAX ? 0 : (long long)at->reach;
    g.gap = (long long)at->gap, g.cap = (long long)at->cap;
    g.heads = (int)at->heads, g.key_heads = (int)at->key_heads, g.dh = (int)at->dh, g.scale = at->scale;
    g.err = c->err;
    // Span of positions any query sees (Attn::span, reference src/ops.rs:54-59).
    long long base = g.reach == 0 ? 0 : ((long long)at->pos > g.reach - 1 ? (long long)at->pos - (g.reach - 1) : 0);
    long long span = (long long)(at->pos + at->m) - g.gap - base;
    int nsplit = attn_splits(g, span < 1 ? 1 : span);
    const size_t room = kNoAllocFloats - kPartOffset;
    while (nsplit > 1 && attn_part_floats(g, nsplit) > room) nsplit--;
    const size_t need = attn_part_floats(g, 1);
    if (attn_part_floats(g, nsplit) > room)
      fail(SLM_ERR_INVALID, "attend_noalloc: m·heads·(dh+2) = " + std::to_string(need) +
                                " floats exceeds the " + std::to_string(room) +
                                " floats of its fixed device scratch; use slm_op_attend");
    Device dev(c);
    float* scratch = scratch_on(c->device);
    auto* pos_dev = reinterpret_cast<long long*>(scratch);
    k_put_pos<<<1, 1, 0, c->stream>>>(pos_dev, (long long)at->pos);
    SLM_LAUNCHED("k_put_pos");
    const int ld = (int)(at->heads * at->dh);
    attention(q, ld, k, v, g, pos_dev, nsplit, scratch + kPartOffset, y, ld, c->stream);
  });
}
