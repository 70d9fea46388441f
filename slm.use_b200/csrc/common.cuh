// Shared definitions of the B200 backend: error handling, launch helpers and
// small device utilities.  Everything here is sm_100a-only code.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "../../include/slm_b200.h"

namespace slm {

// Internal failure, turned into a status code at the C ABI boundary.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    int code = (e == cudaErrorMemoryAllocation) ? SLM_ERR_NOMEM : SLM_ERR_CUDA;
    fail(code, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

#define SLM_CUDA(call) ::slm::check_cuda((call), #call)
#define SLM_LAUNCHED(name) ::slm::check_cuda(cudaGetLastError(), name)
#define SLM_REQUIRE(cond, msg)                          \
  do {                                                  \
    if (!(cond)) ::slm::fail(SLM_ERR_INVALID, (msg));   \
  } while (0)

inline unsigned cdiv(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

// Epilogues of the linear kernels (what is done with each dot product).
enum Epi : int {
  EPI_STORE = 0,  // y = w·x
  EPI_ADD = 1,    // y = res + w·x  (res may be y itself: the residual update)
  EPI_SILU = 2,   // rows j and j + rows/2 pair up: y[j] = amp·gate/(1 + e^-gate)
};

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 16-byte load of data read once per launch (weights, caches):
// bypasses L1 allocation.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  acc = fmaf(a.w, b.w, acc);
  return acc;
}

// silu(g)·u, written as the reference writes it: u·g / (1 + e^-g).
__device__ __forceinline__ float silu_mul(float g, float u) { return u * g / (1.0f + expf(-g)); }

// Block-wide sum for blockDim.x a multiple of 32 (≤ 1024); `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

}  // namespace slm
