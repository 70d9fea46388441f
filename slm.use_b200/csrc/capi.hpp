// Internal definitions behind the opaque handles of include/slm_b200.h.
#pragma once

#include <cuda_runtime.h>

#include <new>
#include <string>

#include "../../include/slm_b200.h"
#include "common.cuh"

struct slm_ctx {
  int device = 0;
  int sms = 0;
  std::string name;
  cudaStream_t stream = nullptr;
  int* err = nullptr;           // device error word (bad ids, sampler limits); err[1]: the arg-max of
                                // the last persistent step on this context (that of `argmax_owner`)
  int* err_host = nullptr;      // pinned copy of it (read after a synchronisation)
  const void* argmax_owner = nullptr;  // session whose persistent step wrote err[1] last
  // Mapped pinned words a persistent step launched by slm_step writes when it
  // ends: [0] its sequence number, [1] its arg-max | error word << 32
  // (slm_sample polls them instead of a copy and a stream synchronisation).
  // [2]: the sequence number of an armed launch that ended without its step;
  // [8] (its own cache line): the host's gate word for an armed launch,
  // sequence << 32 | token (token 0xFFFFFFFF cancels).
  unsigned long long* mbox = nullptr;      // host address
  unsigned long long* mbox_dev = nullptr;  // device address of the same words
  unsigned long long mbox_seq = 0;         // last sequence number given to a launch
  // An armed launch (a persistent step queued before its token is known,
  // waiting on mbox[8]): any library call on the context other than the
  // owner's slm_step cancels it (Device's constructor).
  bool armed = false;
  unsigned long long armed_seq = 0;
  const void* armed_owner = nullptr;
  void* stage = nullptr;        // staging buffer for host arrays (ids, factors)
  size_t stage_bytes = 0;
  void* gemm_ws = nullptr;      // tensor-core GEMM workspace (grown on demand, outside captures)
  size_t gemm_ws_bytes = 0;
  unsigned long long gemm_ws_gen = 0;  // bumped whenever gemm_ws moves (graphs holding it must be re-captured)
  unsigned* merge_cnt = nullptr;  // attention slice counters of slm_op_attend (zero between launches)
  unsigned* gemv_cnt = nullptr;   // kGemvCounters row-block counters of the split GEMV (zero between launches)
  size_t merge_cnt_len = 0;
  // Live buffers and models of this context.  slm_ctx_free while some live
  // only marks the context closing; the last of them to be freed frees it
  // (callers whose finalisers run in any order, such as a garbage collector,
  // stay safe).
  int refs = 0;
  bool closing = false;
};

struct slm_buf {
  slm_ctx* ctx;
  float* ptr;
  size_t len;
};

extern "C" int slm_ctx_stream(slm_ctx* c, void** out);

namespace slm {

void set_error(const std::string& s);

// Makes the context's device current for the lifetime of the object.
struct Device {
  int prev;
  // Also cancels the context's armed launch, unless keep_armed.
  explicit Device(slm_ctx* c, bool keep_armed = false);
  ~Device();
};

// Cancels the context's armed launch, if any: one host write (the kernel ends
// without running its step).
void disarm(slm_ctx* c);

// Takes / drops a reference to a context (see slm_ctx::refs).
void ctx_retain(slm_ctx* c);
void ctx_release(slm_ctx* c);

void* dev_alloc(size_t bytes);
void dev_free(void* p);
void ensure(slm_buf* y, size_t n);
const float* view(const slm_buf* b, size_t off, size_t n, const char* what);
void* stage(slm_ctx* c, const void* host, size_t bytes);
// Sets a.ws/a.ws_bytes to the context's GEMM workspace, growing it if the
// tensor-core path needs more (never during a stream capture).
void gemm_workspace(slm_ctx* c, struct LinearArgs& a, bool capturing);

// Runs f, turning failures into a status code and the thread's error message.
template <class F>
int guard(F&& f) {
  try {
    f();
    set_error("");
    return SLM_OK;
  } catch (const Error& e) {
    set_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_error("host allocation failed");
    return SLM_ERR_NOMEM;
  } catch (const std::exception& e) {
    set_error(e.what());
    return SLM_ERR_INVALID;
  }
}

}  // namespace slm
