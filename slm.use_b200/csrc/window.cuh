// Window geometry of Ops::attend (reference src/ops.rs:31-66): the query at
// position p reads cached positions lo..hi-1 with lo = max(0, p - reach + 1)
// (reach 0 = unbounded) and hi = p + 1 - gap.
#pragma once

namespace slm {

struct Range {
  long long lo, hi;
};

__device__ __forceinline__ Range visible(long long p, long long reach, long long gap) {
  Range r;
  r.lo = (reach <= 0 || p < reach - 1) ? 0 : p - (reach - 1);
  r.hi = p + 1 - gap;
  if (r.hi < r.lo) r.hi = r.lo;
  return r;
}

}  // namespace slm
