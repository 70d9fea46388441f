"""The allocation-free attention entry point (slm_op_attend_noalloc) against
the regular one (slm_op_attend), through the C ABI, on two calls in a row.

It serves callers that cannot call cudaMalloc (it may synchronise the device,
or the process's device memory is reserved by its own allocator): the scratch
lives in a fixed per-device array instead.  Collected last so that a failure
here leaves every other test already run."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # pos, m, reach, gap, cap, heads, key_heads, dh
    (4200, 1, 4096, 0, 4352, 12, 12, 64),   # decode over a full, wrapped window
    (3840, 256, 4096, 0, 4352, 12, 12, 64),  # a prefill chunk
    (9000, 3, None, 4096, 16384, 12, 4, 64),  # global layer: unbounded reach, far gap, GQA
]


def _run_pair(slm, ctx, ops, case, seed):
    pos, m, reach, gap, cap, heads, kh, dh = case
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(m * heads * dh).astype(np.float32)
    k = rng.standard_normal(kh * cap * dh).astype(np.float32)
    v = rng.standard_normal(kh * cap * dh).astype(np.float32)
    qb, kb, vb = ops.upload(q), ops.upload(k), ops.upload(v)
    geo = dict(pos=pos, m=m, reach=reach, gap=gap, cap=cap, heads=heads, key_heads=kh, dh=dh,
               scale=1.0 / math.sqrt(dh))
    want, scores = ops.zeros(m * heads * dh), ops.zeros(1)
    ops.attend(want, scores, qb, kb, vb, **geo)
    got = ops.zeros(m * heads * dh)
    slm.attend_noalloc(ctx, got, qb, kb, vb, **geo)
    return got.read(m * heads * dh), want.read(m * heads * dh)


@pytest.mark.parametrize("first,second", [(0, 1), (1, 2), (2, 0)])
def test_noalloc_attend_matches_attend_twice_in_a_row(slm, first, second):
    ctx = slm.Context(0)
    ops = slm.Ops(ctx)
    for i, case in enumerate((CASES[first], CASES[second])):
        got, want = _run_pair(slm, ctx, ops, case, seed=10 * first + i)
        np.testing.assert_allclose(got, want, atol=2e-5, rtol=1e-4)


def test_noalloc_attend_rejects_work_beyond_its_scratch(slm):
    ctx = slm.Context(0)
    ops = slm.Ops(ctx)
    buf = ops.zeros(16)
    # m·heads·(dh + 2) = 4096·8·66 floats: above the fixed 4 MiB array.
    with pytest.raises(slm.SlmError) as e:
        slm.attend_noalloc(ctx, buf, buf, buf, buf, pos=0, m=4096, reach=8192, gap=0, cap=8192, heads=8,
                           key_heads=8, dh=64, scale=0.125)
    assert "scratch" in str(e.value)
