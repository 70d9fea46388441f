"""The allocation-free attention entry point (slm_op_attend_noalloc) against
the regular one (slm_op_attend), through the C ABI, on two calls in a row.

It serves callers that cannot call cudaMalloc (it may synchronise the device,
or the process's device memory is reserved by its own allocator): the scratch
lives in a fixed per-device array instead.  The test also checks that the
device's free memory is the same before and after the calls.  Collected last
so that a failure here leaves every other test already run."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOM = (1 << 20) - 64  # floats of the fixed scratch available to partials

CASES = [
    # pos, m, reach, gap, cap, heads, key_heads, dh
    (4200, 1, 4096, 0, 4352, 12, 12, 64),     # decode over a full, wrapped window
    (3840, 256, 4096, 0, 4352, 12, 12, 64),   # a prefill chunk (splits trimmed to fit, see below)
    (9000, 3, None, 4096, 16384, 12, 4, 64),  # global layer: unbounded reach, far gap, GQA
    (600, 496, 1024, 0, 1280, 32, 8, 64),     # the largest accepted size: 1,047,552 floats of partials
]


def _need(case):
    _, m, _, _, _, heads, _, dh = case
    return m * heads * (dh + 2)


def test_cases_cover_the_trimmed_and_the_largest_sizes():
    # The chunk case: the library's split rule (two 64-query CTAs per SM over
    # 148 SMs) asks for 6 splits; only 5 fit the array, so the call trims.
    assert 6 * _need(CASES[1]) > ROOM >= 5 * _need(CASES[1])
    assert ROOM - 1024 < _need(CASES[3]) <= ROOM


def _inputs(case, seed):
    pos, m, reach, gap, cap, heads, kh, dh = case
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(m * heads * dh).astype(np.float32)
    k = rng.standard_normal(kh * cap * dh).astype(np.float32)
    v = rng.standard_normal(kh * cap * dh).astype(np.float32)
    geo = dict(pos=pos, m=m, reach=reach, gap=gap, cap=cap, heads=heads, key_heads=kh, dh=dh,
               scale=1.0 / math.sqrt(dh))
    return q, k, v, geo


def _free_bytes():
    import torch
    torch.cuda.synchronize(0)
    return torch.cuda.mem_get_info(0)[0]


@pytest.mark.parametrize("first,second", [(0, 1), (1, 2), (2, 3), (3, 0)])
def test_noalloc_attend_matches_attend_twice_in_a_row(slm, first, second):
    ctx = slm.Context(0)
    ops = slm.Ops(ctx)
    runs = []
    for i, case in enumerate((CASES[first], CASES[second])):
        q, k, v, geo = _inputs(case, seed=10 * first + i)
        qb, kb, vb = ops.upload(q), ops.upload(k), ops.upload(v)
        n = geo["m"] * geo["heads"] * geo["dh"]
        want, scores = ops.zeros(n), ops.zeros(1)
        ops.attend(want, scores, qb, kb, vb, **geo)
        runs.append((geo, qb, kb, vb, ops.zeros(n), want, n))
    # One call of each shape first: it loads the kernels it launches.
    for geo, qb, kb, vb, got, _, _ in runs:
        slm.attend_noalloc(ctx, got, qb, kb, vb, **geo)
    before = _free_bytes()
    # The two calls in a row, each overwriting what the previous one left in
    # the shared scratch.
    for geo, qb, kb, vb, got, _, _ in runs:
        slm.attend_noalloc(ctx, got, qb, kb, vb, **geo)
    assert _free_bytes() == before, "attend_noalloc changed the device's free memory"
    for geo, qb, kb, vb, got, want, n in runs:
        np.testing.assert_allclose(got.read(n), want.read(n), atol=2e-5, rtol=1e-4)


def test_noalloc_attend_rejects_work_beyond_its_scratch(slm):
    ctx = slm.Context(0)
    ops = slm.Ops(ctx)
    buf = ops.zeros(16)
    # m·heads·(dh + 2) = 4096·8·66 floats: above the fixed 4 MiB array.
    with pytest.raises(slm.SlmError) as e:
        slm.attend_noalloc(ctx, buf, buf, buf, buf, pos=0, m=4096, reach=8192, gap=0, cap=8192, heads=8,
                           key_heads=8, dh=64, scale=0.125)
    assert "scratch" in str(e.value)
