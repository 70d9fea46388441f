"""Device sampling (src/sample.rs) against the oracle's pick on the same
logits, history and xorshift64* state: ids must be identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_reference_unit_cases(slm, ctx):
    S = slm.Sampling
    assert slm.pick(ctx, [0.0, 3.0, 1.0], S()) == 1
    assert slm.pick(ctx, [0.0, 3.0, 2.0], S(repeat_penalty=2.0, repeat_window=8), recent=[1]) == 2
    st = [slm.rng_seed(3)]
    for _ in range(50):
        assert slm.pick(ctx, [-9.0, 5.0, -9.0, 1.0], S(temperature=1.0, top_p=0.5), rng_state=st) == 1
    st = [slm.rng_seed(7)]
    for _ in range(50):
        assert slm.pick(ctx, [5.0, 4.0, -9.0, -9.0], S(temperature=1.0, top_k=2), rng_state=st) < 2


CASES = [
    dict(temperature=0.0),
    dict(temperature=0.0, repeat_penalty=1.1, repeat_window=256),
    dict(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=256),
    dict(temperature=1.0, top_k=40),
    dict(temperature=0.7, top_k=1),
    dict(temperature=1.0, top_p=0.9),
    dict(temperature=0.9, top_k=100, top_p=0.8),
    dict(temperature=1.3),
    dict(temperature=1.0, top_k=2048),
    dict(temperature=1.0, top_k=5000),
    dict(temperature=1.0, top_k=5000, top_p=0.9),
    dict(temperature=1.0, top_p=0.99),
]


@pytest.mark.parametrize("case", CASES)
def test_pick_matches_oracle(slm, ctx, oracle, case):
    rng = np.random.default_rng(11)
    s = slm.Sampling(**case)
    st_dev, st_ref = [slm.rng_seed(0)], [oracle.rng_new(0)]
    for trial in range(30):
        logits = (rng.standard_normal(32000) * 2.0).astype(np.float32)
        if trial % 5 == 0:
            logits[rng.integers(0, 32000, 50)] = logits.max()  # ties
        recent = rng.integers(0, 32000, 300).astype(np.uint32)
        got = slm.pick(ctx, logits, s, recent=recent, rng_state=st_dev)
        want = oracle.pick(logits, recent, rng_state=st_ref, **case)
        assert got == want, (case, trial)
        assert st_dev[0] == st_ref[0]


def test_decode_equals_step_and_sample(slm, ctx):
    from conftest import TINY
    model = slm.Model(ctx, TINY)
    s = slm.Sampling(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=16)
    prompt = np.array([5, 9, 14, 2, 77, 31], dtype=np.uint32)
    a, b = model.session(), model.session()
    a.feed(prompt)
    b.feed(prompt)
    st_a, st_b = [slm.rng_seed(0)], [slm.rng_seed(0)]
    hist = list(prompt)
    first = a.sample(s, hist, st_a)
    assert first == b.sample(s, hist, st_b)
    hist.append(first)
    out = a.decode(first, 30, s, recent=hist, rng_state=st_a)
    tok, want = first, []
    for _ in range(30):
        b.step(tok)
        tok = b.sample(s, hist, st_b)
        hist.append(tok)
        want.append(tok)
    np.testing.assert_array_equal(out, want)
    assert st_a == st_b
