"""Armed launches: after a greedy slm_sample the next persistent step is
launched at once and waits (bounded) for slm_step's token on a mapped word.
The tokens must be those of plain launches whatever the host does between
the calls: feed the token at once, pause past the launch's 20 ms bound (it
cancels itself and slm_step launches a plain step), call another library
function (which cancels it), or step another session of the same context.
"""
import time

import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    load_pkg()
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(syn.BASE, vocab_size=1000, d_model=128, n_heads=2, hidden=256, window=48, max_loops=4,
                     default_loops=3)
    return syn.write_model(tmp_path_factory.mktemp("arm"), cfg, seed=11)


def _twins(slm, model, seed):
    prompt = np.random.default_rng(seed).integers(0, 1000, 60)
    a, b = model.session(), model.session()
    a.feed(prompt)
    b.feed(prompt)
    assert a.mega and b.mega
    return a, b, int(np.argmax(a.logits()))


def _greedy_loop(slm, se, tok, n, between=None):
    greedy = slm.Sampling()
    out = []
    for i in range(n):
        se.step(tok)
        tok = se.sample(greedy)
        out.append(tok)
        if between:
            between(i)
    return out


def test_armed_steps_match_plain_decode(slm, ctx, small):
    model = slm.Model(ctx, small)
    a, b, tok = _twins(slm, model, 1)
    want = b.decode(tok, 30, slm.Sampling())
    got = _greedy_loop(slm, a, tok, 30)
    np.testing.assert_array_equal(got, want)
    assert a.pos == b.pos


def test_armed_step_that_ran_out_of_time_is_replaced(slm, ctx, small):
    model = slm.Model(ctx, small)
    a, b, tok = _twins(slm, model, 2)
    want = b.decode(tok, 12, slm.Sampling())
    got = _greedy_loop(slm, a, tok, 12, between=lambda i: time.sleep(0.05) if i % 3 == 1 else None)
    np.testing.assert_array_equal(got, want)
    assert a.pos == b.pos


def test_other_calls_cancel_the_armed_step(slm, ctx, small):
    model = slm.Model(ctx, small)
    a, b, tok = _twins(slm, model, 3)
    want = b.decode(tok, 10, slm.Sampling())
    seen = []
    got = _greedy_loop(slm, a, tok, 10, between=lambda i: seen.append(a.logits()) if i % 2 == 0 else None)
    np.testing.assert_array_equal(got, want)
    # The logits read between the calls are those of the step just taken.
    assert all(int(np.argmax(lg)) == int(t) for lg, t in zip(seen, got[0::2]))
    assert a.pos == b.pos


def test_interleaved_sessions_with_armed_steps(slm, ctx, small):
    model = slm.Model(ctx, small)
    a, a2, ta = _twins(slm, model, 4)
    b, b2, tb = _twins(slm, model, 5)
    want_a = a2.decode(ta, 12, slm.Sampling())
    want_b = b2.decode(tb, 12, slm.Sampling())
    greedy = slm.Sampling()
    got_a, got_b = [], []
    for _ in range(12):
        a.step(ta)
        ta = a.sample(greedy)
        b.step(tb)  # cancels a's armed step, then steps b
        tb = b.sample(greedy)
        got_a.append(ta)
        got_b.append(tb)
    np.testing.assert_array_equal(got_a, want_a)
    np.testing.assert_array_equal(got_b, want_b)
