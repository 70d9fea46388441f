"""Batched decode (slm_batch_*): n sessions stepped together, one token each.

Row i of a batch step must compute what slm_step computes on session i: the
same state updates (ring stores at its own position, its own GLA state) and
logits within the tolerance of the linears' rounding (the batch runs each
linear as one n-row product).  Checked against twin sessions fed the same
prompts and stepped one by one, with prompts of different lengths (so the rows
sit at different positions, some past the window: the rings wrap).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


def _synthetic(tmp_path_factory, name, base, **kw):
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(getattr(syn, base), **kw)
    return syn.write_model(tmp_path_factory.mktemp(name), cfg, seed=5)


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    load_pkg()
    return _synthetic(tmp_path_factory, "b_small", "BASE", vocab_size=1000, d_model=128, n_heads=2, hidden=256,
                      window=48, max_loops=4, default_loops=3)


def _pairs(slm, model, lengths, vocab, seed):
    rng = np.random.default_rng(seed)
    batch_se, twins, lasts = [], [], []
    for n in lengths:
        ids = rng.integers(0, vocab, n)
        a, b = model.session(), model.session()
        a.feed(ids, 256)
        b.feed(ids, 256)
        batch_se.append(a)
        twins.append(b)
        lasts.append(int(np.argmax(b.logits())))
    return batch_se, twins, lasts


@pytest.mark.parametrize("lengths", [[30, 47, 64, 100, 129], [5, 60, 9, 33, 71, 2, 90, 48, 17, 64, 55, 120]])
def test_batch_step_matches_single_sessions(slm, ctx, small, lengths):
    model = slm.Model(ctx, small)
    ses, twins, _ = _pairs(slm, model, lengths, 1000, 0)
    batch = slm.Batch(ses)
    rng = np.random.default_rng(1)
    worst = 0.0
    for _ in range(12):
        ids = rng.integers(0, 1000, len(ses))
        batch.step(ids)
        got = batch.logits()
        for i, tw in enumerate(twins):
            tw.step(int(ids[i]))
            worst = max(worst, float(np.abs(got[i] - tw.logits()).max()))
    assert worst < 2e-4, worst
    for se, tw in zip(ses, twins):
        assert se.pos == tw.pos
    batch.close()


def test_batch_greedy_decode_matches_single_sessions(slm, ctx, small):
    model = slm.Model(ctx, small)
    lengths = [40, 77, 12, 130, 64, 99, 3, 51, 88, 21]
    ses, twins, first = _pairs(slm, model, lengths, 1000, 2)
    batch = slm.Batch(ses)
    out = batch.decode(first, 24)
    greedy = slm.Sampling()
    for i, tw in enumerate(twins):
        np.testing.assert_array_equal(out[:, i], tw.decode(first[i], 24, greedy))
    # A second call continues from where the first stopped.
    out2 = batch.decode(out[-1], 8)
    for i, tw in enumerate(twins):
        np.testing.assert_array_equal(out2[:, i], tw.decode(int(out[-1, i]), 8, greedy))
    assert all(se.pos == tw.pos for se, tw in zip(ses, twins))
    batch.close()


def test_batch_86m_shapes(slm, ctx, tmp_path_factory):
    folder = _synthetic(tmp_path_factory, "b_m86", "BASE", window=128)
    model = slm.Model(ctx, folder)
    ses, twins, first = _pairs(slm, model, [150, 20, 300], 32000, 3)
    batch = slm.Batch(ses)
    rng = np.random.default_rng(4)
    worst = 0.0
    for _ in range(6):
        ids = rng.integers(0, 32000, 3)
        batch.step(ids)
        got = batch.logits()
        for i, tw in enumerate(twins):
            tw.step(int(ids[i]))
            worst = max(worst, float(np.abs(got[i] - tw.logits()).max()))
    assert worst < 1e-3, worst
    batch.close()


def test_batch_refusals(slm, ctx, small, tmp_path_factory):
    model = slm.Model(ctx, small)
    a, b = model.session(3), model.session(2)
    with pytest.raises(slm.SlmError):
        slm.Batch([a, b])  # different loop counts
    with pytest.raises(slm.SlmError):
        slm.Batch([a, a])  # the same session twice
    c = model.session(3)
    batch = slm.Batch([a, c])
    with pytest.raises(slm.SlmError):
        c.close()  # still in the batch
    with pytest.raises(ValueError):
        batch.step([1])  # wrong count
    with pytest.raises(slm.SlmError):
        batch.step([1, 5000])  # id out of range
    batch.close()
    c.close()
    g = _synthetic(tmp_path_factory, "b_g", "GLOBAL", vocab_size=500, d_model=64, n_heads=4, hidden=128, window=16,
                   max_loops=3, default_loops=2, global_kv_heads=2)
    gm = slm.Model(ctx, g)
    with pytest.raises(slm.SlmError):
        slm.Batch([gm.session(), gm.session()])
