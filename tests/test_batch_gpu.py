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


def test_batch_refusals(slm, ctx, small):
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



def test_batch_sampled_decode_matches_single_sessions(slm, ctx, small):
    # Per-row sampling: each row its own settings, history and RNG state; the
    # device sampler of a single session (slm_decode) gives the same ids.
    model = slm.Model(ctx, small)
    lengths = [40, 77, 12, 130, 64, 99]
    ses, twins, first = _pairs(slm, model, lengths, 1000, 6)
    batch = slm.Batch(ses)
    settings = [slm.Sampling(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=64),
                slm.Sampling(),  # greedy row
                slm.Sampling(temperature=1.0, top_p=0.9),
                slm.Sampling(temperature=0.7, top_k=5, top_p=0.8, repeat_penalty=1.3, repeat_window=16),
                slm.Sampling(temperature=1.2),
                slm.Sampling(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=256)]
    rng = np.random.default_rng(7)
    hists = [[int(t) for t in rng.integers(0, 1000, n)] for n in (50, 0, 10, 300, 5, 70)]
    states = [slm.rng_seed(100 + i) for i in range(len(ses))]
    out = batch.sample_decode(first, 20, settings, hists, states)
    for i, tw in enumerate(twins):
        st = [slm.rng_seed(100 + i)]
        want = tw.decode(first[i], 20, settings[i], hists[i], st)
        np.testing.assert_array_equal(out[:, i], want, err_msg=str(i))
        assert states[i] == st[0]
    batch.close()


def test_batch_rows_match_oracle_on_a_wrapped_window(slm, ctx, oracle, tmp_path_factory):
    # 86M-class shapes with a full, wrapped 4096 window: every row restored
    # from its own oracle state at positions past the ring's capacity (4352),
    # then stepped in the batch with the oracle's tokens; logits within 1e-3
    # of the oracle's, and per-row sampling (configs[2]'s settings) draw for
    # draw against the oracle's pick.
    syn = __import__("slm_b200.synthetic").synthetic
    folder = syn.write_model(tmp_path_factory.mktemp("b_m86w"), syn.BASE, seed=0)
    model, omodel = slm.Model(ctx, folder), oracle.Model(folder)
    positions = [4400, 4610, 5000, 4353]
    ses, refs = [], []
    for i, pos in enumerate(positions):
        dev, ref = model.session(4), omodel.session(4)
        ref.fill(pos, 30 + i)
        dev.set_pos(pos)
        for j, a in enumerate(ref.state()):
            dev.state_write(j, a["data"], a["cap"])
        ses.append(dev)
        refs.append(ref)
    batch = slm.Batch(ses)
    toks = [11, 222, 3333, 4444]
    worst = 0.0
    for _ in range(6):
        batch.step(toks)
        got = batch.logits()
        nxt = []
        for i, ref in enumerate(refs):
            ref.step(toks[i])
            lg = ref.logits()
            worst = max(worst, float(np.abs(got[i] - lg).max()))
            nxt.append(int(np.argmax(lg)))
        toks = nxt
    assert worst < 1e-3, worst
    # Sampled rows against the oracle's pick, teacher-forced through slm_batch_step.
    c3 = dict(temperature=0.8, top_k=40, top_p=1.0, repeat_penalty=1.1, repeat_window=256)
    s = slm.Sampling(**c3)
    hists = [[int(t) for t in np.random.default_rng(40 + i).integers(0, 32000, 256)] for i in range(4)]
    st_ref = [oracle.rng_new(i) for i in range(4)]
    st_dev = [slm.rng_seed(i) for i in range(4)]
    got = batch.sample_decode(toks, 1, [s] * 4, hists, st_dev)[0]
    for i, ref in enumerate(refs):
        ref.step(toks[i])
        st = [st_ref[i]]
        want = oracle.pick(ref.logits(), np.array(hists[i], dtype=np.uint32), rng_state=st, **c3)
        assert int(got[i]) == want and st_dev[i] == st[0], i
    batch.close()


@pytest.fixture(scope="module")
def small_g(tmp_path_factory):
    load_pkg()
    # Global variant with GQA (4 heads over 2 cache heads), kshift, norm_e, logn
    # and a far gap that opens after 16 positions.
    return _synthetic(tmp_path_factory, "b_g", "GLOBAL", vocab_size=500, d_model=64, n_heads=4, hidden=128,
                      window=16, max_loops=3, default_loops=2, global_kv_heads=2)


def test_batch_global_layers_match_single_sessions(slm, ctx, small_g):
    # Rows before and after the far gap opens (prompts of 3 … 90 ids), each
    # with its own global cache, position and shifted-key input.
    model = slm.Model(ctx, small_g)
    ses, twins, first = _pairs(slm, model, [3, 10, 15, 16, 40, 90], 500, 8)
    batch = slm.Batch(ses)
    rng = np.random.default_rng(9)
    worst = 0.0
    for _ in range(20):
        ids = rng.integers(0, 500, len(ses))
        batch.step(ids)
        got = batch.logits()
        for i, tw in enumerate(twins):
            tw.step(int(ids[i]))
            worst = max(worst, float(np.abs(got[i] - tw.logits()).max()))
    assert worst < 2e-4, worst
    out = batch.decode([int(np.argmax(got[i])) for i in range(len(ses))], 12)
    greedy = slm.Sampling()
    for i, tw in enumerate(twins):
        np.testing.assert_array_equal(out[:, i], tw.decode(int(np.argmax(got[i])), 12, greedy))
    batch.close()


def test_batch_global_rows_match_oracle_across_cache_growth(slm, ctx, oracle, tmp_path_factory):
    # The 86M-class G variant (S | LS | SG): rows restored from the oracle at
    # positions past 16384 and one just below 8192, whose global caches grow
    # from 8192 to 16384 slots during the batch's steps.
    syn = __import__("slm_b200.synthetic").synthetic
    folder = syn.write_model(tmp_path_factory.mktemp("b_g86"), syn.GLOBAL, seed=0)
    model, omodel = slm.Model(ctx, folder), oracle.Model(folder)
    positions = [16400, 8188, 17000]
    ses, refs = [], []
    for i, pos in enumerate(positions):
        dev, ref = model.session(4), omodel.session(4)
        ref.fill(pos, 50 + i)
        dev.set_pos(pos)
        for j, a in enumerate(ref.state()):
            dev.state_write(j, a["data"], a["cap"])
        ses.append(dev)
        refs.append(ref)
    batch = slm.Batch(ses)
    toks = [7, 77, 777]
    worst = 0.0
    for _ in range(8):
        batch.step(toks)
        got = batch.logits()
        nxt = []
        for i, ref in enumerate(refs):
            ref.step(toks[i])
            lg = ref.logits()
            worst = max(worst, float(np.abs(got[i] - lg).max()))
            nxt.append(int(np.argmax(lg)))
        toks = nxt
    assert worst < 1e-3, worst
    grown = [a for a in ses[1].state_arrays() if a["kind"] == "G" and a["part"] == "k"]
    assert grown and all(a["cap"] == 16384 for a in grown)
    batch.close()
