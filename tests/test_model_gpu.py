"""Model-level parity through the C ABI: the tiny golden fixture (the
reference's own parity test, tests/parity.rs), synthetic models against the
CPU oracle, and chunked prefill against token-by-token decode."""
import numpy as np
import pytest

from conftest import SPLITS, TINY, TOLERANCE, load_pkg, run_split

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(slm, ctx):
    return slm.Model(ctx, TINY)


@pytest.mark.parametrize("graph", [True, False])
def test_tiny_plain_decode(tiny, golden, graph):
    def factory(loops):
        se = tiny.session(loops)
        se.set_graph(graph)
        return se

    checked, md, same = run_split(factory, golden, 0, 1)
    assert checked == 40
    assert md < TOLERANCE and same, md


@pytest.mark.parametrize("split,chunk", SPLITS)
def test_tiny_chunked_prefill(tiny, golden, split, chunk):
    checked, md, same = run_split(tiny.session, golden, split, chunk)
    assert checked == 41 - split
    assert md < TOLERANCE and same, (split, chunk, md)


def test_tiny_state_bytes(tiny, oracle):
    ref = oracle.Model(TINY)
    a, b = tiny.session(3), ref.session(3)
    ids = np.arange(13) % 97
    a.feed(ids, 5)
    b.feed(ids, 5)
    assert a.state_bytes() == b.state_bytes()
    assert a.pos == b.pos == 13


def _synthetic(tmp_path_factory, name, base, **kw):
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(getattr(syn, base), **kw)
    return syn.write_model(tmp_path_factory.mktemp(name), cfg, seed=5)


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    load_pkg()
    return _synthetic(tmp_path_factory, "small", "BASE", vocab_size=1000, d_model=128, n_heads=2, hidden=256,
                      window=48, max_loops=4, default_loops=3)


@pytest.fixture(scope="module")
def small_g(tmp_path_factory):
    load_pkg()
    return _synthetic(tmp_path_factory, "small_g", "GLOBAL", vocab_size=500, d_model=64, n_heads=4, hidden=128,
                      window=16, max_loops=3, default_loops=2, global_kv_heads=2)


def compare(dev, ref, ids, limit, steps, atol):
    dev.feed(ids, limit)
    ref.feed(ids, limit)
    worst = float(np.abs(dev.logits() - ref.logits()).max())
    tok = int(np.argmax(ref.logits()))
    for _ in range(steps):
        dev.step(tok)
        ref.step(tok)
        a, b = dev.logits(), ref.logits()
        worst = max(worst, float(np.abs(a - b).max()))
        tok = int(np.argmax(b))
    assert worst < atol, worst
    return worst


@pytest.mark.parametrize("limit", [256, 7, 1])
def test_small_model_matches_oracle(slm, ctx, oracle, small, limit):
    ids = np.random.default_rng(0).integers(0, 1000, 300)
    dev = slm.Model(ctx, small).session()
    ref = oracle.Model(small).session()
    compare(dev, ref, ids, limit, 20, 2e-4)


def test_global_variant_matches_oracle(slm, ctx, oracle, small_g):
    ids = np.random.default_rng(1).integers(0, 500, 200)
    dev = slm.Model(ctx, small_g).session()
    ref = oracle.Model(small_g).session()
    compare(dev, ref, ids, 64, 20, 2e-4)


def test_global_cache_grows_on_device(slm, ctx, oracle, small_g):
    # 8192 slots first (src/model.rs:320); crossing it doubles the cache.
    ids = np.random.default_rng(2).integers(0, 500, 8250)
    dev = slm.Model(ctx, small_g).session(1)
    ref = oracle.Model(small_g).session(1)
    compare(dev, ref, ids, 256, 5, 5e-4)
    assert dev.state_bytes() == ref.state_bytes()


def test_chunked_prefill_gives_the_same_greedy_tokens(slm, ctx, small):
    model = slm.Model(ctx, small)
    ids = np.random.default_rng(3).integers(0, 1000, 333)
    a, b = model.session(), model.session()
    a.feed(ids, 256)
    for t in ids:
        b.step(int(t))
    greedy = slm.Sampling()
    first_a, first_b = a.sample(greedy), b.sample(greedy)
    assert first_a == first_b
    ta = a.decode(first_a, 48, greedy)
    tb = b.decode(first_b, 48, greedy)
    np.testing.assert_array_equal(ta, tb)


def test_86m_shapes_match_oracle(slm, ctx, oracle, tmp_path_factory):
    folder = _synthetic(tmp_path_factory, "m86", "BASE", window=128)
    ids = np.random.default_rng(4).integers(0, 32000, 160)
    dev = slm.Model(ctx, folder).session(2)
    ref = oracle.Model(folder).session(2)
    compare(dev, ref, ids, 64, 4, 1e-3)


def test_86m_shapes_full_chunks_match_oracle(slm, ctx, oracle, tmp_path_factory):
    # 256-token chunks: the wide linears (qkv, qkvg, up) run as the bf16x3
    # tensor-core GEMM, the 768-wide ones as the FastFP32 kernel.
    folder = _synthetic(tmp_path_factory, "m86c", "BASE", window=128)
    ids = np.random.default_rng(6).integers(0, 32000, 300)
    dev = slm.Model(ctx, folder).session(2)
    ref = oracle.Model(folder).session(2)
    compare(dev, ref, ids, 256, 2, 1e-3)


def test_errors_are_statuses(slm, ctx, tiny):
    se = tiny.session()
    with pytest.raises(slm.SlmError):
        se.step(97)  # vocab is 97
    with pytest.raises(slm.SlmError):
        se.feed([1, 2, 500])
    with pytest.raises(slm.SlmError):
        tiny.session(7)  # max_loops 6
    with pytest.raises(slm.SlmError):
        slm.Model(ctx, TINY.parent / "missing")


def test_persistent_kernel_matches_graph_path(slm, ctx, small):
    model = slm.Model(ctx, small)
    ids = np.random.default_rng(6).integers(0, 1000, 360)
    a, b = model.session(), model.session()
    b.set_mega(False)
    assert a.mega and not b.mega
    # 8 blocks of 3 phases (projection, attention or GLA with o, one MLP phase), inject, logits
    assert a.stat(slm.SLM_STAT_PHASES) == 3 * 8 + 2
    a.feed(ids[:300])
    b.feed(ids[:300])
    worst = 0.0
    for t in ids[300:]:  # crosses the ring's wrap (cap = 48 + 256)
        a.step(int(t))
        b.step(int(t))
        worst = max(worst, float(np.abs(a.logits() - b.logits()).max()))
    assert worst < 2e-5, worst
    greedy = slm.Sampling()
    first = a.sample(greedy)
    assert first == b.sample(greedy)
    np.testing.assert_array_equal(a.decode(first, 64, greedy), b.decode(first, 64, greedy))
    assert a.pos == b.pos


@pytest.mark.parametrize("which", ["small", "g64"])
def test_fused_mlp_matches_two_phase_mlp(slm, ctx, request, monkeypatch, which):
    # The persistent step runs each MLP as one phase whose residual sum is
    # int64 fixed point; SLM_MEGA_FUSE_MLP=0 keeps gate/up and down as two
    # phases with float adds.  Same tokens, logits within fp32 noise; two fused
    # sessions give bit-identical logits (integer sums do not depend on the
    # order in which CTAs add).
    model = slm.Model(ctx, request.getfixturevalue(which))
    a = model.session()
    monkeypatch.setenv("SLM_MEGA_FUSE_MLP", "0")
    b = model.session()
    monkeypatch.delenv("SLM_MEGA_FUSE_MLP")
    c = model.session()
    monkeypatch.setenv("SLM_MEGA_MLP_CTA", "1")  # tiles split by rows, a CTA barrier per tile
    e = model.session()
    monkeypatch.delenv("SLM_MEGA_MLP_CTA")
    monkeypatch.setenv("SLM_MEGA_FUSE_ATTN_O", "0")  # S and L blocks keep o as its own phase
    f = model.session()
    monkeypatch.delenv("SLM_MEGA_FUSE_ATTN_O")
    assert a.mega and b.mega and c.mega and e.mega and f.mega
    n = {k: se.stat(slm.SLM_STAT_PHASES) for k, se in zip("abcef", (a, b, c, e, f))}
    assert n["a"] == n["c"] == n["e"] < n["f"] < n["b"]
    if which == "small":  # 5 S and 3 L blocks
        assert n["b"] - n["f"] == 8 and n["f"] - n["a"] == 8
    ids = np.random.default_rng(13).integers(0, 1000, 90)
    for se in (a, b, c, e, f):
        se.feed(ids)
    tok = int(np.argmax(b.logits()))
    worst = 0.0
    for _ in range(40):
        for se in (a, b, c, e, f):
            se.step(tok)
        la, lb, lc, le, lf = a.logits(), b.logits(), c.logits(), e.logits(), f.logits()
        worst = max(worst, *(float(np.abs(x - lb).max()) for x in (la, le, lf)))
        np.testing.assert_array_equal(la, lc)
        tok = int(np.argmax(lb))
    assert worst < 2e-5, worst
    greedy = slm.Sampling()
    first = a.sample(greedy)
    assert first == b.sample(greedy) == c.sample(greedy)
    np.testing.assert_array_equal(a.decode(first, 32, greedy), b.decode(first, 32, greedy))


def test_persistent_kernel_sampling_path(slm, ctx, small):
    model = slm.Model(ctx, small)
    s = slm.Sampling(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=64)
    prompt = np.random.default_rng(7).integers(0, 1000, 70)
    a, b = model.session(), model.session()
    b.set_mega(False)
    a.feed(prompt)
    b.feed(prompt)
    sa, sb = [slm.rng_seed(5)], [slm.rng_seed(5)]
    first = a.sample(s, list(prompt), sa)
    assert first == b.sample(s, list(prompt), sb)
    hist = list(prompt) + [first]
    np.testing.assert_array_equal(a.decode(first, 40, s, hist, sa), b.decode(first, 40, s, hist, sb))


def test_greedy_sample_after_persistent_steps(slm, ctx, oracle, small):
    # slm_sample with greedy settings reads the arg-max the persistent step
    # computed; with a penalty, after a feed, or after graph steps it runs the
    # sampler.  Every case must equal pick on the logits read back.
    model = slm.Model(ctx, small)
    se = model.session()
    prompt = np.random.default_rng(8).integers(0, 1000, 40)
    se.feed(prompt)
    greedy = slm.Sampling()
    st = [slm.rng_seed(1)]
    tok = se.sample(greedy, [], st)
    assert tok == int(np.argmax(se.logits()))
    for step in range(12):
        if step == 6:
            se.set_mega(False)
        se.step(tok)
        lg = se.logits()
        assert se.sample(greedy, [], st) == int(np.argmax(lg))
        pen = slm.Sampling(repeat_penalty=1.3, repeat_window=16)
        recent = [int(t) for t in prompt[-16:]]
        want = oracle.pick(lg, np.array(recent, dtype=np.uint32), repeat_penalty=1.3, repeat_window=16)
        tok = se.sample(pen, recent, st)
        assert tok == want


def test_greedy_sample_with_interleaved_sessions(slm, ctx, small):
    # Persistent steps pass the id in the launch and greedy sampling reads the
    # arg-max beside the context's error word when this session stepped last;
    # sessions stepped in turn on one context must each get their own.
    model = slm.Model(ctx, small)
    a, b = model.session(), model.session()
    rng = np.random.default_rng(14)
    a.feed(rng.integers(0, 1000, 30))
    b.feed(rng.integers(0, 1000, 50))
    greedy = slm.Sampling()
    ta, tb = a.sample(greedy), b.sample(greedy)
    for i in range(10):
        a.step(ta)
        b.step(tb)
        if i % 3 == 2:
            a.step(ta)  # two steps of a in a row: the later one counts
        la, lb = a.logits(), b.logits()
        ta, tb = a.sample(greedy), b.sample(greedy)
        assert ta == int(np.argmax(la)) and tb == int(np.argmax(lb))
        assert a.sample(greedy) == ta  # sampling again reads the same step
    b.close()
    a.step(ta)
    assert a.sample(greedy) == int(np.argmax(a.logits()))


@pytest.fixture(scope="module")
def g64(tmp_path_factory):
    load_pkg()
    # Global variant with head size 64 and GQA (6 heads over 2 cache heads), a
    # short window so the far gap opens after 32 positions.
    return _synthetic(tmp_path_factory, "g64", "GLOBAL", vocab_size=1000, d_model=384, n_heads=6, hidden=768,
                      window=32, max_loops=3, default_loops=2, global_kv_heads=2)


def _lockstep(a, b, tok, steps, atol):
    worst = 0.0
    for _ in range(steps):
        a.step(tok)
        b.step(tok)
        la, lb = a.logits(), b.logits()
        worst = max(worst, float(np.abs(la - lb).max()))
        assert int(np.argmax(la)) == int(np.argmax(lb))
        tok = int(np.argmax(lb))
    assert worst < atol, worst
    return tok


def test_persistent_kernel_runs_global_layers(slm, ctx, oracle, g64):
    # Persistent steps of a model with a global layer (norm_e, logn, kshift,
    # far gap, GQA) against the graph path, from before the far gap opens to
    # well after, and against the oracle.
    model = slm.Model(ctx, g64)
    a, b = model.session(), model.session()
    assert a.mega, a.stat(3)
    b.set_mega(False)
    ids = np.random.default_rng(11).integers(0, 1000, 20)
    a.feed(ids)
    b.feed(ids)
    tok = _lockstep(a, b, int(np.argmax(b.logits())), 50, 2e-5)
    ref = oracle.Model(g64).session()
    ref.feed(ids)
    # Replay the same tokens on the oracle: a's history is ids + the 50 stepped ones.
    c = model.session()
    c.feed(ids)
    t = int(np.argmax(c.logits()))
    worst = 0.0
    for _ in range(50):
        c.step(t)
        ref.step(t)
        worst = max(worst, float(np.abs(c.logits() - ref.logits()).max()))
        t = int(np.argmax(ref.logits()))
    assert worst < 2e-4, worst
    assert a.state_bytes() == b.state_bytes()


def test_persistent_kernel_follows_global_cache_growth(slm, ctx, g64):
    # The first global cache holds 8192 positions; stepping across it moves the
    # cache and the persistent step must follow (its plan is refreshed).
    model = slm.Model(ctx, g64)
    a, b = model.session(1), model.session(1)
    b.set_mega(False)
    ids = np.random.default_rng(12).integers(0, 1000, 8180)
    a.feed(ids)
    b.feed(ids)
    _lockstep(a, b, int(np.argmax(b.logits())), 24, 2e-5)
    assert a.pos == b.pos == 8204
    greedy = slm.Sampling()
    first = a.sample(greedy)
    assert first == b.sample(greedy)
    np.testing.assert_array_equal(a.decode(first, 16, greedy), b.decode(first, 16, greedy))


def test_persistent_kernel_is_refused_where_it_does_not_apply(slm, tiny):
    se = tiny.session()
    assert not se.mega  # head size 8 and a global layer
    with pytest.raises(slm.SlmError):
        se.set_mega(True)


def test_handles_free_in_any_order(slm):
    # A garbage collector may finalise a context before its buffers, or a
    # model before its sessions: freeing a handle that still has live
    # children defers its release to the last child.
    ctx = slm.Context(0)
    ops = slm.Ops(ctx)
    buf = ops.upload(np.arange(8, dtype=np.float32))
    model = slm.Model(ctx, TINY)
    se = model.session(3)
    ctx.close()
    model.close()
    se.feed([1, 2, 3])  # the session still works: its model and context live on
    assert se.logits().shape == (97,)
    np.testing.assert_array_equal(buf.read(8), np.arange(8, dtype=np.float32))
    se.close()
    buf.close()
