"""bf16 weights in the persistent decode step (SLM_OPT_BF16).

The step streams bf16 copies of its matrices and keeps f32 arithmetic,
caches and state.  Parity is checked on a model whose weights are already
bf16-exact (every matrix rounded to bf16 and stored as f32): the oracle then
computes with exactly the weights the kernel reads, and the logits must agree
within the f32 bar (1e-3).  On an ordinary f32 model the bf16 step's logits
differ by the weights' rounding; that difference is bounded here (0.2, with
the greedy id unchanged at least 75 % of the time) and stated in DESIGN.md.
"""
import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


def to_bf16_exact(a):
    """Rounds float32 values to the nearest bf16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    load_pkg()
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.BASE
    plain = syn.write_model(tmp_path_factory.mktemp("bf_plain"), cfg, seed=0)
    exact = tmp_path_factory.mktemp("bf_exact")
    syn.write_model(exact, cfg, seed=0)
    tensors = {k: (to_bf16_exact(v) if v.ndim == 2 else v) for k, v in syn.make_tensors(cfg, seed=0).items()}
    syn.write_safetensors(exact / "model.safetensors", tensors)
    return plain, exact


def restore(dev, ref, pos, seed):
    ref.fill(pos, seed)
    dev.set_pos(pos)
    for i, a in enumerate(ref.state()):
        dev.state_write(i, a["data"], a["cap"])


def test_rounding_helper_matches_known_values():
    x = np.array([1.0, 1.00390625, 1.0029296875, -2.5, 3.1415927], dtype=np.float32)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa wins (1.0)
    np.testing.assert_array_equal(to_bf16_exact(x)[:2], np.array([1.0, 1.0], dtype=np.float32))
    assert to_bf16_exact(x)[3] == -2.5
    assert abs(float(to_bf16_exact(x)[4]) - 3.140625) < 1e-7


def test_bf16_step_matches_oracle_on_bf16_exact_weights(slm, ctx, oracle, models):
    _, exact = models
    model, omodel = slm.Model(ctx, exact), oracle.Model(exact)
    dev, ref = model.session(4), omodel.session(4)
    dev.set_bf16(True)
    assert dev.mega
    restore(dev, ref, 4400, seed=7)
    tok, worst = 17, 0.0
    for _ in range(16):
        dev.step(tok)
        ref.step(tok)
        a, b = dev.logits(), ref.logits()
        worst = max(worst, float(np.abs(a - b).max()))
        tok = int(np.argmax(b))
    assert worst < 1e-3, worst
    # The greedy decode in one launch gives the oracle's tokens too.
    dev2, ref2 = model.session(4), omodel.session(4)
    dev2.set_bf16(True)
    restore(dev2, ref2, 4400, seed=8)
    got = dev2.decode(5, 12, slm.Sampling())
    want, lg, t = [], [], 5
    for _ in range(12):
        ref2.step(t)
        lg.append(ref2.logits())
        t = int(np.argmax(lg[-1]))
        want.append(t)
    for k, (g, w) in enumerate(zip(got, want)):
        if g != w:  # only at a near tie of the oracle's logits; later ids follow other inputs
            assert lg[k][int(g)] >= lg[k][w] - 2e-3, (k, g, w)
            break


def test_bf16_step_stays_close_to_f32(slm, ctx, models):
    plain, _ = models
    model = slm.Model(ctx, plain)
    a, b = model.session(4), model.session(4)
    b.set_bf16(True)
    ids = np.random.default_rng(9).integers(0, 32000, 300)
    a.feed(ids)
    b.feed(ids)
    tok, worst, same = int(np.argmax(a.logits())), 0.0, 0
    for _ in range(40):
        a.step(tok)
        b.step(tok)
        la, lb = a.logits(), b.logits()
        worst = max(worst, float(np.abs(la - lb).max()))
        same += int(np.argmax(la) == np.argmax(lb))
        tok = int(np.argmax(la))
    print(f"bf16 against f32 weights: max |dlogit| {worst:.4f}, same greedy id {same}/40")
    assert worst < 0.2, worst
    assert same >= 30, same
    b.set_bf16(False)  # back to f32: identical to the f32 session from here
    a.step(tok)
    b.step(tok)
    np.testing.assert_allclose(b.logits(), a.logits(), atol=0.2)


def test_bf16_refused_where_it_does_not_apply(slm, ctx, tmp_path_factory):
    syn = __import__("slm_b200.synthetic").synthetic
    small = syn.write_model(tmp_path_factory.mktemp("bf_small"),
                            syn.scaled(syn.BASE, vocab_size=1000, d_model=128, n_heads=2, hidden=256, window=48,
                                       max_loops=4, default_loops=3), seed=5)
    se = slm.Model(ctx, small).session()
    with pytest.raises(slm.SlmError):
        se.set_bf16(True)  # d_model 128 is not a multiple of 256
