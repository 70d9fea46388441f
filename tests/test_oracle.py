"""The CPU oracle against the reference's golden vectors (CPU only).

Pins the oracle: the tiny fixture's PyTorch logits at every position, plain
decode and the nine chunked-prefill splits of tests/parity.rs, and the
sampler's known-answer tests of src/sample.rs:95-152."""
import numpy as np
import pytest

from conftest import SPLITS, TINY, TOLERANCE, run_split


@pytest.fixture(scope="module")
def tiny(oracle):
    return oracle.Model(TINY)


def test_plain_decode_matches_pytorch(tiny, golden):
    checked, md, same = run_split(tiny.session, golden, 0, 1)
    assert checked == 40
    assert md < TOLERANCE and same


@pytest.mark.parametrize("split,chunk", SPLITS)
def test_chunked_prefill_matches_pytorch(tiny, golden, split, chunk):
    checked, md, same = run_split(tiny.session, golden, split, chunk)
    assert checked == 41 - split
    assert md < TOLERANCE and same, (split, chunk, md)


def test_state_bytes_and_loops(tiny, oracle):
    se = tiny.session(3)
    c = tiny.cfg
    dh = c["d_model"] // c["n_heads"]
    cap = c["window"] + 256
    # S blocks: prelude 1 + coda 1 + 3 loops × 1; L: 3 loops × 1; G: coda 1 at pos 0.
    want = (5 * 2 * c["n_heads"] * cap * dh + 3 * c["n_heads"] * dh * dh + c["d_model"]) * 4
    assert se.state_bytes() == want
    with pytest.raises(ValueError):
        tiny.session(7)  # max_loops is 6 (src/config.rs:96-105)


def test_greedy_takes_the_largest(oracle):
    assert oracle.pick([0.0, 3.0, 1.0], []) == 1


def test_penalty_can_change_the_choice(oracle):
    assert oracle.pick([0.0, 3.0, 2.0], [1], repeat_penalty=2.0, repeat_window=8) == 2


def test_top_p_keeps_the_likely_tokens(oracle):
    st = [oracle.rng_new(3)]
    for _ in range(200):
        assert oracle.pick([-9.0, 5.0, -9.0, 1.0], [], temperature=1.0, top_p=0.5, rng_state=st) == 1


def test_top_k_limits_the_candidates(oracle):
    st = [oracle.rng_new(7)]
    for _ in range(200):
        assert oracle.pick([5.0, 4.0, -9.0, -9.0], [], temperature=1.0, top_k=2, rng_state=st) < 2


def test_rng_matches_xorshift64star(oracle):
    # Rng::new(1) and its first draws, computed here with Python integers.
    s = (1 * 0x9E3779B97F4A7C15 | 1) & (2**64 - 1)
    st = [oracle.rng_new(1)]
    assert st[0] == s
    import ctypes
    for _ in range(5):
        s ^= s >> 12
        s ^= (s << 25) & (2**64 - 1)
        s ^= s >> 27
        want = np.float32(((s * 0x2545F4914F6CDD1D) & (2**64 - 1)) >> 40) / np.float32(1 << 24)
        c = ctypes.c_uint64(st[0])
        got = oracle.lib().orc_rng_next(ctypes.byref(c))
        st[0] = c.value
        assert st[0] == s and np.float32(got) == want


def test_attend_matches_direct_softmax(oracle):
    rng = np.random.default_rng(0)
    heads, kh, dh, cap, pos, m, reach = 4, 2, 8, 12, 9, 3, 5
    q = rng.standard_normal(m * heads * dh).astype(np.float32)
    k = rng.standard_normal(kh * cap * dh).astype(np.float32)
    v = rng.standard_normal(kh * cap * dh).astype(np.float32)
    y = oracle.attend(q, k, v, pos, m, reach, 0, cap, heads, kh, dh, 0.5)
    for i in range(m):
        p = pos + i
        lo = max(0, p - reach + 1)
        for h in range(heads):
            g = h // (heads // kh)
            ks = np.stack([k[(g * cap + t % cap) * dh:(g * cap + t % cap + 1) * dh] for t in range(lo, p + 1)])
            vs = np.stack([v[(g * cap + t % cap) * dh:(g * cap + t % cap + 1) * dh] for t in range(lo, p + 1)])
            s = ks @ q[(i * heads + h) * dh:(i * heads + h + 1) * dh] * 0.5
            w = np.exp(s - s.max())
            want = (w / w.sum()) @ vs
            np.testing.assert_allclose(y[(i * heads + h) * dh:(i * heads + h + 1) * dh], want, atol=1e-5)
