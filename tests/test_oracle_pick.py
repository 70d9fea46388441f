"""The CPU oracle's pick (src/sample.rs:33-93) against a float32 numpy
restatement, on edge cases beyond the reference's own sampler tests: the
penalty's sign rule, duplicate recent ids, the repeat window, top-k with
top-p, temperature with top-k 1.  After top-k the candidate order is the
canonical one (logit descending in f32 total order, then id ascending): the
reference's select_nth_unstable order is unspecified.  CPU only."""
import numpy as np
import pytest

MASK = (1 << 64) - 1


def next_f32(st):
    """Rng::next_f32 (src/sample.rs:25-30): xorshift64*, top 24 bits."""
    x = st[0]
    x ^= x >> 12
    x ^= (x << 25) & MASK
    x ^= x >> 27
    st[0] = x
    return np.float32(((x * 0x2545F4914F6CDD1D) & MASK) >> 40) / np.float32(1 << 24)


def pick_ref(logits, recent, temperature=0.0, top_k=0, top_p=1.0, repeat_penalty=1.0, repeat_window=0,
             st=None):
    lg = np.array(logits, dtype=np.float32)
    f = np.float32
    if repeat_penalty != 1.0:
        start = max(0, len(recent) - repeat_window)
        for t in sorted(set(int(t) for t in recent[start:])):
            lg[t] = lg[t] / f(repeat_penalty) if lg[t] > 0 else lg[t] * f(repeat_penalty)
    if temperature <= 0.0:
        return int(np.argmax(lg))  # first maximum
    ids = list(range(len(lg)))
    canon = lambda i: (-float(lg[i]), i)  # noqa: E731
    if 0 < top_k < len(ids):
        ids = sorted(ids, key=canon)[:top_k]
    if top_p < 1.0:
        ids = sorted(ids, key=canon)
    top = max(lg[i] for i in ids)
    w = [f(np.exp(f((lg[i] - top) / f(temperature)))) for i in ids]
    if top_p < 1.0:
        total = f(0.0)
        for x in w:
            total = f(total + x)
        enough, held, keep = f(f(top_p) * total), f(0.0), len(w)
        for j, x in enumerate(w):
            held = f(held + x)
            if held >= enough:
                keep = j + 1
                break
        ids, w = ids[:keep], w[:keep]
    total = f(0.0)
    for x in w:
        total = f(total + x)
    r = f(next_f32(st) * total)
    for i, x in zip(ids, w):
        r = f(r - x)
        if r <= 0.0:
            return i
    return ids[-1]


def seed(s):
    """Rng::new (src/sample.rs:21-23)."""
    return ((s * 0x9E3779B97F4A7C15) & MASK) | 1


def test_penalty_divides_positive_and_multiplies_negative(oracle):
    lg = np.array([2.0, 1.9, -0.5, -0.4], dtype=np.float32)
    # 0 falls to 1.0 (< 1.9); 3 falls to -0.8 (< -0.5): greedy moves to 1.
    assert oracle.pick(lg, [0, 3], repeat_penalty=2.0, repeat_window=8) == 1
    assert pick_ref(lg, [0, 3], repeat_penalty=2.0, repeat_window=8) == 1


def test_duplicate_recent_ids_are_penalised_once(oracle):
    lg = np.array([3.0, 2.0], dtype=np.float32)
    # Once: 3 / 1.4 = 2.14 > 2 stays first; applied three times it would not.
    assert oracle.pick(lg, [0, 0, 0], repeat_penalty=1.4, repeat_window=8) == 0


def test_only_the_last_window_ids_count(oracle):
    lg = np.array([3.0, 2.9, 0.0], dtype=np.float32)
    recent = [0] + [2] * 4  # id 0 falls outside a window of 4
    assert oracle.pick(lg, recent, repeat_penalty=5.0, repeat_window=4) == 0
    assert oracle.pick(lg, recent, repeat_penalty=5.0, repeat_window=5) == 1


def test_greedy_takes_the_first_maximum(oracle):
    lg = np.array([1.0, 4.0, 4.0, -2.0], dtype=np.float32)
    assert oracle.pick(lg, []) == 1


def test_top_k_one_is_greedy_at_any_temperature(oracle):
    lg = np.random.default_rng(1).standard_normal(500).astype(np.float32)
    st = [seed(7)]
    for _ in range(20):
        assert oracle.pick(lg, [], temperature=2.5, top_k=1, rng_state=st) == int(np.argmax(lg))


CASES = [
    dict(temperature=0.8),
    dict(temperature=0.8, top_k=40),
    dict(temperature=1.3, top_p=0.9),
    dict(temperature=0.7, top_k=100, top_p=0.5),
    dict(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=256),
    dict(temperature=0.5, top_p=0.0),  # keeps only the most likely id
]


@pytest.mark.parametrize("kw", CASES)
def test_pick_sequence_matches_the_restatement(oracle, kw):
    rng = np.random.default_rng(3)
    lg = (rng.standard_normal(3000) * 3).astype(np.float32)
    recent = [int(t) for t in rng.integers(0, 3000, 300)]
    a, b = [seed(11)], [seed(11)]
    for _ in range(30):
        got = oracle.pick(lg, recent, rng_state=a, **kw)
        want = pick_ref(lg, recent, st=b, **kw)
        assert got == want
        assert a[0] == b[0]  # the same xorshift64* state after the draw
        recent.append(got)
