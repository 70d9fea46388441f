"""Op-level checks of the CPU oracle against direct float64 restatements of
the reference CPU backend's formulas (src/cpu.rs:187-403, geometry
src/ops.rs:31-66), on the edge cases that geometry allows: ring slots that
wrap, unbounded reach with a far gap, grouped key heads, queries that see
nothing, zero vectors.  CPU only: these pin the checker that the GPU parity
tests compare against."""
import numpy as np
import pytest


def rnd(seed, n, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


def visible(p, reach, gap):
    """Attn::range (src/ops.rs:60-65): max(0, p - reach + 1) .. p + 1 - gap (empty if negative)."""
    lo = 0 if reach is None else max(0, p - reach + 1)
    return range(lo, max(0, p + 1 - gap))


def attend_ref(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, scale):
    """src/cpu.rs:352-403 in float64: max-subtracted softmax over ring slots p % cap."""
    q, k, v = (a.astype(np.float64).reshape(-1, dh) for a in (q, k, v))
    y = np.zeros((m * heads, dh))
    group = heads // kh
    for i in range(m):
        r = visible(pos + i, reach, gap)
        if len(r) == 0:
            continue
        for h in range(heads):
            rows = [(h // group) * cap + p % cap for p in r]
            s = k[rows] @ q[i * heads + h] * scale
            w = np.exp(s - s.max())
            y[i * heads + h] = (w / w.sum()) @ v[rows]
    return y.reshape(-1)


ATTN = [
    # pos, m, reach, gap, cap, heads, key_heads, dh
    (9, 3, 5, 0, 12, 4, 2, 8),        # window, grouped key heads
    (40, 6, 16, 0, 20, 2, 2, 8),      # ring slots wrap (pos > cap)
    (30, 5, None, 8, 64, 4, 2, 8),    # unbounded reach, far gap
    (3, 4, None, 8, 64, 4, 2, 8),     # every query sees nothing: zeros
    (6, 5, None, 8, 64, 2, 1, 16),    # the later queries start to see
    (0, 1, 4, 0, 4, 1, 1, 4),         # one position
    (100, 2, 1, 0, 8, 3, 3, 8),       # reach 1: each query sees itself only
]


@pytest.mark.parametrize("pos,m,reach,gap,cap,heads,kh,dh", ATTN)
def test_attend_geometry(oracle, pos, m, reach, gap, cap, heads, kh, dh):
    q, k, v = rnd(1, m * heads * dh), rnd(2, kh * cap * dh), rnd(3, kh * cap * dh)
    got = oracle.attend(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, 0.35)
    want = attend_ref(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, 0.35)
    np.testing.assert_allclose(got, want, atol=2e-6, rtol=1e-5)
    for i in range(m):
        if len(visible(pos + i, reach, gap)) == 0:
            assert not got[i * heads * dh:(i + 1) * heads * dh].any()


def test_attend_large_scores_stay_finite(oracle):
    # Scores far beyond exp's range: the max subtraction keeps the softmax finite.
    q, k, v = rnd(4, 2 * 8, 30.0), rnd(5, 2 * 16 * 8, 30.0), rnd(6, 2 * 16 * 8)
    got = oracle.attend(q, k, v, 15, 1, 16, 0, 16, 2, 2, 8, 1.0)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, attend_ref(q, k, v, 15, 1, 16, 0, 16, 2, 2, 8, 1.0), atol=1e-5)


def test_gla_recurrence(oracle):
    """src/cpu.rs:284-329: per head, in token order, S = σ(-(decay + bias))·S + kᵀv, y = q·S."""
    m, heads, dh = 5, 3, 8
    q, k, v = rnd(7, m * heads * dh), rnd(8, m * heads * dh), rnd(9, m * heads * dh)
    decay, bias = rnd(10, m * heads, 2.0), rnd(11, heads)
    s0 = rnd(12, heads * dh * dh)
    s = s0.copy()
    got = oracle.gla(s, q, k, v, decay, bias, m, heads, dh)
    S = s0.astype(np.float64).reshape(heads, dh, dh)
    want = np.zeros((m, heads, dh))
    for i in range(m):
        for h in range(heads):
            at = (i * heads + h) * dh
            d = 1.0 / (1.0 + np.exp(float(decay[i * heads + h]) + float(bias[h])))
            S[h] = d * S[h] + np.outer(k[at:at + dh], v[at:at + dh])
            want[i, h] = q[at:at + dh].astype(np.float64) @ S[h]
    np.testing.assert_allclose(got, want.reshape(-1), atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(s, S.reshape(-1), atol=2e-5, rtol=1e-5)


def test_rms_groups(oracle):
    """src/cpu.rs:187-207: y = x·w / sqrt(mean(x²) + eps) per group."""
    groups, size, eps = 4, 16, 1e-6
    x, w = rnd(13, groups * size), rnd(14, size)
    got = oracle.rms(x, w, groups, size, eps)
    g = x.astype(np.float64).reshape(groups, size)
    want = g / np.sqrt((g * g).mean(axis=1, keepdims=True) + eps) * w
    np.testing.assert_allclose(got, want.reshape(-1), rtol=1e-5, atol=1e-6)


def test_l2norm_clamps_a_zero_head(oracle):
    """src/cpu.rs:270-282: x / max(‖x‖, 1e-12); a zero head stays zero."""
    heads, dh = 3, 8
    x = rnd(15, heads * dh)
    x[dh:2 * dh] = 0.0
    got = oracle.l2norm(x, heads, dh)
    h = x.astype(np.float64).reshape(heads, dh)
    want = h / np.maximum(np.linalg.norm(h, axis=1, keepdims=True), 1e-12)
    np.testing.assert_allclose(got, want.reshape(-1), rtol=1e-5, atol=1e-7)
    assert not got[dh:2 * dh].any()


def test_silu_mul_at_the_extremes(oracle):
    """src/cpu.rs:209-215: y = u·g / (1 + e^-g), including |g| beyond exp's range."""
    g = np.array([-200.0, -20.0, -1.0, 0.0, 0.5, 3.0, 90.0], dtype=np.float32)
    u = rnd(16, len(g))
    got = oracle.silu_mul(g, u)
    gd = g.astype(np.float64)
    want = u * gd / (1.0 + np.exp(-gd))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-30)
    assert np.isfinite(got).all()


def test_rope_half_split(oracle):
    """src/cpu.rs:217-268: angle (pos + i)·inv[j]; pairs (j, j + dh/2) rotated."""
    m, heads, dh, pos = 3, 2, 8, 1000
    half = dh // 2
    inv = (1.0 / 10000.0 ** (np.arange(half) * 2.0 / dh)).astype(np.float32)
    c, s = oracle.rope_table(inv, pos, m, half)
    ang = (np.arange(pos, pos + m, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    np.testing.assert_allclose(c.reshape(m, half), np.cos(ang.astype(np.float64)), atol=2e-6)
    np.testing.assert_allclose(s.reshape(m, half), np.sin(ang.astype(np.float64)), atol=2e-6)
    x = rnd(17, m * heads * dh)
    got = oracle.rope(x, c, s, m, heads, dh).reshape(m, heads, dh)
    xv = x.reshape(m, heads, dh).astype(np.float64)
    cc, ss = c.reshape(m, 1, half).astype(np.float64), s.reshape(m, 1, half).astype(np.float64)
    a, b = xv[..., :half], xv[..., half:]
    np.testing.assert_allclose(got[..., :half], a * cc - b * ss, atol=1e-6)
    np.testing.assert_allclose(got[..., half:], a * ss + b * cc, atol=1e-6)


def test_store_wraps_the_ring(oracle):
    """src/cpu.rs:331-350: row i of head h goes to slot (pos + i) % cap."""
    m, heads, dh, cap, pos = 5, 2, 4, 6, 4
    cache = np.full(heads * cap * dh, -1.0, dtype=np.float32)
    src = rnd(18, m * heads * dh)
    oracle.store(cache, src, pos, m, cap, heads, dh)
    c = cache.reshape(heads, cap, dh)
    for i in range(m):
        for h in range(heads):
            np.testing.assert_array_equal(c[h, (pos + i) % cap], src[(i * heads + h) * dh:(i * heads + h + 1) * dh])
    untouched = {(pos + i) % cap for i in range(m)} ^ set(range(cap))
    for slot in untouched:
        assert (c[:, slot] == -1.0).all()
