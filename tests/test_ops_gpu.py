"""Op-level parity: each `Ops` method through the C ABI against the CPU
oracle (src/cpu.rs restated) on the same seeded inputs.  fp32 with a
different summation order, so the bar is a small absolute/relative error."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)


def rand(*shape, scale=1.0):
    return (RNG.standard_normal(shape).astype(np.float32) * np.float32(scale)).ravel()


@pytest.fixture(scope="module")
def ops(slm, ctx):
    return slm.Ops(ctx)


def close(got, want, atol=2e-5, rtol=1e-4):
    np.testing.assert_allclose(got, want, atol=atol, rtol=rtol)


@pytest.mark.parametrize("rows,cols,m", [(96, 32, 1), (2304, 768, 1), (768, 3072, 3), (6144, 768, 8),
                                         (2304, 768, 17), (768, 768, 256), (5, 7, 3), (32000, 768, 1),
                                         (12, 768, 1), (130, 36, 70), (768, 3072, 64), (32000, 768, 40),
                                         (100, 64, 33), (2048, 768, 9)])
def test_linear(ops, oracle, rows, cols, m):
    w, x = rand(rows, cols, scale=0.02), rand(m, cols)
    y = ops.zeros(1)
    ops.linear(y, ops.upload(w), rows, cols, ops.upload(x), m)
    close(y.read(m * rows), oracle.linear(w.reshape(rows, cols), x, m), atol=1e-5)


def test_linear_reads_at_an_offset(ops, oracle):
    rows, cols, m = 64, 32, 2
    w, x = rand(rows, cols), rand(m * cols + 32)
    y = ops.zeros(1)
    ops.linear(y, ops.upload(w), rows, cols, (ops.upload(x), 32), m)
    close(y.read(m * rows), oracle.linear(w.reshape(rows, cols), x[32:], m))


@pytest.mark.parametrize("groups,size", [(1, 768), (5, 768), (48, 64), (3, 8), (2, 100)])
def test_rms(ops, oracle, groups, size):
    x, w = rand(groups * size), rand(size)
    y = ops.zeros(1)
    ops.rms(y, ops.upload(x), ops.upload(w), groups, size, 1e-6)
    close(y.read(groups * size), oracle.rms(x, w, groups, size, 1e-6))


def test_silu_mul(ops, oracle):
    g, u = rand(5000, scale=4), rand(5000)
    y = ops.zeros(1)
    ops.silu_mul(y, ops.upload(g), ops.upload(u), 5000)
    close(y.read(5000), oracle.silu_mul(g, u))


@pytest.mark.parametrize("pos,m,heads,dh", [(0, 1, 4, 8), (5000, 3, 12, 64), (4095, 256, 12, 64)])
def test_rope_table_and_rope(ops, oracle, pos, m, heads, dh):
    half = dh // 2
    inv = np.array([1.0 / math.pow(10000.0, (2 * i) / dh) for i in range(half)], dtype=np.float32)
    c, s = ops.zeros(1), ops.zeros(1)
    ops.rope_table(c, s, ops.upload(inv), pos, m, half)
    wc, ws = oracle.rope_table(inv, pos, m, half)
    close(c.read(m * half), wc, atol=2e-6, rtol=0)
    close(s.read(m * half), ws, atol=2e-6, rtol=0)
    x = rand(m * heads * dh)
    y = ops.zeros(1)
    ops.rope(y, ops.upload(x), ops.upload(wc), ops.upload(ws), m, heads, dh)
    close(y.read(m * heads * dh), oracle.rope(x, wc, ws, m, heads, dh))


def test_l2norm(ops, oracle):
    x = rand(37 * 64)
    x[:64] = 0  # the 1e-12 clamp
    y = ops.zeros(1)
    ops.l2norm(y, ops.upload(x), 37, 64)
    close(y.read(37 * 64), oracle.l2norm(x, 37, 64))


# Head size 64 with m >= 32 takes the chunked kernel (64-token sub-chunks,
# ragged last ones included); other m >= 8 with head size 32/64/128 the
# column-parallel one; the rest the per-head kernel.
@pytest.mark.parametrize("m,heads,dh", [(1, 12, 64), (37, 4, 8), (256, 12, 64), (5, 2, 128), (100, 12, 64),
                                        (40, 3, 32), (33, 2, 128), (8, 1, 64), (32, 2, 64), (64, 3, 64),
                                        (65, 2, 64), (129, 1, 64), (300, 4, 64)])
def test_gla(ops, oracle, m, heads, dh):
    n = m * heads * dh
    q, k, v = rand(n, scale=0.2), rand(n, scale=0.2), rand(n)
    dec, bias = rand(m * heads), rand(heads)
    s0 = rand(heads * dh * dh, scale=0.1)
    sd = ops.upload(s0)
    y = ops.zeros(1)
    ops.gla(y, sd, ops.upload(q), ops.upload(k), ops.upload(v), ops.upload(dec), ops.upload(bias), m, heads, dh)
    s_cpu = s0.copy()
    want = oracle.gla(s_cpu, q, k, v, dec, bias, m, heads, dh)
    close(y.read(n), want, atol=1e-4)
    close(sd.read(heads * dh * dh), s_cpu, atol=1e-4)


def test_gla_extreme_decays(ops, oracle):
    # Decays near 1 (z = -12), near 0 (z = +30) and exactly 0 (z = +100:
    # e^z overflows) in long runs, so the chunked kernel's running log-decay
    # reaches its clamp and spans a wide range within a sub-chunk.
    m, heads, dh = 256, 4, 64
    n = m * heads * dh
    q, k, v = rand(n, scale=0.2), rand(n, scale=0.2), rand(n)
    z = np.where(np.arange(m * heads) % 7 == 0, 30.0, -12.0).astype(np.float32)
    z[5 * heads:6 * heads] = 100.0
    dec, bias = z, np.zeros(heads, dtype=np.float32)
    s0 = rand(heads * dh * dh, scale=0.1)
    sd = ops.upload(s0)
    y = ops.zeros(1)
    ops.gla(y, sd, ops.upload(q), ops.upload(k), ops.upload(v), ops.upload(dec), ops.upload(bias), m, heads, dh)
    s_cpu = s0.copy()
    want = oracle.gla(s_cpu, q, k, v, dec, bias, m, heads, dh)
    close(y.read(n), want, atol=1e-4)
    close(sd.read(heads * dh * dh), s_cpu, atol=1e-4)


def test_store_wraps_the_ring(ops, oracle):
    heads, dh, cap, m, pos = 3, 8, 10, 7, 6
    src = rand(m * heads * dh)
    cache0 = rand(heads * cap * dh)
    c = ops.upload(cache0)
    ops.store(c, ops.upload(src), pos, m, cap, heads, dh)
    want = cache0.copy()
    oracle.store(want, src, pos, m, cap, heads, dh)
    np.testing.assert_array_equal(c.read(heads * cap * dh), want)


ATTN_CASES = [
    # pos, m, reach, gap, cap, heads, key_heads, dh
    (0, 1, 8, 0, 264, 4, 4, 8),           # first token
    (4200, 1, 4096, 0, 4352, 12, 12, 64),  # full window, ring wrapped
    (4200, 8, 4096, 0, 4352, 12, 12, 64),
    (100, 17, 64, 0, 320, 12, 12, 64),     # tile path, window cuts in
    (3840, 256, 4096, 0, 4352, 12, 12, 64),
    (30, 5, None, 8, 64, 4, 2, 8),         # global: unbounded reach, far gap, GQA
    (3, 4, None, 8, 64, 4, 2, 8),          # every query sees nothing: zeros
    (20, 40, None, 8, 64, 8, 4, 16),       # some queries see nothing
    (9000, 1, None, 4096, 16384, 12, 4, 64),
    (50, 3, 40, 0, 300, 2, 1, 256),        # the largest head size
    (4200, 256, 4096, 0, 4352, 12, 12, 64),  # 64-query tiles over a wrapped ring
    (9000, 256, None, 4096, 16384, 12, 4, 64),  # global, far gap, GQA
    (3, 100, None, 8, 300, 4, 2, 64),      # the first queries see nothing; ragged last tile
    (500, 70, 48, 0, 304, 3, 3, 64),       # short window inside one tile
]


@pytest.mark.parametrize("pos,m,reach,gap,cap,heads,kh,dh", ATTN_CASES)
def test_attend(ops, oracle, pos, m, reach, gap, cap, heads, kh, dh):
    q = rand(m * heads * dh)
    k, v = rand(kh * cap * dh), rand(kh * cap * dh)
    scale = 1.0 / math.sqrt(dh)
    y, scores = ops.zeros(1), ops.zeros(1)
    ops.attend(y, scores, ops.upload(q), ops.upload(k), ops.upload(v), pos=pos, m=m, reach=reach, gap=gap, cap=cap,
               heads=heads, key_heads=kh, dh=dh, scale=scale)
    want = oracle.attend(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, scale)
    close(y.read(m * heads * dh), want, atol=2e-5)


@pytest.mark.parametrize("growth", [4.0, 6.5])
def test_attend_with_scores_growing_along_the_window(ops, oracle, growth):
    # Scores step up by `growth` nats every 64 positions (four steps, then
    # back down), so a query's running max grows across the first tiles of
    # its slice: the tensor-core pass rescales the output it holds in tensor
    # memory (each tile at 6.5 nats, every other at 4, when the max has moved
    # past 2^8).
    pos, m, reach, gap, cap, heads, kh, dh = 3840, 256, 4096, 0, 4352, 2, 2, 64
    scale = 0.125
    qv = rand(dh)
    qv *= np.float32(8.0 / np.linalg.norm(qv))  # |q| = 8: score = scale·|q|·(k along q)
    q = (np.tile(qv, m * heads) + rand(m * heads * dh, scale=0.05)).astype(np.float32)
    level = growth * ((np.arange(cap) // 64) % 4)  # slot = position: no wrap below 4352
    k1 = (level[:, None] * (qv / 8.0)[None, :] / np.float32(scale * 8.0)).astype(np.float32)
    k = (np.tile(k1.ravel(), kh) + rand(kh * cap * dh, scale=0.1)).astype(np.float32)
    v = rand(kh * cap * dh)
    y, scores = ops.zeros(1), ops.zeros(1)
    ops.attend(y, scores, ops.upload(q), ops.upload(k), ops.upload(v), pos=pos, m=m, reach=reach, gap=gap, cap=cap,
               heads=heads, key_heads=kh, dh=dh, scale=scale)
    want = oracle.attend(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, scale)
    close(y.read(m * heads * dh), want, atol=2e-5)


def test_attend_reads_q_at_an_odd_offset(ops, oracle):
    # q at a view offset that is not a multiple of 4 floats: staged, not faulted.
    pos, m, reach, gap, cap, heads, kh, dh = 300, 20, 64, 0, 320, 4, 4, 64
    q = rand(m * heads * dh + 3)
    k, v = rand(kh * cap * dh), rand(kh * cap * dh)
    y, scores = ops.zeros(1), ops.zeros(1)
    ops.attend(y, scores, (ops.upload(q), 3), ops.upload(k), ops.upload(v), pos=pos, m=m, reach=reach, gap=gap,
               cap=cap, heads=heads, key_heads=kh, dh=dh, scale=0.125)
    want = oracle.attend(q[3:], k, v, pos, m, reach, gap, cap, heads, kh, dh, 0.125)
    close(y.read(m * heads * dh), want, atol=2e-5)


def test_small_ops(ops, oracle):
    d, m = 16, 5
    w = rand(11 * d)
    y = ops.zeros(1)
    ids = np.array([3, 0, 10, 3, 7], dtype=np.uint32)
    ops.gather(y, ops.upload(w), ids, d)
    np.testing.assert_array_equal(y.read(m * d), w.reshape(11, d)[ids].ravel())
    x = rand(m * d + 4)
    xb = ops.upload(x)
    ops.copy(y, (xb, 4), m * d)
    np.testing.assert_array_equal(y.read(m * d), x[4:])
    first = rand(d)
    ops.shift(y, ops.upload(first), (xb, 4), m, d)
    np.testing.assert_array_equal(y.read(m * d), np.concatenate([first, x[4:4 + (m - 1) * d]]))
    ops.columns(y, xb, 3, 6, 2, 3)
    np.testing.assert_array_equal(y.read(9), np.concatenate([x[i * 6 + 2:i * 6 + 5] for i in range(3)]))
    a, b = rand(m * d), rand(m * d)
    ops.add(y, ops.upload(a), ops.upload(b), m * d)
    np.testing.assert_array_equal(y.read(m * d), a + b)
    row = rand(d)
    ops.add_row(y, ops.upload(a), ops.upload(row), m, d)
    np.testing.assert_array_equal(y.read(m * d), (a.reshape(m, d) + row).ravel())
    f = rand(m)
    ops.scale_rows(y, ops.upload(a), f, d)
    np.testing.assert_array_equal(y.read(m * d), (a.reshape(m, d) * f[:, None]).ravel())
    ops.mix(y, ops.upload(a), ops.upload(b), m * d, 0.25)
    np.testing.assert_allclose(y.read(m * d), a + np.float32(0.25) * (b - a), rtol=1e-6, atol=1e-7)


def test_bad_shapes_are_errors(slm, ops):
    small = ops.zeros(4)
    with pytest.raises(slm.SlmError):
        ops.linear(ops.zeros(1), small, 8, 8, small, 1)
    with pytest.raises(slm.SlmError):
        ops.gather(ops.zeros(1), small, [9], 4)
