"""The reference CUDA backend on the GPU: its own kernels (kernels/slm.cu built
from source into oracle/_ref/slm.ptx, JIT-compiled by the driver) under the C++
restatement of its host side (oracle/ref_cuda.cpp).

* The reference's own `cuda_matches_reference` test (tests/parity.rs:15-60):
  the tiny fixture, token by token and at nine chunk splits, within 1e-4 of
  the stored PyTorch logits and with the same arg-max.  This pins the
  restated host side (launch shapes, views, ring arithmetic) on the
  reference's own GPU arithmetic.
* Synthetic models (every layer type, a global cache that grows through the
  host) against the CPU oracle.
* This library against the reference CUDA backend on the 86M-class shapes.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import SPLITS, TINY, TOLERANCE, load_pkg, run_split

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rc():
    from oracle import ref_cuda
    if not ref_cuda.available():
        pytest.skip("reference CUDA baseline not built (make -C oracle ref)")
    return ref_cuda


@pytest.fixture(scope="module")
def backend(rc):
    b = rc.Backend(0)
    yield b
    b.close()


def _synthetic(tmp_path_factory, name, base, **kw):
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(getattr(syn, base), **kw)
    return syn.write_model(tmp_path_factory.mktemp(name), cfg, seed=5)


@pytest.mark.parametrize("split,chunk", [(0, 1)] + SPLITS)
def test_reference_cuda_matches_fixture(rc, backend, golden, split, chunk):
    model = rc.Model(backend, TINY)
    checked, md, same = run_split(lambda loops: model.session(loops), golden, split, chunk)
    assert checked == (40 if split == 0 else 41 - split)
    assert md < TOLERANCE, (split, chunk, md)
    assert same, (split, chunk)


def _compare(a, b, ids, limit, steps):
    a.feed(ids, limit)
    b.feed(ids, limit)
    worst = float(np.abs(a.logits() - b.logits()).max())
    tok = int(np.argmax(b.logits()))
    for _ in range(steps):
        a.step(tok)
        b.step(tok)
        la, lb = a.logits(), b.logits()
        worst = max(worst, float(np.abs(la - lb).max()))
        tok = int(np.argmax(lb))
    return worst


def test_reference_cuda_matches_oracle_on_synthetic_models(rc, backend, oracle, tmp_path_factory):
    load_pkg()
    small = _synthetic(tmp_path_factory, "rc_small", "BASE", vocab_size=1000, d_model=128, n_heads=2, hidden=256,
                       window=48, max_loops=4, default_loops=3)
    ids = np.random.default_rng(0).integers(0, 1000, 300)
    assert _compare(rc.Model(backend, small).session(), oracle.Model(small).session(), ids, 64, 10) < 2e-4
    small_g = _synthetic(tmp_path_factory, "rc_small_g", "GLOBAL", vocab_size=500, d_model=64, n_heads=4,
                         hidden=128, window=16, max_loops=3, default_loops=2, global_kv_heads=2)
    # 8192 global slots first (src/model.rs:320): 8250 positions make the cache grow once.
    ids = np.random.default_rng(2).integers(0, 500, 8250)
    assert _compare(rc.Model(backend, small_g).session(1), oracle.Model(small_g).session(1), ids, 256, 5) < 5e-4


def test_library_matches_reference_cuda_on_86m_shapes(rc, backend, ctx, tmp_path_factory):
    slm = load_pkg()
    folder = _synthetic(tmp_path_factory, "rc_m86", "BASE", window=128)
    ids = np.random.default_rng(4).integers(0, 32000, 300)
    worst = _compare(slm.Model(ctx, folder).session(2), rc.Model(backend, folder).session(2), ids, 256, 8)
    assert worst < 1e-3, worst
