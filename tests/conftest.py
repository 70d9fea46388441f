"""Shared fixtures.  `-m gpu` tests need an sm_100 device; the rest run on CPU."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
TINY = GOLDEN / "tiny"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def load_pkg():
    """Imports the package folder `slm.use_b200` as module `slm_b200`."""
    if "slm_b200" in sys.modules:
        return sys.modules["slm_b200"]
    pkg = ROOT / "slm.use_b200"
    spec = importlib.util.spec_from_file_location("slm_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["slm_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def slm():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    return O


@pytest.fixture(scope="session")
def ctx(slm):
    c = slm.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def golden(oracle):
    e = oracle.read_safetensors(TINY / "expected.safetensors")
    return {"tokens": e["tokens"].astype(np.uint32), "loops": int(e["loops"][0]),
            "positions": e["positions"].astype(np.int64), "logits": e["logits"]}


# (split, chunk) pairs of the reference's parity test (tests/parity.rs:15-46).
SPLITS = [(1, 1), (5, 2), (8, 8), (9, 3), (20, 7), (30, 16), (39, 256), (40, 5), (40, 40)]
TOLERANCE = 1e-4  # tests/parity.rs:13


def run_split(session_factory, golden, split, chunk):
    """verify::run_split (src/verify.rs:79-119): max |Δlogit| and same-argmax tally."""
    toks, logits = golden["tokens"], golden["logits"]
    se = session_factory(golden["loops"])
    md, same, checked = 0.0, True, 0

    def check(got, want):
        nonlocal md, same, checked
        md = max(md, float(np.abs(got - want).max()))
        same &= int(np.argmax(got)) == int(np.argmax(want))
        checked += 1

    if split > 0:
        se.feed(toks[:split], chunk)
        check(se.logits(), logits[split - 1])
    for t in range(split, len(toks)):
        se.step(int(toks[t]))
        check(se.logits(), logits[t])
    return checked, md, same
