"""The C ABI library loads and exports every symbol include/slm_b200.h
declares; on a machine without a GPU every call fails with a status, never a
crash (CPU only)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "slm_b200.h"


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(slm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_ops_trait():
    names = declared()
    # One entry point per method of the reference's Ops trait (src/ops.rs:68-228).
    for op in ("gather", "copy", "shift", "columns", "linear", "add", "add_row", "scale_rows", "mix", "rms",
               "silu_mul", "rope_table", "rope", "l2norm", "gla", "store", "attend"):
        assert f"slm_op_{op}" in names
    for f in ("slm_zeros", "slm_upload", "slm_read", "slm_flush", "slm_model_load", "slm_session_new", "slm_feed",
              "slm_step", "slm_logits", "slm_state_bytes", "slm_sample", "slm_decode", "slm_pick"):
        assert f in names


def test_library_exports_every_declared_symbol(slm):
    lib = slm.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header(slm):
    assert set(declared()) <= set(slm._SIGS)


def test_calls_fail_with_a_status_without_a_gpu(slm):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert slm.device_count() == 0
    with pytest.raises(slm.SlmError) as e:
        slm.Context(0)
    assert e.value.code in (1, 2)
    assert slm.lib().slm_last_error()


def test_null_arguments_are_rejected(slm):
    lib = slm.lib()
    assert lib.slm_ctx_new(0, None) == 1
    assert lib.slm_model_load(None, b"x", None) == 1
    assert lib.slm_feed(None, None, 0, 1) == 1
    assert b"null" in lib.slm_last_error() or b"bad" in lib.slm_last_error()


def test_rng_seed_matches_the_reference(slm, oracle):
    for seed in (0, 1, 7, 2**63 + 5):
        assert slm.rng_seed(seed) == oracle.rng_new(seed)
