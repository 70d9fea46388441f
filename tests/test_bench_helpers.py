"""bench.py's bookkeeping on CPU: algorithmic bytes and flops of the C2
workload (SURVEY-style arithmetic restated from the model shapes) and the
phase list of the persistent step (52 phases at R = 4 for S | LS | S)."""
from __future__ import annotations

import sys

from conftest import ROOT, load_pkg


def _bench():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import bench
    return bench


def _syn():
    load_pkg()
    return __import__("slm_b200.synthetic").synthetic


def test_decode_bytes_of_the_86m_config():
    b, syn = _bench(), _syn()
    byts = b.decode_bytes(syn.BASE, 4)
    assert abs(byts["total"] / 1e6 - 640.4) < 0.1       # weights + KV + GLA state per token
    assert abs(b.decode_bytes(syn.BASE, 8)["total"] / 1e6 - 1054) < 1
    assert abs(b.decode_bytes(syn.BASE, 16)["total"] / 1e6 - 1882) < 1


def test_prefill_flops_of_the_86m_config():
    b, syn = _bench(), _syn()
    per_token = b.prefill_flops(syn.BASE, 4, 4096) / 4096
    assert abs(per_token / 1e9 - 0.233) < 0.001


def test_phase_kinds_match_the_plan_shape():
    b, syn = _bench(), _syn()
    kinds = b.phase_kinds(syn.BASE, 4)
    assert len(kinds) == 52 and kinds[0] == "S1" and kinds[5] == "inject" and kinds[-1] == "logits"
    assert len(b.phase_kinds(syn.GLOBAL, 4)) == 57
    assert kinds.count("attn") == 6 and kinds.count("gla") == 4
