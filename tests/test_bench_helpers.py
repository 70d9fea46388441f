"""bench.py's bookkeeping on CPU: algorithmic bytes and flops of the C2
workload (restated from the model shapes) and the phase list of the
persistent step (42 phases at R = 4 for S | LS | S with fused MLPs, 52 with
two-phase MLPs)."""
from __future__ import annotations

import sys

import numpy as np

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
    two = b.phase_kinds(syn.BASE, 4, fused=False)
    assert len(two) == 52 and two[0] == "S1" and two[5] == "inject" and two[-1] == "logits"
    assert len(b.phase_kinds(syn.GLOBAL, 4, fused=False)) == 57
    assert two.count("attn") == 6 and two.count("gla") == 4
    # Fused MLPs: one phase per block fewer (10 blocks at R = 4); o in the
    # attention / GLA phase of the 6 S and 4 L blocks: 10 fewer again.
    mlp = b.phase_kinds(syn.BASE, 4, attn_o=False)
    assert len(mlp) == 42 and mlp[4] == "inject" and mlp.count("mlp") == 10
    kinds = b.phase_kinds(syn.BASE, 4)
    assert len(kinds) == 32 and kinds[3] == "inject" and kinds.count("o") == 0 and kinds.count("attn") == 6
    assert b.trace_kinds(np.zeros((32, 3, 8), dtype=np.int64), syn.BASE, 4) == kinds
    assert b.trace_kinds(np.zeros((42, 3, 8), dtype=np.int64), syn.BASE, 4) == mlp
    assert b.trace_kinds(np.zeros((52, 3, 8), dtype=np.int64), syn.BASE, 4) == two
    assert b.trace_kinds(np.zeros((7, 3, 8), dtype=np.int64), syn.BASE, 4) is None
