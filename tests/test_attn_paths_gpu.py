"""Both slice passes for prefill-sized attention (head size 64, m > 8) against
the oracle: the tensor-core pass (the default) runs in this process through
test_ops_gpu.py; the FP32 flash-tile pass, which SLM_ATTN_TC=0 selects (read
once, at the first attention call), runs here in a child process on the same
kinds of cases."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import math, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from conftest import load_pkg
from oracle import oracle as O
slm = load_pkg()
ctx = slm.Context(0)
ops = slm.Ops(ctx)
rng = np.random.default_rng(7)
cases = [(3840, 256, 4096, 0, 4352, 12, 12, 64), (4200, 256, 4096, 0, 4352, 12, 12, 64),
         (9000, 256, None, 4096, 16384, 12, 4, 64), (3, 100, None, 8, 300, 4, 2, 64), (100, 17, 64, 0, 320, 12, 12, 64)]
for pos, m, reach, gap, cap, heads, kh, dh in cases:
    q = rng.standard_normal(m * heads * dh).astype(np.float32)
    k = rng.standard_normal(kh * cap * dh).astype(np.float32)
    v = rng.standard_normal(kh * cap * dh).astype(np.float32)
    y, scores = ops.zeros(1), ops.zeros(1)
    ops.attend(y, scores, ops.upload(q), ops.upload(k), ops.upload(v), pos=pos, m=m, reach=reach, gap=gap, cap=cap,
               heads=heads, key_heads=kh, dh=dh, scale=1.0 / math.sqrt(dh))
    want = O.attend(q, k, v, pos, m, reach, gap, cap, heads, kh, dh, 1.0 / math.sqrt(dh))
    np.testing.assert_allclose(y.read(m * heads * dh), want, atol=2e-5, rtol=1e-4)
ctx.close()
print("ok")
"""


def test_flash_tile_pass_matches_oracle():
    env = dict(os.environ, SLM_ATTN_TC="0")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT / "tests")], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.strip().endswith("ok")
