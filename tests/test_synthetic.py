"""Synthetic models are written in the reference's format (CPU only)."""
import numpy as np

from conftest import load_pkg


def test_synthetic_round_trip(tmp_path, oracle):
    syn = load_pkg().synthetic if hasattr(load_pkg(), "synthetic") else __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(syn.GLOBAL, vocab_size=50, d_model=32, n_heads=4, hidden=48, window=8, max_loops=4,
                     default_loops=2, global_kv_heads=2)
    folder = syn.write_model(tmp_path / "m", cfg, seed=3)
    t = oracle.read_safetensors(folder / "model.safetensors")
    shapes = syn.tensor_shapes(cfg)
    assert {k: tuple(v.shape) for k, v in t.items()} == shapes
    assert np.all(t["norm_f.weight"] == 1) and np.all(t["core.0.mixer.decay.bias"] == 0)
    assert abs(float(t["embed.weight"].std()) - 0.02) < 0.005
    m = oracle.Model(folder)
    se = m.session()
    se.feed(np.arange(20) % 50, 7)
    assert np.isfinite(se.logits()).all()
