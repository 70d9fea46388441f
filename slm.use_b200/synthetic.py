"""Seeded random-init models in the reference's on-disk format.

No checkpoint of the 86M-class model is available offline, so the benchmark
and the large parity tests run on models written here: config.json with the
fields of the reference's Config (src/config.rs:22-52) and an f32
model.safetensors with the tensor names Model::load and Block::load read
(src/model.rs:114-153, 236-251).  Matrices are N(0, 0.02); norm weights are 1
and the decay bias 0 (no published initialisation exists).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

# The 86M-class shape of the benchmark (d 768, 12 heads × 64, FFN 3072,
# vocab 32000, window 4096, layout S | LS | S).
BASE = dict(vocab_size=32000, d_model=768, n_heads=12, hidden=3072, prelude="S", core="LS", coda="S",
            window=4096, max_loops=16, default_loops=4, rope_base=10000.0, norm_eps=1e-6, damp=1.0,
            global_kv_heads=4, global_logn=0, global_kshift=0, global_emb=0, global_far=0)

# The global-attention variant (layout S | LS | SG, with the tiny fixture's
# G options).
GLOBAL = dict(BASE, coda="SG", global_logn=16, global_kshift=1, global_emb=1, global_far=1)


def tensor_shapes(cfg: dict) -> dict[str, tuple]:
    d, h, f, v = cfg["d_model"], cfg["n_heads"], cfg["hidden"], cfg["vocab_size"]
    dh = d // h
    kd = cfg["global_kv_heads"] * dh
    shapes: dict[str, tuple] = {}

    def block(prefix: str, kind: str) -> None:
        if kind == "S":
            shapes[f"{prefix}.mixer.qkv.weight"] = (3 * d, d)
        elif kind == "L":
            shapes[f"{prefix}.mixer.qkvg.weight"] = (4 * d, d)
            shapes[f"{prefix}.mixer.decay.weight"] = (h, d)
            shapes[f"{prefix}.mixer.decay.bias"] = (h,)
            shapes[f"{prefix}.mixer.head_norm.weight"] = (dh,)
        elif kind == "G":
            shapes[f"{prefix}.mixer.q.weight"] = (d, d)
            shapes[f"{prefix}.mixer.kv.weight"] = (2 * kd, d)
            if cfg["global_emb"]:
                shapes[f"{prefix}.mixer.norm_e.weight"] = (d,)
        else:
            raise ValueError(f"unknown layer type {kind}")
        shapes[f"{prefix}.mixer.o.weight"] = (d, d)
        shapes[f"{prefix}.norm1.weight"] = (d,)
        shapes[f"{prefix}.norm2.weight"] = (d,)
        shapes[f"{prefix}.mlp.up.weight"] = (2 * f, d)
        shapes[f"{prefix}.mlp.down.weight"] = (d, f)

    for part in ("prelude", "core", "coda"):
        for i, kind in enumerate(cfg[part]):
            block(f"{part}.{i}", kind)
    if cfg["core"]:
        shapes["inject_e.weight"] = (d, d)
        shapes["loop_embed.weight"] = (cfg["max_loops"], d)
    shapes["embed.weight"] = (v, d)
    shapes["norm_f.weight"] = (d,)
    return shapes


def make_tensors(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(tensor_shapes(cfg)):
        shape = tensor_shapes(cfg)[name]
        if name.endswith("norm1.weight") or name.endswith("norm2.weight") or "norm" in name.split(".")[-2]:
            out[name] = np.ones(shape, dtype=np.float32)
        elif name.endswith("decay.bias"):
            out[name] = np.zeros(shape, dtype=np.float32)
        else:
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return out


def write_safetensors(path, tensors: dict[str, np.ndarray]) -> None:
    header = {}
    offset = 0
    for name, t in tensors.items():
        n = t.size * 4
        header[name] = {"dtype": "F32", "shape": list(t.shape), "data_offsets": [offset, offset + n]}
        offset += n
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for t in tensors.values():
            f.write(np.ascontiguousarray(t, dtype="<f4").tobytes())


def write_model(folder, cfg: dict, seed: int = 0) -> Path:
    """Writes config.json + model.safetensors; returns the folder."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    conf = {k: v for k, v in cfg.items() if k != "hidden"}
    conf.update(loop_lora=0, state_loops=0, global_rope_base=0.0)
    (folder / "config.json").write_text(json.dumps(conf, indent=1))
    write_safetensors(folder / "model.safetensors", make_tensors(cfg, seed))
    return folder


def scaled(cfg: dict, **kw) -> dict:
    """A copy of cfg with some fields replaced (small test shapes)."""
    c = dict(cfg)
    c.update(kw)
    return c
