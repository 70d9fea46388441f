"""ctypes front end of the CPU oracle (liboracle.so, built from slm_oracle.cpp).

TEST INFRASTRUCTURE ONLY.  The parity tests, `__graft_entry__.smoke()` and the
CPU-baseline leg of `bench.py` use it as the checker; the product package never
imports it.  It mirrors the reference's model-level API (src/model.rs:
Model::load / session / feed / step / logits / state_bytes) and its sampler
(src/sample.rs: pick, Rng), plus one function per `Ops` method for op-level
parity tests.
"""
from __future__ import annotations

import ctypes
import json
import struct
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_lib = None


def build() -> None:
    """Compiles liboracle.so with the Makefile beside this file."""
    import subprocess

    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_error.restype = ctypes.c_char_p
        L.orc_model_new.restype = ctypes.c_void_p
        L.orc_model_new.argtypes = [ctypes.c_char_p] * 3 + [_i64p, _f32p]
        L.orc_model_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int]
        L.orc_model_finish.argtypes = [ctypes.c_void_p]
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_session_new.restype = ctypes.c_void_p
        L.orc_session_new.argtypes = [ctypes.c_void_p, ctypes.c_int64]
        L.orc_session_free.argtypes = [ctypes.c_void_p]
        L.orc_session_pos.restype = ctypes.c_int64
        L.orc_session_pos.argtypes = [ctypes.c_void_p]
        L.orc_feed.argtypes = [ctypes.c_void_p, _u32p, ctypes.c_int64, ctypes.c_int64]
        L.orc_step.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.orc_logits.argtypes = [ctypes.c_void_p, _f32p]
        L.orc_state_bytes.restype = ctypes.c_int64
        L.orc_state_bytes.argtypes = [ctypes.c_void_p]
        L.orc_session_fill.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64]
        L.orc_state_count.restype = ctypes.c_int64
        L.orc_state_count.argtypes = [ctypes.c_void_p]
        L.orc_state_info.restype = _f32p
        L.orc_state_info.argtypes = [ctypes.c_void_p, ctypes.c_int64, _i64p]
        L.orc_pick.restype = ctypes.c_uint32
        L.orc_pick.argtypes = [_f32p, ctypes.c_int64, _u32p, ctypes.c_int64, ctypes.c_float,
                               ctypes.c_uint32, ctypes.c_float, ctypes.c_float, ctypes.c_uint32, _u64p]
        L.orc_rng_new.restype = ctypes.c_uint64
        L.orc_rng_new.argtypes = [ctypes.c_uint64]
        L.orc_rng_next.restype = ctypes.c_float
        L.orc_rng_next.argtypes = [_u64p]
        L.orc_threads.restype = ctypes.c_int
        L.orc_threads.argtypes = [ctypes.c_int]
        i64, f32, vp = ctypes.c_int64, ctypes.c_float, _f32p
        L.orc_linear.argtypes = [vp, vp, i64, i64, vp, i64]
        L.orc_rms.argtypes = [vp, vp, vp, i64, i64, f32]
        L.orc_silu_mul.argtypes = [vp, vp, vp, i64]
        L.orc_rope_table.argtypes = [vp, vp, vp, i64, i64, i64]
        L.orc_rope.argtypes = [vp, vp, vp, vp, i64, i64, i64]
        L.orc_l2norm.argtypes = [vp, vp, i64, i64]
        L.orc_gla.argtypes = [vp] * 7 + [i64, i64, i64]
        L.orc_store.argtypes = [vp, vp, i64, i64, i64, i64, i64]
        L.orc_attend.argtypes = [vp, vp, vp, vp] + [i64] * 8 + [f32]
        L.orc_add.argtypes = [vp, vp, vp, i64]
        L.orc_add_row.argtypes = [vp, vp, vp, i64, i64]
        L.orc_scale_rows.argtypes = [vp, vp, vp, i64, i64]
        L.orc_mix.argtypes = [vp, vp, vp, i64, f32]
        _lib = L
    return _lib


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _up(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_u32p)


# ---------------------------------------------------------------------------
# safetensors (format only: 8-byte little-endian header size, JSON header,
# raw little-endian tensors)
# ---------------------------------------------------------------------------

def read_safetensors(path) -> dict[str, np.ndarray]:
    raw = Path(path).read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    out = {}
    base = 8 + n
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        if meta["dtype"] != "F32":
            raise ValueError(f"{name}: expected f32 weights")
        a, b = meta["data_offsets"]
        out[name] = np.frombuffer(raw[base + a:base + b], dtype="<f4").reshape(meta["shape"]).copy()
    return out


def read_config(path) -> dict:
    """config.json with the reference's defaults and checks (src/config.rs:22-80)."""
    cfg = json.loads(Path(path).read_text())
    cfg.setdefault("global_kv_heads", 4)
    cfg.setdefault("damp", 1.0)
    for key in ("global_logn", "global_kshift", "global_emb", "global_far", "loop_lora", "state_loops"):
        cfg.setdefault(key, 0)
    cfg.setdefault("global_rope_base", 0.0)
    if cfg["loop_lora"]:
        raise ValueError("loop_lora models are not supported")
    if cfg["state_loops"]:
        raise ValueError("state_loops models are not supported")
    if cfg["global_rope_base"] != 0.0:
        raise ValueError("global_rope_base is not supported")
    return cfg


class Model:
    """Model::load (src/model.rs:226-269) from a folder with config.json and model.safetensors."""

    def __init__(self, folder, tensors: dict | None = None, cfg: dict | None = None):
        L = lib()
        folder = Path(folder) if folder is not None else None
        self.cfg = cfg if cfg is not None else read_config(folder / "config.json")
        c = self.cfg
        tensors = tensors if tensors is not None else read_safetensors(folder / "model.safetensors")
        ints = np.array([c["vocab_size"], c["d_model"], c["n_heads"], c["global_kv_heads"], c["window"],
                         c["max_loops"], c["default_loops"], c["global_logn"], c["global_kshift"],
                         c["global_emb"], c["global_far"]], dtype=np.int64)
        floats = np.array([c["damp"], c["rope_base"], c["norm_eps"]], dtype=np.float32)
        self._h = L.orc_model_new(c["prelude"].encode(), c["core"].encode(), c["coda"].encode(),
                                  ints.ctypes.data_as(_i64p), _fp(floats))
        for name, t in tensors.items():
            t = np.ascontiguousarray(t, dtype=np.float32)
            shape = np.array(t.shape, dtype=np.int64)
            L.orc_model_set(self._h, name.encode(), _fp(t), shape.ctypes.data_as(_i64p), t.ndim)
        if L.orc_model_finish(self._h) != 0:
            raise RuntimeError(L.orc_error().decode())

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.orc_model_free(self._h)
            self._h = None

    def session(self, loops: int | None = None) -> "Session":
        return Session(self, loops)


class Session:
    def __init__(self, model: Model, loops: int | None):
        self.model = model
        self.vocab = model.cfg["vocab_size"]
        h = lib().orc_session_new(model._h, loops or 0)
        if not h:
            raise ValueError(lib().orc_error().decode())
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.orc_session_free(self._h)
            self._h = None

    @property
    def pos(self) -> int:
        return lib().orc_session_pos(self._h)

    def feed(self, ids, limit: int = 256) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        if lib().orc_feed(self._h, _up(ids), len(ids), limit) != 0:
            raise ValueError(lib().orc_error().decode())

    def step(self, token: int) -> None:
        if lib().orc_step(self._h, int(token)) != 0:
            raise ValueError(lib().orc_error().decode())

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        lib().orc_logits(self._h, _fp(out))
        return out

    def state_bytes(self) -> int:
        return lib().orc_state_bytes(self._h)

    def fill(self, pos: int, seed: int = 0) -> None:
        lib().orc_session_fill(self._h, pos, seed)

    def state(self) -> list[dict]:
        """The state arrays in step order (S k, v; L s; G k, v, prev per block), each a dict with
        kind, part, cap and a copy of its values."""
        out = []
        info = np.zeros(4, dtype=np.int64)
        for i in range(lib().orc_state_count(self._h)):
            ptr = lib().orc_state_info(self._h, i, info.ctypes.data_as(_i64p))
            data = np.ctypeslib.as_array(ptr, shape=(int(info[3]),)).copy()
            out.append({"kind": chr(info[0]), "part": chr(info[1]), "cap": int(info[2]), "data": data})
        return out


def rng_new(seed: int) -> int:
    return lib().orc_rng_new(seed)


def pick(logits, recent, temperature=0.0, top_k=0, top_p=1.0, repeat_penalty=1.0,
         repeat_window=0, rng_state: list | None = None) -> int:
    """sample.rs:33-93; rng_state is a one-element list holding the xorshift64* state."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n = len(recent)
    recent = np.ascontiguousarray(recent if n else [0], dtype=np.uint32)
    st = ctypes.c_uint64(rng_state[0] if rng_state else rng_new(0))
    out = lib().orc_pick(_fp(logits), len(logits), _up(recent), n,
                         temperature, top_k, top_p, repeat_penalty, repeat_window, ctypes.byref(st))
    if rng_state is not None:
        rng_state[0] = st.value
    return int(out)


# ---------------------------------------------------------------------------
# Op level: one function per `Ops` method, on numpy arrays (src/cpu.rs)
# ---------------------------------------------------------------------------

def linear(w, x, m):
    rows, cols = w.shape
    y = np.empty(m * rows, dtype=np.float32)
    lib().orc_linear(_fp(y), _fp(w), rows, cols, _fp(x), m)
    return y


def rms(x, w, groups, size, eps):
    y = np.empty(groups * size, dtype=np.float32)
    lib().orc_rms(_fp(y), _fp(x), _fp(w), ctypes.c_int64(groups), ctypes.c_int64(size), ctypes.c_float(eps))
    return y


def silu_mul(g, u):
    y = np.empty(len(g), dtype=np.float32)
    lib().orc_silu_mul(_fp(y), _fp(g), _fp(u), ctypes.c_int64(len(g)))
    return y


def rope_table(inv, pos, m, half):
    c = np.empty(m * half, dtype=np.float32)
    s = np.empty(m * half, dtype=np.float32)
    lib().orc_rope_table(_fp(c), _fp(s), _fp(inv), ctypes.c_int64(pos), ctypes.c_int64(m), ctypes.c_int64(half))
    return c, s


def rope(x, c, s, m, heads, dh):
    y = np.empty(m * heads * dh, dtype=np.float32)
    lib().orc_rope(_fp(y), _fp(x), _fp(c), _fp(s), ctypes.c_int64(m), ctypes.c_int64(heads), ctypes.c_int64(dh))
    return y


def l2norm(x, heads, dh):
    y = np.empty(heads * dh, dtype=np.float32)
    lib().orc_l2norm(_fp(y), _fp(x), ctypes.c_int64(heads), ctypes.c_int64(dh))
    return y


def gla(s, q, k, v, decay, bias, m, heads, dh):
    """Returns y; updates the state s in place."""
    y = np.empty(m * heads * dh, dtype=np.float32)
    lib().orc_gla(_fp(y), _fp(s), _fp(q), _fp(k), _fp(v), _fp(decay), _fp(bias),
                  ctypes.c_int64(m), ctypes.c_int64(heads), ctypes.c_int64(dh))
    return y


def store(cache, src, pos, m, cap, heads, dh):
    lib().orc_store(_fp(cache), _fp(src), ctypes.c_int64(pos), ctypes.c_int64(m), ctypes.c_int64(cap),
                    ctypes.c_int64(heads), ctypes.c_int64(dh))


def attend(q, k, v, pos, m, reach, gap, cap, heads, key_heads, dh, scale):
    """reach None means unbounded (usize::MAX in the reference)."""
    y = np.empty(m * heads * dh, dtype=np.float32)
    lib().orc_attend(_fp(y), _fp(q), _fp(k), _fp(v), *[ctypes.c_int64(int(a)) for a in
                     (pos, m, reach or 0, gap, cap, heads, key_heads, dh)], ctypes.c_float(scale))
    return y
