"""ctypes front end of the reference CUDA baseline (_ref/libslm_refcuda.so).

BASELINE AND TEST INFRASTRUCTURE ONLY: the reference's own kernels
(kernels/slm.cu, built from source into _ref/slm.ptx by `make -C oracle ref`,
JIT-compiled by the driver) driven by a C++ restatement of the reference's
src/cuda.rs and src/model.rs (ref_cuda.cpp).  The parity tests use it to check
the restated oracle against the reference's GPU arithmetic, and bench.py times
it beside the product on the same GPU.  The product package never imports it.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from .oracle import read_config, read_safetensors

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
LIB_PATH = REF / "libslm_refcuda.so"
PTX_PATH = REF / "slm.ptx"

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_lib = None


def available() -> bool:
    """True when the PTX and the driver library have been built."""
    return LIB_PATH.exists() and PTX_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"{LIB_PATH} or {PTX_PATH} is missing: run `make -C oracle ref`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.rc_error.restype = ctypes.c_char_p
        L.rc_new.restype = _vp
        L.rc_new.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.rc_free.argtypes = [_vp]
        L.rc_counts.argtypes = [_vp, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong)]
        L.rc_model_new.restype = _vp
        L.rc_model_new.argtypes = [_vp, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _i64p, _f32p]
        L.rc_model_set.argtypes = [_vp, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int]
        L.rc_model_finish.argtypes = [_vp]
        L.rc_model_free.argtypes = [_vp]
        L.rc_session_new.restype = _vp
        L.rc_session_new.argtypes = [_vp, ctypes.c_int64]
        L.rc_session_free.argtypes = [_vp, _vp]
        L.rc_session_pos.restype = ctypes.c_int64
        L.rc_session_pos.argtypes = [_vp]
        L.rc_feed.argtypes = [_vp, _vp, _u32p, ctypes.c_int64, ctypes.c_int64]
        L.rc_step.argtypes = [_vp, _vp, ctypes.c_uint32]
        L.rc_logits.argtypes = [_vp, _vp, _f32p]
        L.rc_sync.argtypes = [_vp]
        _lib = L
    return _lib


def _check(code: int) -> None:
    if code != 0:
        raise RuntimeError(lib().rc_error().decode())


class Backend:
    """Cuda::probe (src/cuda.rs:73-120): the module loaded on one device."""

    def __init__(self, device: int = 0):
        L = lib()
        self._free = L.rc_free
        self._h = L.rc_new(str(PTX_PATH).encode(), device)
        if not self._h:
            raise RuntimeError(L.rc_error().decode())

    def counts(self) -> tuple[int, int]:
        """Kernel launches and host synchronisations so far."""
        a, b = ctypes.c_longlong(), ctypes.c_longlong()
        lib().rc_counts(self._h, ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value

    def sync(self) -> None:
        _check(lib().rc_sync(self._h))

    def close(self):
        if getattr(self, "_h", None):
            self._free(self._h)
            self._h = None

    __del__ = close


class Model:
    """Model::load (src/model.rs:226-269) on the reference CUDA backend."""

    def __init__(self, backend: Backend, folder, tensors: dict | None = None, cfg: dict | None = None):
        L = lib()
        self.backend = backend
        folder = Path(folder) if folder is not None else None
        self.cfg = cfg if cfg is not None else read_config(folder / "config.json")
        c = self.cfg
        tensors = tensors if tensors is not None else read_safetensors(folder / "model.safetensors")
        ints = np.array([c["vocab_size"], c["d_model"], c["n_heads"], c["global_kv_heads"], c["window"],
                         c["max_loops"], c["default_loops"], c["global_logn"], c["global_kshift"],
                         c["global_emb"], c["global_far"]], dtype=np.int64)
        floats = np.array([c["damp"], c["rope_base"], c["norm_eps"]], dtype=np.float32)
        self._free = L.rc_model_free
        self._h = L.rc_model_new(backend._h, c["prelude"].encode(), c["core"].encode(), c["coda"].encode(),
                                 ints.ctypes.data_as(_i64p), floats.ctypes.data_as(_f32p))
        for name, t in tensors.items():
            t = np.ascontiguousarray(t, dtype=np.float32)
            shape = np.array(t.shape, dtype=np.int64)
            _check(L.rc_model_set(self._h, name.encode(), t.ctypes.data_as(_f32p), shape.ctypes.data_as(_i64p),
                                  t.ndim))
        _check(L.rc_model_finish(self._h))
        self.vocab = c["vocab_size"]

    def session(self, loops: int | None = None) -> "Session":
        return Session(self, loops)

    def close(self):
        if getattr(self, "_h", None):
            self._free(self._h)
            self._h = None

    __del__ = close


class Session:
    def __init__(self, model: Model, loops: int | None):
        L = lib()
        self.model = model
        self._free = L.rc_session_free
        self._h = L.rc_session_new(model._h, loops or 0)
        if not self._h:
            raise RuntimeError(L.rc_error().decode())

    @property
    def pos(self) -> int:
        return lib().rc_session_pos(self._h)

    def feed(self, ids, limit: int = 256) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        _check(lib().rc_feed(self.model._h, self._h, ids.ctypes.data_as(_u32p), len(ids), limit))

    def step(self, token: int) -> None:
        _check(lib().rc_step(self.model._h, self._h, int(token)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.model.vocab, dtype=np.float32)
        _check(lib().rc_logits(self.model._h, self._h, out.ctypes.data_as(_f32p)))
        return out

    def close(self):
        if getattr(self, "_h", None):
            self._free(self.model._h, self._h)
            self._h = None

    __del__ = close
