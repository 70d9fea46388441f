"""Python host mirror of the B200 backend for the SLM.use token loop.

A thin ctypes layer over libslm_b200.so (C ABI in include/slm_b200.h).  Names,
argument meaning and errors follow the reference:

  * `Ops` — one method per method of the reference's `Ops` trait
    (src/ops.rs:68-228) on device buffers (`Buf`);
  * `Model` / `Session` — Model::load, session, feed, step, logits, state_bytes
    (src/model.rs:225-690);
  * `Sampling`, `rng_seed`, `Session.sample` — pick and Rng (src/sample.rs).

There is no CPU fallback: importing works anywhere, but every call needs the
library and an sm_100 GPU, and raises `SlmError` otherwise.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libslm_b200.so"
CHUNK = 256  # src/model.rs:27

_c = ctypes
_f32p = _c.POINTER(_c.c_float)
_u32p = _c.POINTER(_c.c_uint32)
_u64p = _c.POINTER(_c.c_uint64)
_vp = _c.c_void_p
_sz = _c.c_size_t

SLM_OPT_GRAPH = 1
SLM_OPT_MEGA = 2
SLM_OPT_TRACE = 3
SLM_OPT_TEST_STALL = 4
SLM_OPT_BF16 = 5
SLM_STAT_STEP_KERNELS, SLM_STAT_GRAPHS, SLM_STAT_MEGA, SLM_STAT_PHASES = 1, 2, 3, 4
SIZE_MAX = (1 << 64) - 1


class SlmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _Attn(_c.Structure):
    _fields_ = [(n, _sz) for n in ("pos", "m", "reach", "gap", "cap", "heads", "key_heads", "dh")] + [
        ("scale", _c.c_float)]


class _Sampling(_c.Structure):
    _fields_ = [("temperature", _c.c_float), ("top_k", _c.c_uint32), ("top_p", _c.c_float),
                ("repeat_penalty", _c.c_float), ("repeat_window", _c.c_uint32)]


class _StateArray(_c.Structure):
    _fields_ = [("kind", _c.c_char), ("part", _c.c_char)] + [(n, _sz) for n in ("heads", "cap", "dh", "floats")]


class _Info(_c.Structure):
    _fields_ = [(n, _sz) for n in ("vocab", "d_model", "heads", "head_dim", "kv_heads", "hidden", "window",
                                   "max_loops", "default_loops", "params")] + [
        ("prelude", _c.c_char * 32), ("core", _c.c_char * 32), ("coda", _c.c_char * 32)]


_lib = None

# name -> (restype, argtypes)
_SIGS = {
    "slm_last_error": (_c.c_char_p, []),
    "slm_version": (_c.c_char_p, []),
    "slm_device_count": (_c.c_int, [_c.POINTER(_c.c_int)]),
    "slm_ctx_new": (_c.c_int, [_c.c_int, _c.POINTER(_vp)]),
    "slm_ctx_free": (_c.c_int, [_vp]),
    "slm_ctx_name": (_c.c_int, [_vp, _c.c_char_p, _sz]),
    "slm_ctx_sync": (_c.c_int, [_vp]),
    "slm_ctx_stream": (_c.c_int, [_vp, _c.POINTER(_vp)]),
    "slm_zeros": (_c.c_int, [_vp, _sz, _c.POINTER(_vp)]),
    "slm_upload": (_c.c_int, [_vp, _f32p, _sz, _c.POINTER(_vp)]),
    "slm_read": (_c.c_int, [_vp, _vp, _sz, _f32p]),
    "slm_buf_free": (_c.c_int, [_vp]),
    "slm_buf_len": (_sz, [_vp]),
    "slm_buf_ptr": (_vp, [_vp]),
    "slm_flush": (_c.c_int, [_vp]),
    "slm_op_gather": (_c.c_int, [_vp, _vp, _vp, _u32p, _sz, _sz]),
    "slm_op_copy": (_c.c_int, [_vp, _vp, _vp, _sz, _sz]),
    "slm_op_shift": (_c.c_int, [_vp, _vp, _vp, _vp, _sz, _sz, _sz]),
    "slm_op_columns": (_c.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz]),
    "slm_op_linear": (_c.c_int, [_vp, _vp, _vp, _sz, _sz, _vp, _sz, _sz]),
    "slm_op_add": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "slm_op_add_row": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _sz]),
    "slm_op_scale_rows": (_c.c_int, [_vp, _vp, _vp, _sz, _f32p, _sz, _sz]),
    "slm_op_mix": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _c.c_float]),
    "slm_op_rms": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _c.c_float]),
    "slm_op_silu_mul": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "slm_op_rope_table": (_c.c_int, [_vp, _vp, _vp, _vp, _sz, _sz, _sz]),
    "slm_op_rope": (_c.c_int, [_vp, _vp, _vp, _sz, _vp, _vp, _sz, _sz, _sz]),
    "slm_op_l2norm": (_c.c_int, [_vp, _vp, _vp, _sz, _sz, _sz]),
    "slm_op_gla": (_c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _vp, _sz, _sz, _sz]),
    "slm_op_store": (_c.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz]),
    "slm_op_attend": (_c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp, _vp, _c.POINTER(_Attn)]),
    "slm_op_attend_noalloc": (_c.c_int, [_vp, _vp, _vp, _vp, _vp, _c.POINTER(_Attn)]),
    "slm_model_load": (_c.c_int, [_vp, _c.c_char_p, _c.POINTER(_vp)]),
    "slm_model_free": (_c.c_int, [_vp]),
    "slm_model_info_get": (_c.c_int, [_vp, _c.POINTER(_Info)]),
    "slm_session_new": (_c.c_int, [_vp, _sz, _c.POINTER(_vp)]),
    "slm_session_free": (_c.c_int, [_vp]),
    "slm_session_pos": (_c.c_int, [_vp, _c.POINTER(_sz)]),
    "slm_session_loops": (_c.c_int, [_vp, _c.POINTER(_sz)]),
    "slm_session_set": (_c.c_int, [_vp, _c.c_int, _c.c_int64]),
    "slm_session_stat": (_c.c_int, [_vp, _c.c_int, _c.POINTER(_c.c_int64)]),
    "slm_session_trace": (_c.c_int, [_vp, _u64p, _sz, _c.POINTER(_sz)]),
    "slm_feed": (_c.c_int, [_vp, _u32p, _sz, _sz]),
    "slm_step": (_c.c_int, [_vp, _c.c_uint32]),
    "slm_logits": (_c.c_int, [_vp, _f32p]),
    "slm_state_bytes": (_c.c_int, [_vp, _c.POINTER(_sz)]),
    "slm_session_state_count": (_c.c_int, [_vp, _c.POINTER(_sz)]),
    "slm_session_state_info": (_c.c_int, [_vp, _sz, _c.POINTER(_StateArray)]),
    "slm_session_state_read": (_c.c_int, [_vp, _sz, _f32p]),
    "slm_session_state_write": (_c.c_int, [_vp, _sz, _f32p, _sz]),
    "slm_session_set_pos": (_c.c_int, [_vp, _sz]),
    "slm_rng_seed": (_c.c_uint64, [_c.c_uint64]),
    "slm_sample": (_c.c_int, [_vp, _c.POINTER(_Sampling), _u32p, _sz, _u64p, _u32p]),
    "slm_pick": (_c.c_int, [_vp, _vp, _sz, _c.POINTER(_Sampling), _u32p, _sz, _u64p, _u32p]),
    "slm_decode": (_c.c_int, [_vp, _c.c_uint32, _sz, _c.POINTER(_Sampling), _u32p, _sz, _u64p, _u32p]),
    "slm_batch_new": (_c.c_int, [_c.POINTER(_vp), _sz, _c.POINTER(_vp)]),
    "slm_batch_free": (_c.c_int, [_vp]),
    "slm_batch_size": (_c.c_int, [_vp, _c.POINTER(_sz)]),
    "slm_batch_step": (_c.c_int, [_vp, _u32p]),
    "slm_batch_logits": (_c.c_int, [_vp, _f32p]),
    "slm_batch_decode": (_c.c_int, [_vp, _u32p, _sz, _u32p]),
    "slm_batch_sample_decode": (_c.c_int, [_vp, _u32p, _sz, _c.POINTER(_Sampling), _c.POINTER(_u32p),
                                           _c.POINTER(_sz), _u64p, _u32p]),
}


def lib():
    """Loads libslm_b200.so (built by build.py); raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise SlmError(2, f"{LIB_PATH} is missing: run `python slm.use_b200/build.py`")
        L = _c.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(code: int) -> None:
    if code != 0:
        raise SlmError(code, lib().slm_last_error().decode())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


def pick(ctx: "Context", logits, s: "Sampling", recent=(), rng_state: list | None = None) -> int:
    """pick (src/sample.rs:33-93) on the device for host logits."""
    ops = Ops(ctx)
    buf = ops.upload(logits)
    rec = _u32(recent if len(recent) else [0])
    st = _c.c_uint64(rng_state[0] if rng_state is not None else rng_seed(0))
    out = _c.c_uint32(0)
    sc = s._c()
    _check(lib().slm_pick(ctx._h, buf._h, len(logits), _c.byref(sc), rec.ctypes.data_as(_u32p), len(recent),
                          _c.byref(st), _c.byref(out)))
    if rng_state is not None:
        rng_state[0] = st.value
    buf.close()
    return out.value


def device_count() -> int:
    n = _c.c_int(0)
    _check(lib().slm_device_count(_c.byref(n)))
    return n.value


def rng_seed(seed: int) -> int:
    """Rng::new (src/sample.rs:21-23): the initial xorshift64* state."""
    return int(lib().slm_rng_seed(seed))


_SEED0: int | None = None
_NO_RECENT = None


def _seed0() -> int:
    """rng_seed(0), computed once (the state a sample() call without one starts from)."""
    global _SEED0
    if _SEED0 is None:
        _SEED0 = rng_seed(0)
    return _SEED0


def _no_recent():
    """Pointer to a one-word buffer for calls with no recent ids (n = 0)."""
    global _NO_RECENT
    if _NO_RECENT is None:
        arr = np.zeros(1, dtype=np.uint32)
        _NO_RECENT = (arr, arr.ctypes.data_as(_u32p))
    return _NO_RECENT[1]


# ---------------------------------------------------------------------------
# Context and buffers
# ---------------------------------------------------------------------------

class Context:
    """One device and one stream (the reference's Cuda::probe, src/cuda.rs:71-120)."""

    def __init__(self, device: int = 0):
        h = _vp()
        _check(lib().slm_ctx_new(device, _c.byref(h)))
        self._h = h
        self._free = lib().slm_ctx_free
        self.device = device

    def close(self):
        # The free function is looked up while the module is intact: at
        # interpreter exit its globals may already be gone.
        if getattr(self, "_h", None):
            free = getattr(self, "_free", None) or lib().slm_ctx_free
            free(self._h)
            self._h = None

    __del__ = close

    @property
    def name(self) -> str:
        buf = _c.create_string_buffer(256)
        _check(lib().slm_ctx_name(self._h, buf, 256))
        return buf.value.decode()

    def sync(self) -> None:
        _check(lib().slm_ctx_sync(self._h))

    @property
    def stream(self) -> int:
        p = _vp()
        _check(lib().slm_ctx_stream(self._h, _c.byref(p)))
        return int(p.value or 0)


class Buf:
    """A device f32 buffer (the reference's Ops::Buf)."""

    def __init__(self, ctx: Context, handle):
        self.ctx = ctx
        self._ctx_h = ctx._h  # stays valid while the buffer lives (the library defers the context's release)
        self._h = handle
        self._free = lib().slm_buf_free

    def close(self):
        # The free function is looked up while the module is intact: at
        # interpreter exit its globals may already be gone.
        if getattr(self, "_h", None):
            free = getattr(self, "_free", None) or lib().slm_buf_free
            free(self._h)
            self._h = None

    __del__ = close

    def __len__(self) -> int:
        return int(lib().slm_buf_len(self._h))

    @property
    def ptr(self) -> int:
        return int(lib().slm_buf_ptr(self._h) or 0)

    def read(self, n: int | None = None) -> np.ndarray:
        n = len(self) if n is None else n
        out = np.empty(n, dtype=np.float32)
        _check(lib().slm_read(self._ctx_h, self._h, n, out.ctypes.data_as(_f32p)))
        return out


class Ops:
    """The reference's `Ops` trait (src/ops.rs:68-228) on one context.

    Arguments that the trait passes as `At<Buf>` are a (Buf, offset) pair here;
    a bare Buf means offset 0.  Outputs are grown when too small."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self._c = ctx._h

    @staticmethod
    def _at(x):
        return (x[0], int(x[1])) if isinstance(x, tuple) else (x, 0)

    def name(self) -> str:
        return self.ctx.name

    def zeros(self, n: int) -> Buf:
        h = _vp()
        _check(lib().slm_zeros(self._c, n, _c.byref(h)))
        return Buf(self.ctx, h)

    def upload(self, data) -> Buf:
        a = _f32(data).ravel()
        h = _vp()
        _check(lib().slm_upload(self._c, a.ctypes.data_as(_f32p), a.size, _c.byref(h)))
        return Buf(self.ctx, h)

    def read(self, buf: Buf, n: int) -> np.ndarray:
        return buf.read(n)

    def flush(self, keep=()) -> None:
        _check(lib().slm_flush(self._c))

    def gather(self, y: Buf, w: Buf, ids, d: int) -> None:
        ids = _u32(ids)
        _check(lib().slm_op_gather(self._c, y._h, w._h, ids.ctypes.data_as(_u32p), ids.size, d))

    def copy(self, y: Buf, x, n: int) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_copy(self._c, y._h, xb._h, xo, n))

    def shift(self, y: Buf, first: Buf, x, m: int, d: int) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_shift(self._c, y._h, first._h, xb._h, xo, m, d))

    def columns(self, y: Buf, x: Buf, m: int, stride: int, off: int, length: int) -> None:
        _check(lib().slm_op_columns(self._c, y._h, x._h, m, stride, off, length))

    def linear(self, y: Buf, w: Buf, rows: int, cols: int, x, m: int) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_linear(self._c, y._h, w._h, rows, cols, xb._h, xo, m))

    def add(self, y: Buf, a, b, n: int) -> None:
        (ab, ao), (bb, bo) = self._at(a), self._at(b)
        _check(lib().slm_op_add(self._c, y._h, ab._h, ao, bb._h, bo, n))

    def add_row(self, y: Buf, x, row, m: int, d: int) -> None:
        (xb, xo), (rb, ro) = self._at(x), self._at(row)
        _check(lib().slm_op_add_row(self._c, y._h, xb._h, xo, rb._h, ro, m, d))

    def scale_rows(self, y: Buf, x, f, d: int) -> None:
        xb, xo = self._at(x)
        f = _f32(f)
        _check(lib().slm_op_scale_rows(self._c, y._h, xb._h, xo, f.ctypes.data_as(_f32p), f.size, d))

    def mix(self, y: Buf, a, b, n: int, t: float) -> None:
        (ab, ao), (bb, bo) = self._at(a), self._at(b)
        _check(lib().slm_op_mix(self._c, y._h, ab._h, ao, bb._h, bo, n, t))

    def rms(self, y: Buf, x, w: Buf, groups: int, size: int, eps: float) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_rms(self._c, y._h, xb._h, xo, w._h, groups, size, eps))

    def silu_mul(self, y: Buf, g, u, n: int) -> None:
        (gb, go), (ub, uo) = self._at(g), self._at(u)
        _check(lib().slm_op_silu_mul(self._c, y._h, gb._h, go, ub._h, uo, n))

    def rope_table(self, cos: Buf, sin: Buf, inv: Buf, pos: int, m: int, half: int) -> None:
        _check(lib().slm_op_rope_table(self._c, cos._h, sin._h, inv._h, pos, m, half))

    def rope(self, y: Buf, x, cos: Buf, sin: Buf, m: int, heads: int, dh: int) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_rope(self._c, y._h, xb._h, xo, cos._h, sin._h, m, heads, dh))

    def l2norm(self, y: Buf, x, heads: int, dh: int) -> None:
        xb, xo = self._at(x)
        _check(lib().slm_op_l2norm(self._c, y._h, xb._h, xo, heads, dh))

    def gla(self, y: Buf, s: Buf, q, k, v, decay: Buf, bias: Buf, m: int, heads: int, dh: int) -> None:
        (qb, qo), (kb, ko), (vb, vo) = self._at(q), self._at(k), self._at(v)
        _check(lib().slm_op_gla(self._c, y._h, s._h, qb._h, qo, kb._h, ko, vb._h, vo, decay._h, bias._h, m, heads,
                                dh))

    def store(self, cache: Buf, src, pos: int, m: int, cap: int, heads: int, dh: int) -> None:
        sb, so = self._at(src)
        _check(lib().slm_op_store(self._c, cache._h, sb._h, so, pos, m, cap, heads, dh))

    def attend(self, y: Buf, scores: Buf, q, k: Buf, v: Buf, *, pos: int, m: int, reach: int | None, gap: int,
               cap: int, heads: int, key_heads: int, dh: int, scale: float) -> None:
        """Attn (src/ops.rs:31-46); reach None is unbounded (usize::MAX)."""
        qb, qo = self._at(q)
        a = _Attn(pos, m, SIZE_MAX if reach is None else reach, gap, cap, heads, key_heads, dh, scale)
        _check(lib().slm_op_attend(self._c, y._h, scores._h, qb._h, qo, k._h, v._h, _c.byref(a)))


def attend_noalloc(ctx: Context, y: Buf, q: Buf, k: Buf, v: Buf, *, pos: int, m: int, reach: int | None, gap: int,
                   cap: int, heads: int, key_heads: int, dh: int, scale: float) -> None:
    """Ops::attend on caller-owned device buffers with no device allocation
    (scratch in a fixed per-device array); see slm_op_attend_noalloc."""
    a = _Attn(pos, m, SIZE_MAX if reach is None else reach, gap, cap, heads, key_heads, dh, scale)
    _check(lib().slm_op_attend_noalloc(ctx._h, y.ptr, q.ptr, k.ptr, v.ptr, _c.byref(a)))


# ---------------------------------------------------------------------------
# Model level
# ---------------------------------------------------------------------------

@dataclass
class Sampling:
    """src/sample.rs:3-15."""
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repeat_penalty: float = 1.0
    repeat_window: int = 0

    def _c(self) -> _Sampling:
        return _Sampling(self.temperature, self.top_k, self.top_p, self.repeat_penalty, self.repeat_window)

    def _ref(self):
        """byref of the C struct, rebuilt only when a field changed (per-token calls reuse it)."""
        key = (self.temperature, self.top_k, self.top_p, self.repeat_penalty, self.repeat_window)
        c = self.__dict__.get("_cache")
        if c is None or c[0] != key:
            sc = self._c()
            c = (key, sc, _c.byref(sc))
            self.__dict__["_cache"] = c
        return c[2]


class Model:
    """Model::load (src/model.rs:226-269) on a context."""

    def __init__(self, ctx: Context, folder):
        self.ctx = ctx
        h = _vp()
        _check(lib().slm_model_load(ctx._h, str(folder).encode(), _c.byref(h)))
        self._h = h
        self._free = lib().slm_model_free
        info = _Info()
        _check(lib().slm_model_info_get(h, _c.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in _Info._fields_}
        for k in ("prelude", "core", "coda"):
            self.info[k] = self.info[k].decode()
        self.vocab = info.vocab

    def close(self):
        # The free function is looked up while the module is intact: at
        # interpreter exit its globals may already be gone.
        if getattr(self, "_h", None):
            free = getattr(self, "_free", None) or lib().slm_model_free
            free(self._h)
            self._h = None

    __del__ = close

    def params(self) -> int:
        return self.info["params"]

    def session(self, loops: int | None = None) -> "Session":
        return Session(self, loops)


class Session:
    """Session (src/model.rs:209-223) with feed/step/logits and device sampling."""

    def __init__(self, model: Model, loops: int | None = None):
        self.model = model
        h = _vp()
        _check(lib().slm_session_new(model._h, loops or 0, _c.byref(h)))
        self._h = h
        self._free = lib().slm_session_free
        self.vocab = model.vocab
        # Per-token sample() arguments, reused across calls.
        self._st, self._out = _c.c_uint64(0), _c.c_uint32(0)
        self._st_ref, self._out_ref = _c.byref(self._st), _c.byref(self._out)

    def close(self):
        # The free function is looked up while the module is intact: at
        # interpreter exit its globals may already be gone.
        if getattr(self, "_h", None):
            free = getattr(self, "_free", None) or lib().slm_session_free
            code = free(self._h)
            if code != 0:  # e.g. still in a batch: the session stays open
                raise SlmError(code, lib().slm_last_error().decode())
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        v = _sz()
        _check(lib().slm_session_pos(self._h, _c.byref(v)))
        return v.value

    @property
    def loops(self) -> int:
        v = _sz()
        _check(lib().slm_session_loops(self._h, _c.byref(v)))
        return v.value

    def stat(self, what: int) -> int:
        v = _c.c_int64(0)
        _check(lib().slm_session_stat(self._h, what, _c.byref(v)))
        return v.value

    @property
    def step_kernels(self) -> int:
        """Kernels one captured m = 1 step launches."""
        return self.stat(1)

    def set_graph(self, on: bool) -> None:
        _check(lib().slm_session_set(self._h, SLM_OPT_GRAPH, 1 if on else 0))

    def set_mega(self, on: bool) -> None:
        """Run m = 1 steps as one persistent kernel (where the model allows it)."""
        _check(lib().slm_session_set(self._h, SLM_OPT_MEGA, 1 if on else 0))

    def set_bf16(self, on: bool) -> None:
        """Stream bf16 copies of the weights in persistent steps (f32 arithmetic; not a parity mode)."""
        _check(lib().slm_session_set(self._h, SLM_OPT_BF16, 1 if on else 0))

    def set_stall_test(self, on: bool) -> None:
        """Test hook: the next persistent steps wait for a barrier arrival that never comes."""
        _check(lib().slm_session_set(self._h, SLM_OPT_TEST_STALL, 1 if on else 0))

    def set_trace(self, on: bool) -> None:
        _check(lib().slm_session_set(self._h, SLM_OPT_TRACE, 1 if on else 0))

    def trace(self) -> np.ndarray:
        """Timeline of the last persistent step: [phase][cta][8] (start, barrier, waited, prologue,
        compute, epilogue ns, tiles, 0)."""
        n = _sz(0)
        _check(lib().slm_session_trace(self._h, None, 0, _c.byref(n)))
        out = np.empty(n.value, dtype=np.uint64)
        _check(lib().slm_session_trace(self._h, out.ctypes.data_as(_u64p), n.value, _c.byref(n)))
        phases = self.stat(SLM_STAT_PHASES)
        return out.reshape(phases, -1, 8)

    @property
    def mega(self) -> bool:
        return self.stat(SLM_STAT_MEGA) == 1

    def feed(self, ids, limit: int = CHUNK) -> None:
        ids = _u32(ids)
        _check(lib().slm_feed(self._h, ids.ctypes.data_as(_u32p), ids.size, limit))

    def step(self, token: int) -> None:
        _check(lib().slm_step(self._h, int(token)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        _check(lib().slm_logits(self._h, out.ctypes.data_as(_f32p)))
        return out

    def state_bytes(self) -> int:
        v = _sz()
        _check(lib().slm_state_bytes(self._h, _c.byref(v)))
        return v.value

    def state_arrays(self) -> list[dict]:
        """Descriptions of the session's state arrays in step order (kind, part, heads, cap, dh, floats)."""
        n = _sz()
        _check(lib().slm_session_state_count(self._h, _c.byref(n)))
        out = []
        for i in range(n.value):
            a = _StateArray()
            _check(lib().slm_session_state_info(self._h, i, _c.byref(a)))
            out.append({"kind": a.kind.decode(), "part": a.part.decode(), "heads": a.heads, "cap": a.cap,
                        "dh": a.dh, "floats": a.floats})
        return out

    def state_read(self, i: int) -> np.ndarray:
        """State array i as a flat float32 array."""
        a = _StateArray()
        _check(lib().slm_session_state_info(self._h, i, _c.byref(a)))
        out = np.empty(a.floats, dtype=np.float32)
        _check(lib().slm_session_state_read(self._h, i, out.ctypes.data_as(_f32p)))
        return out

    def state_write(self, i: int, data, cap: int = 0) -> None:
        """Overwrites state array i; a cache comes as [heads][cap][dh] (cap 0: the array's own)."""
        data = _f32(data)
        if cap == 0:
            a = _StateArray()
            _check(lib().slm_session_state_info(self._h, i, _c.byref(a)))
            cap = a.cap or 1
        _check(lib().slm_session_state_write(self._h, i, data.ctypes.data_as(_f32p), cap))

    def set_pos(self, pos: int) -> None:
        """Puts the session at position pos (its state arrays unchanged)."""
        _check(lib().slm_session_set_pos(self._h, pos))

    def sample(self, s: Sampling, recent=(), rng_state: list | None = None) -> int:
        """pick (src/sample.rs:33-93) on the device; rng_state is a one-element list."""
        if len(recent):
            rec = _u32(recent)
            rp, n = rec.ctypes.data_as(_u32p), rec.size
        else:
            rp, n = _no_recent(), 0
        st = self._st
        st.value = rng_state[0] if rng_state is not None else _seed0()
        _check(lib().slm_sample(self._h, s._ref(), rp, n, self._st_ref, self._out_ref))
        if rng_state is not None:
            rng_state[0] = st.value
        return self._out.value

    def decode(self, first: int, n: int, s: Sampling, recent=(), rng_state: list | None = None) -> np.ndarray:
        """n steps on the device: feed `first`, then each sampled id."""
        rec = _u32(recent if len(recent) else [0])
        st = _c.c_uint64(rng_state[0] if rng_state is not None else rng_seed(0))
        out = np.empty(n, dtype=np.uint32)
        sc = s._c()
        _check(lib().slm_decode(self._h, int(first), n, _c.byref(sc), rec.ctypes.data_as(_u32p), len(recent),
                                _c.byref(st), out.ctypes.data_as(_u32p)))
        if rng_state is not None:
            rng_state[0] = st.value
        return out


class Batch:
    """Several sessions of one model stepped together, one token each per step
    (slm_batch_*; no counterpart in the reference, whose server runs one
    request at a time).  The sessions must outlive the batch."""

    def __init__(self, sessions):
        self.sessions = list(sessions)
        n = len(self.sessions)
        hs = (_vp * n)(*[se._h for se in self.sessions])
        h = _vp()
        _check(lib().slm_batch_new(hs, n, _c.byref(h)))
        self._h = h
        self._free = lib().slm_batch_free
        self.n = n
        self.vocab = self.sessions[0].vocab

    def close(self):
        # The free function is looked up while the module is intact: at
        # interpreter exit its globals may already be gone.
        if getattr(self, "_h", None):
            self._free(self._h)
            self._h = None

    __del__ = close

    def step(self, ids) -> None:
        """Feeds ids[i] to session i."""
        ids = _u32(ids)
        if ids.size != self.n:
            raise ValueError(f"expected {self.n} ids")
        _check(lib().slm_batch_step(self._h, ids.ctypes.data_as(_u32p)))

    def logits(self) -> np.ndarray:
        """[n][vocab] logits of the last step."""
        out = np.empty((self.n, self.vocab), dtype=np.float32)
        _check(lib().slm_batch_logits(self._h, out.ctypes.data_as(_f32p)))
        return out

    def sample_decode(self, first, steps: int, samplings, recents=None, rng_states=None) -> np.ndarray:
        """`steps` steps of every session with per-row sampling: row i uses samplings[i], the
        history recents[i] (sampled ids join it) and the xorshift64* state rng_states[i] (a list,
        updated in place).  Returns [steps][n] sampled ids."""
        first = _u32(first)
        n = self.n
        if first.size != n or len(samplings) != n:
            raise ValueError(f"expected {n} ids and samplings")
        sc = (_Sampling * n)(*[sp._c() for sp in samplings])
        recents = recents if recents is not None else [[] for _ in range(n)]
        arrs = [_u32(r if len(r) else [0]) for r in recents]
        ptrs = (_u32p * n)(*[a.ctypes.data_as(_u32p) for a in arrs])
        counts = (_sz * n)(*[len(r) for r in recents])
        st = np.array(rng_states if rng_states is not None else [rng_seed(0)] * n, dtype=np.uint64)
        out = np.empty((steps, n), dtype=np.uint32)
        _check(lib().slm_batch_sample_decode(self._h, first.ctypes.data_as(_u32p), steps, sc, ptrs, counts,
                                             st.ctypes.data_as(_u64p), out.ctypes.data_as(_u32p)))
        if rng_states is not None:
            rng_states[:] = [int(v) for v in st]
        return out

    def decode(self, first, steps: int) -> np.ndarray:
        """`steps` greedy steps of every session: [steps][n] picked ids."""
        first = _u32(first)
        if first.size != self.n:
            raise ValueError(f"expected {self.n} ids")
        out = np.empty((steps, self.n), dtype=np.uint32)
        _check(lib().slm_batch_decode(self._h, first.ctypes.data_as(_u32p), steps, out.ctypes.data_as(_u32p)))
        return out
