"""Builds libslm_b200.so in this folder from csrc/ with nvcc for sm_100a.

    python slm.use_b200/build.py [--force]

Objects go to _build/ beside this file; a source is recompiled when it, or any
header in csrc/ or include/, is newer than its object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT = HERE / "libslm_b200.so"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


# The CUTLASS release the gemm_*.cu kernels are written and tested against.
CUTLASS_VERSION = (4, 5, 0)


def _cutlass_version(root: Path) -> tuple:
    import re
    text = (root / "include" / "cutlass" / "version.h").read_text()
    parts = dict(re.findall(r"#define CUTLASS_(MAJOR|MINOR|PATCH) (\d+)", text))
    return tuple(int(parts.get(k, -1)) for k in ("MAJOR", "MINOR", "PATCH"))


def _cutlass_includes() -> list[str]:
    """CUTLASS/CuTe headers for the gemm_*.cu kernels: $SLM_CUTLASS_DIR (a
    CUTLASS source tree), else the copy vendored in the image's flashinfer
    wheel (flashinfer/data/cutlass).  The tree must be CUTLASS_VERSION."""
    import site
    env = os.environ.get("SLM_CUTLASS_DIR", "")
    roots = [Path(env)] if env else [Path(p) / "flashinfer" / "data" / "cutlass" for p in site.getsitepackages()]
    for r in roots:
        if (r / "include" / "cutlass" / "cutlass.h").exists():
            got = _cutlass_version(r)
            if got != CUTLASS_VERSION:
                raise RuntimeError(f"CUTLASS at {r} is {'.'.join(map(str, got))}; the gemm_*.cu kernels are pinned "
                                   f"to {'.'.join(map(str, CUTLASS_VERSION))} (set SLM_CUTLASS_DIR to such a tree)")
            return ["-I", str(r / "include"), "-I", str(r / "tools" / "util" / "include")]
    raise RuntimeError("CUTLASS headers not found: set SLM_CUTLASS_DIR to a CUTLASS "
                       f"{'.'.join(map(str, CUTLASS_VERSION))} source tree")


ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", str(INCLUDE)]


def _sources():
    return sorted(list(SRC.glob("*.cu")) + list(SRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(SRC.glob("*.cuh")) + list(SRC.glob("*.hpp")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
        return obj
    lang = ["-x", "cu"]
    extra = _cutlass_includes() if src.name.startswith("gemm_") else []
    cmd = [NVCC, *ARCH, *FLAGS, *extra, *lang, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(OUT)
    return OUT


if __name__ == "__main__":
    try:
        build(force="--force" in sys.argv, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        print("BUILD FAILED", file=sys.stderr)
        sys.exit(1)
