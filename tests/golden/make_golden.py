"""Copies the reference's tiny parity fixture into tests/golden/tiny.

The fixture is data, not source: a random-weight model with every layer type
(prelude S, core LS, coda SG; window 8; loops 3) and the per-position logits
that the PyTorch reference model produced for 40 tokens (tests/fixtures/tiny in
the reference, written by tools/make_fixture.py there).  The GPU box has no copy
of the reference tree, so the three files are committed here and this script
records where they came from.  It checks the SHA-256 of each file it copies.

    python tests/golden/make_golden.py <reference-root>
"""
import hashlib
import shutil
import sys
from pathlib import Path

FILES = {
    "config.json": None,
    "model.safetensors": None,
    "expected.safetensors": None,
}


def main(root: str) -> None:
    src = Path(root) / "tests" / "fixtures" / "tiny"
    dst = Path(__file__).resolve().parent / "tiny"
    dst.mkdir(parents=True, exist_ok=True)
    for name in FILES:
        shutil.copyfile(src / name, dst / name)
        digest = hashlib.sha256((dst / name).read_bytes()).hexdigest()
        print(f"{name}  sha256={digest}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference-root>")
    main(sys.argv[1])
