"""Builds the oracle's C port (oracle/_build/liboracle.so) and, when the
reference sources are present, the reference kernel library (oracle/_ref/).
Test infrastructure only."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB = BUILD / "liboracle.so"
CFLAGS = ["-O3", "-march=x86-64-v3", "-mtune=generic", "-ffp-contract=off", "-fopenmp",
          "-fPIC", "-shared", "-std=c11"]


def build(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted((HERE / "c").glob("*.c"))
    if force or not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in srcs):
        cmd = ["gcc", *CFLAGS, "-o", str(LIB), *map(str, srcs), "-lm"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("oracle C build failed")
    try:
        from .ref_msl import build_ref
    except ImportError:
        build_ref = None
    if build_ref is not None:
        build_ref.build_if_present()
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
