"""Compiles the reference's Metal kernel sources (read from the reference
tree at build time) into oracle/_ref/libivf_kernels_ref.so. Outputs go only to
oracle/_ref/ (git-ignored). Oracle infrastructure only."""
from __future__ import annotations

import ast
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref"
# The reference checkout: METALFAISS_REFERENCE, else its default location.
REF_ROOT = Path(os.environ.get("METALFAISS_REFERENCE", "/root/reference"))
REF_FILE = REF_ROOT / "python/metalfaiss/faissmlx/kernels/ivf_kernels.py"
LIB = OUT / "libivf_kernels_ref.so"

# C types of the buffers, by the names the reference's launchers give them
# (python/metalfaiss/faissmlx/kernels/ivf_kernels.py:252-403: Q/X float32, ids int32,
# shape uint32, outputs float32 + int32).
CTYPES = {"Q": "float", "X": "float", "ids": "int", "shape": "uint", "vals_parts": "float",
          "ids_parts": "int", "out_vals": "float", "out_ids": "int"}


def extract(path: Path):
    tree = ast.parse(path.read_text())
    strings = {}
    kernels = []
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and isinstance(node.value, ast.Constant) \
                and isinstance(node.value.value, str) and len(node.targets) == 1 \
                and isinstance(node.targets[0], ast.Name):
            strings[node.targets[0].id] = node.value.value
    for node in ast.walk(tree):
        if isinstance(node, ast.Call) and getattr(node.func, "attr", "") == "metal_kernel":
            kw = {k.arg: k.value for k in node.keywords}
            name = kw["name"].value
            ins = [e.value for e in kw["input_names"].elts]
            outs = [e.value for e in kw["output_names"].elts]
            src = strings[kw["source"].id]
            kernels.append({"name": name, "inputs": ins, "outputs": outs, "source": src})
    return kernels


def generate(kernels) -> str:
    parts = ['#include "msl_shim.h"\n']
    for k in kernels:
        n = k["name"]
        names = k["inputs"] + k["outputs"]
        fields = []
        for i, nm in enumerate(names):
            const = "const " if i < len(k["inputs"]) else ""
            fields.append(f"  {const}{CTYPES[nm]}* {nm};")
        parts.append(f"namespace k_{n} {{\nstruct Args {{\n" + "\n".join(fields) + "\n};\n")
        binds = []
        for i, nm in enumerate(names):
            const = "const " if i < len(k["inputs"]) else ""
            binds.append(f"  {const}device {CTYPES[nm]}* {nm} = a.{nm};")
        parts.append("static void body(void* ctx) {\n  Args& a = *static_cast<Args*>(ctx);\n"
                     + "\n".join(binds) + "\n#line 1 \"" + n + "\"\n" + k["source"] + "\n}\n}\n")
        casts = ", ".join(f"({('const ' if i < len(k['inputs']) else '')}{CTYPES[nm]}*)bufs[{i}]"
                          for i, nm in enumerate(names))
        parts.append(f'extern "C" void run_{n}(void** bufs, unsigned gx, unsigned tx) {{\n'
                     f"  k_{n}::Args a{{{casts}}};\n  msl_launch(gx, tx, k_{n}::body, &a);\n}}\n")
    return "\n".join(parts)


def build(force: bool = False) -> Path:
    if not REF_FILE.exists():
        raise FileNotFoundError(REF_FILE)
    OUT.mkdir(exist_ok=True)
    kernels = extract(REF_FILE)
    cpp = OUT / "ivf_kernels_ref.cpp"
    cpp.write_text(generate(kernels))
    (OUT / "kernels.json").write_text(json.dumps(
        [{"name": k["name"], "inputs": k["inputs"], "outputs": k["outputs"]} for k in kernels], indent=1))
    # Thread-local arrays of the kernels start zeroed (Metal leaves them undefined).
    cmd = ["g++", "-O2", "-std=c++20", "-fPIC", "-shared", "-pthread", "-ffp-contract=off",
           "-ftrivial-auto-var-init=zero", "-I", str(HERE), "-o", str(LIB), str(cpp),
           str(HERE / "msl_launch.cpp")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("reference kernel build failed")
    return LIB


def build_if_present():
    if REF_FILE.exists():
        return build()
    return None


if __name__ == "__main__":
    print(build())
