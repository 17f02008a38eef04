"""Build libloopspec_engine.so in-tree for sm_100a with nvcc.

    python -m loopspec_b200.build            # rebuild if any source is newer
    python -m loopspec_b200.build --force
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# translation units compiled in parallel, then linked into one library
SRCS = [os.path.join(HERE, "csrc", "engine.cu")]
OUT = os.path.join(HERE, "libloopspec_engine.so")
OBJ_DIR = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-diag-suppress", "177"]


def _sources():
    return glob.glob(os.path.join(HERE, "csrc", "*")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(OUT):
        newest = max(os.path.getmtime(p) for p in _sources())
        if os.path.getmtime(OUT) >= newest:
            return OUT
    os.makedirs(OBJ_DIR, exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    for src in SRCS:
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *(["-Xptxas=-v"] if verbose else []), "-c", "-o", obj, src]
        jobs.append((obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    errors = []
    for obj, proc in jobs:
        out, err = proc.communicate()
        if proc.returncode != 0:
            errors.append(out + err)
        elif verbose:
            sys.stderr.write(err)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = OUT + ".tmp"
    res = subprocess.run([nvcc, *ARCH, "-shared", "-o", tmp, *(o for o, _ in jobs)],
                         capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
