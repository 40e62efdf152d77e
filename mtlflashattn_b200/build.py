"""Builds libmfa.so in-tree with nvcc for sm_100a.

Usage: python -m mtlflashattn_b200.build [--verbose]
The library has no dependency on torch: plain nvcc, static cudart, and the driver entry
point for cuTensorMapEncodeTiled resolved at run time (no -lcuda needed).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "mfa_api.cu")
OUT = os.path.join(HERE, "libmfa.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; CUDA 12.8+ is required to build libmfa.so")
    return cand


def sources() -> list[str]:
    d = os.path.join(HERE, "csrc")
    inc = os.path.join(os.path.dirname(HERE), "include")
    return [os.path.join(d, f) for f in sorted(os.listdir(d))] + [
        os.path.join(inc, f) for f in sorted(os.listdir(inc))]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(verbose: bool = False, force: bool = False, defines=(), out: str | None = None) -> str:
    """Compile libmfa.so (or, with ``out``, a variant of it at that path; ``defines`` are
    extra NAME=VALUE macros, e.g. the tuning knobs at the top of csrc/fa_sm100.cuh)."""
    target = out or OUT
    if not force and out is None and not defines and up_to_date():
        return OUT
    cmd = [nvcc_path(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
           "-Xcompiler", "-fPIC", "-shared", *[f"-D{d}" for d in defines], "-o", target + ".tmp",
           SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    os.replace(target + ".tmp", target)
    return target


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
