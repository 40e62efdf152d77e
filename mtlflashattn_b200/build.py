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
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "libmfa.so")
# The same library with device-side bounds checks (-DMFA_CHECKS=1): select it with
# MTLFLASHATTN_LIB to debug a failing shape (a failed check sets MFA_ERR_CHECK, never traps).
CHECKS_OUT = os.path.join(HERE, "libmfa_checks.so")
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


# Each translation unit with its math flags: the library is built with fast math (the tcgen05
# kernel's exponentials are ex2.approx by design); the fp32 CUDA-core forward is the accuracy
# path and is compiled with IEEE division / square root, accurate expf / tanhf / logf and no
# flush to zero.
UNITS = (("mfa_api.cu", ["--use_fast_math"]),
         ("simt_fwd.cu", ["-ftz=false", "-prec-div=true", "-prec-sqrt=true"]))


def build(verbose: bool = False, force: bool = False, defines=(), out: str | None = None) -> str:
    """Compile libmfa.so (or, with ``out``, a variant of it at that path; ``defines`` are
    extra NAME=VALUE macros, e.g. the tuning knobs at the top of csrc/fa_sm100.cuh)."""
    target = out or OUT
    if not force and out is None and not defines and up_to_date():
        return OUT
    base = [nvcc_path(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
            *[f"-D{d}" for d in defines]]
    if verbose:
        base.insert(1, "-Xptxas=-v")
    objs = []
    logs = []
    with tempfile.TemporaryDirectory() as tmp:
        for src, flags in UNITS:
            obj = os.path.join(tmp, src + ".o")
            r = subprocess.run([*base, *flags, "-c", "-o", obj, os.path.join(HERE, "csrc", src)],
                               capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n" + r.stdout + r.stderr)
            logs.append(r.stdout + r.stderr)
            objs.append(obj)
        r = subprocess.run([nvcc_path(), *ARCH, "-shared", "-o", target + ".tmp", *objs],
                           capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write("".join(logs))
    os.replace(target + ".tmp", target)
    return target


def build_checks(force: bool = False) -> str:
    """Build libmfa_checks.so (the MFA_CHECKS=1 debug variant) next to libmfa.so."""
    if not force and os.path.exists(CHECKS_OUT) and all(
            os.path.getmtime(s) <= os.path.getmtime(CHECKS_OUT) for s in sources()):
        return CHECKS_OUT
    return build(force=True, defines=("MFA_CHECKS=1",), out=CHECKS_OUT)


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
    if "--checks" in sys.argv:
        print(build_checks(force=True))
