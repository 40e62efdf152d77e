"""Loads tests/golden/golden.pt (written by make_golden.py from the reference itself) and
regenerates each case's inputs from its seed with the same CPU generator the reference's tests
use, checking them against the stored float64 sums."""
from __future__ import annotations

import functools
import os

import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.pt")


def _draw_dense(shape, dtype, seed):
    B, Lq, Lk, Hq, Hkv, D = shape
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, Lq, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, Lk, Hkv, D, generator=g).to(dtype)
    v = torch.randn(B, Lk, Hkv, D, generator=g).to(dtype)
    return q, k, v


def _draw_varlen(lq, lk, Hq, Hkv, D, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(sum(lq), Hq, D, generator=g).to(dtype)
    k = torch.randn(sum(lk), Hkv, D, generator=g).to(dtype)
    v = torch.randn(sum(lk), Hkv, D, generator=g).to(dtype)
    return q, k, v


@functools.lru_cache(maxsize=1)
def load_cases():
    data = torch.load(GOLDEN, weights_only=False)
    out = []
    for c in data["cases"]:
        c = dict(c)
        if c["kind"] == "dense":
            q, k, v = _draw_dense(c["shape"], c["dtype"], c["seed"])
        else:
            q, k, v = _draw_varlen(c["lq"], c["lk"], c["Hq"], c["Hkv"], c["D"], c["dtype"], c["seed"])
        sums = [float(t.double().sum()) for t in (q, k, v)]
        for a, b in zip(sums, c["input_sums"]):
            if abs(a - b) > 1e-6 * max(1.0, abs(b)):
                raise RuntimeError(f"golden case {c['name']}: regenerated inputs differ "
                                   f"(CPU generator drift): {sums} vs {c['input_sums']}")
        c.update(q=q, k=k, v=v)
        out.append(c)
    return out


def case_ids():
    return [c["name"] for c in load_cases()]
