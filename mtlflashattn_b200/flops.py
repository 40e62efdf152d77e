"""Algorithmic work of an attention forward, for throughput and roofline reporting.

FLOPs = 4 * D * (number of unmasked (query, key) pairs) per (batch, head): 2*D for q.k and
2*D for p.v. The reference's bench formula 4*B*H*L^2*D*(0.5 if causal)
(bench/bench_attn.py:47) is ``reference_formula_flops``; for causal Lq = Lk it differs from
the exact count by L/(2L^2) relative (< 0.02% at L = 8192).
"""
from __future__ import annotations

import torch


def attention_pairs(Lq, Lk, causal=False, window=(-1, -1), key_offset=0, lk_total=None):
    """Unmasked (query, key) pairs of one (batch, head) with bottom-right alignment, for local
    keys [key_offset, key_offset + Lk) of a problem with lk_total keys."""
    if Lq <= 0 or Lk <= 0:
        return 0
    lk_total = Lk if lk_total is None else lk_total
    centre = torch.arange(Lq, dtype=torch.int64) + (lk_total - Lq)
    lo = torch.full_like(centre, key_offset)
    hi = torch.full_like(centre, key_offset + Lk)
    wl, wr = window
    if wl >= 0:
        lo = torch.maximum(lo, centre - wl)
    if causal:
        hi = torch.minimum(hi, centre + 1)
    if wr >= 0:
        hi = torch.minimum(hi, centre + wr + 1)
    return int((hi - lo).clamp_min(0).sum())


def attention_flops(B, Hq, Lq, Lk, D, causal=False, window=(-1, -1), **kw):
    return 4 * D * B * Hq * attention_pairs(Lq, Lk, causal, window, **kw)


def varlen_flops(lens_q, lens_k, Hq, D, causal=False, window=(-1, -1)):
    return sum(attention_flops(1, Hq, a, b, D, causal, window) for a, b in zip(lens_q, lens_k))


def reference_formula_flops(B, H, L, D, causal):
    return 4 * B * H * L * L * D * (0.5 if causal else 1.0)


def compulsory_bytes(B, Hq, Hkv, Lq, Lk, D, elem=2, out_elem=None):
    """HBM bytes that must move at least once: Q, K, V read and O written."""
    out_elem = elem if out_elem is None else out_elem
    return B * D * (Lq * Hq * elem + 2 * Lk * Hkv * elem + Lq * Hq * out_elem)
