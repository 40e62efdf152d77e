"""Opt-in routing of ``F.scaled_dot_product_attention`` to this engine on B200.

Contract kept from the reference's patch (metal_flash_attn/sdpa.py:1-193, its tests
tests/test_sdpa_patch.py): ``install(min_score_gb=None, min_seq=None, fast_min_seq=None)`` /
``uninstall()``, the kill switch ``MTLFLASHATTN_SDPA=off``, the environment knobs
``MTLFLASHATTN_SDPA_MIN_GB``, ``MTLFLASHATTN_SDPA_MIN_SEQ`` and ``MTLFLASHATTN_SDPA_FAST_MIN_SEQ``,
``_eligibility(q, k, v, attn_mask, dropout_p, is_causal) -> (bool, reason)`` with the reasons
``fast-tier``, ``correctness-large-seq``, ``oom-rescue`` and ``fits(...)``, refusal of top-left
causal calls with Lq != Lk, and a bitwise stock result for every call that is not routed.

The decisions are re-derived for CUDA. Stock SDPA on a B200 is exact at every length (its fused
flash / cuDNN / memory-efficient backends never materialise the score matrix), so the only
reason to route a call is that this engine is faster on it, and the only safety net left is
the memory one:

* ``fast-tier``: the tcgen05 kernel would run the call (fp16/bf16, D % 8 == 0, aligned) and
  max(Lq, Lk) >= ``fast_min_seq``. The default comes from ``calibrate()`` on B200 against stock
  SDPA with its default backend choice (see DEFAULT_FAST_MIN_SEQ).
* ``correctness-large-seq``: kept as the name of a length floor that routes every tier,
  including the fp32 CUDA-core kernel. Stock SDPA is not wrong on CUDA, and the CUDA-core
  kernel is slower than stock's fused fp32 path, so by default this floor is off; setting
  ``MTLFLASHATTN_SDPA_MIN_SEQ`` (or ``min_seq``) turns it on, e.g. for bitwise agreement with
  this engine's own fp32 kernel.
* ``oom-rescue``: a call whose dense score matrix (B * Hq * Lq * Lk * 2 bytes) would reach
  ``min_score_gb``: stock's math backend, the one it falls back to when no fused backend takes
  a call, would materialise it.

A value head dim different from the query/key one is routed too, when a gate fires and both
dims are at most 128: zero columns are exact no-ops in both products (extra q/k columns add
0 to every score, extra v columns give output columns that are sliced off), so the call runs on
the fast kernel with q/k/v padded to the larger dim. Calls no gate routes go to stock SDPA,
which handles uneven value dims exactly on CUDA.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from ._kernel import MAX_HEAD_DIM, _select_tier, flash_attn_forward

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)

# Crossover of this engine over stock SDPA, measured by calibrate() on B200 with torch 2.11
# (bf16, D 64/128, causal and not, L 256-8192, 16 heads): stock SDPA (its cuDNN attention on
# this GPU) was faster on every shape, by 12-19% at L = 8192 and more at short lengths, so by
# default no call is routed for speed. MTLFLASHATTN_SDPA_FAST_MIN_SEQ (or fast_min_seq) turns
# the gate on where calibrate() finds a crossover (e.g. a torch build without that backend).
DEFAULT_FAST_MIN_SEQ = None
DEFAULT_MIN_GB = 12.0


class _Gates:
    __slots__ = ("orig", "min_score_bytes", "min_seq", "fast_min_seq")

    def __init__(self):
        self.orig = None
        self.min_score_bytes = None
        self.min_seq = None
        self.fast_min_seq = None


_g = _Gates()


def _env_number(name, cast, default):
    raw = os.environ.get(name)
    if raw is None or raw.strip() == "":
        return default
    return cast(raw)


def _structure(q, k, v, attn_mask, dropout_p, is_causal, enable_gqa):
    """Why the engine cannot take this call at all (None if it can)."""
    if q.device.type != "cuda":
        return "not-cuda"
    if attn_mask is not None:
        return "attn_mask"
    if dropout_p:
        return "dropout"
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        return f"ndim({q.dim()})"
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        return f"dtype({q.dtype})"
    if k.device != q.device or v.device != q.device:
        return "devices"
    Dqk, Dv = q.shape[-1], v.shape[-1]
    if k.shape[-1] != Dqk or max(Dqk, Dv) > MAX_HEAD_DIM:
        return f"head_dim({Dqk}/{Dv})"
    Hq, Hkv = q.shape[1], k.shape[1]
    if v.shape[1] != Hkv or Hkv == 0 or Hq % Hkv != 0 or (Hq != Hkv and not enable_gqa):
        return f"heads({Hq}/{Hkv})"
    if k.shape[2] != v.shape[2] or k.shape[0] != q.shape[0] or v.shape[0] != q.shape[0]:
        return "shape-mismatch"
    # SDPA's is_causal keeps the top-left triangle; this engine aligns it bottom-right. The two
    # agree only when Lq == Lk.
    if is_causal and q.shape[2] != k.shape[2]:
        return "causal-cross-length"
    return None


def _decide(q, k, v, attn_mask, dropout_p, is_causal, enable_gqa=True):
    why = _structure(q, k, v, attn_mask, dropout_p, is_causal, enable_gqa)
    if why is not None:
        return False, why
    B, Hq, Lq, D = q.shape
    Lk = k.shape[2]
    longest = max(Lq, Lk)
    if _g.min_seq is not None and longest >= _g.min_seq:
        return True, "correctness-large-seq"
    if (_g.fast_min_seq is not None and longest >= _g.fast_min_seq
            and _select_tier(q, k, v) == "tcgen05"):
        return True, "fast-tier"
    scores = B * Hq * Lq * Lk * 2
    if scores >= _g.min_score_bytes:
        return True, "oom-rescue"
    return False, f"fits({scores / 1024 ** 3:.2f}GB)"


def _eligibility(q, k, v, attn_mask, dropout_p, is_causal):
    """(routed?, reason) for a call on heads-second q/k/v, as the installed gates decide it."""
    return _decide(q, k, v, attn_mask, dropout_p, is_causal)


def _pad_last(t, d):
    return t if t.shape[-1] == d else F.pad(t, (0, d - t.shape[-1]))


def _engine(query, key, value, is_causal, scale):
    s = scale if scale is not None else 1.0 / math.sqrt(query.shape[-1])
    Dqk, Dv = query.shape[-1], value.shape[-1]
    if Dqk == Dv:
        return flash_attn_forward(query, key, value, scale=s, causal=is_causal)
    d = max(Dqk, Dv)
    d += (-d) % 8  # keep the padded calls on the tensor-core kernel
    d = min(d, MAX_HEAD_DIM)
    out = flash_attn_forward(_pad_last(query, d), _pad_last(key, d), _pad_last(value, d),
                             scale=s, causal=is_causal)
    return out[..., :Dv]


def _patched(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
             **kwargs):
    ok, _ = _decide(query, key, value, attn_mask, dropout_p, is_causal,
                    enable_gqa=bool(kwargs.get("enable_gqa", False)))
    if ok:
        try:
            return _engine(query, key, value, is_causal, scale)
        except Exception as e:  # a routed call never fails where stock would succeed
            print(f"[mtlflashattn_b200/sdpa] engine declined the call ({e}); using stock SDPA")
    return _g.orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                   is_causal=is_causal, scale=scale, **kwargs)


def __getattr__(name):  # ``sdpa._orig`` as in the reference's module
    if name == "_orig":
        return _g.orig
    raise AttributeError(name)


def install(min_score_gb=None, min_seq=None, fast_min_seq=None):
    """Route eligible ``F.scaled_dot_product_attention`` calls to this engine. Returns True if
    this call installed the patch (False if it was already installed or switched off)."""
    if _g.orig is not None:
        return False
    if os.environ.get("MTLFLASHATTN_SDPA", "auto").strip().lower() in ("off", "0", "false", "no"):
        return False
    gb = min_score_gb if min_score_gb is not None else _env_number(
        "MTLFLASHATTN_SDPA_MIN_GB", float, DEFAULT_MIN_GB)
    _g.min_score_bytes = int(gb * 1024 ** 3)
    _g.min_seq = min_seq if min_seq is not None else _env_number(
        "MTLFLASHATTN_SDPA_MIN_SEQ", int, None)
    _g.fast_min_seq = fast_min_seq if fast_min_seq is not None else _env_number(
        "MTLFLASHATTN_SDPA_FAST_MIN_SEQ", int, DEFAULT_FAST_MIN_SEQ)
    _g.orig = F.scaled_dot_product_attention
    F.scaled_dot_product_attention = _patched
    return True


def uninstall():
    """Put the original op back. Returns True if a patch was removed."""
    if _g.orig is None:
        return False
    F.scaled_dot_product_attention = _g.orig
    _g.orig = None
    _g.min_score_bytes = _g.min_seq = _g.fast_min_seq = None
    return True


def calibrate(lengths=(256, 512, 1024, 2048, 4096, 8192), heads=16, dims=(64, 128),
              dtypes=(torch.bfloat16,), causal=(False, True), iters=20, device="cuda"):
    """Time this engine against stock SDPA on this GPU (B=1, ``heads`` heads, Lq = Lk).

    Returns a list of dicts (shape, engine_ms, stock_ms, speedup) and the smallest length at and
    above which the engine is faster on every measured shape: the value to use as
    ``MTLFLASHATTN_SDPA_FAST_MIN_SEQ``. Inputs are N(0,1); each timing is the mean of ``iters``
    calls after three warm-up calls, by CUDA events on the current stream."""
    stock = _g.orig or F.scaled_dot_product_attention
    rows = []
    gen = torch.Generator(device=device).manual_seed(0)
    for dt in dtypes:
        for D in dims:
            for c in causal:
                for L in lengths:
                    q, k, v = (torch.randn(1, heads, L, D, device=device, generator=gen).to(dt)
                               for _ in range(3))

                    def t(fn):
                        for _ in range(3):
                            fn()
                        s = torch.cuda.Event(enable_timing=True)
                        e = torch.cuda.Event(enable_timing=True)
                        s.record()
                        for _ in range(iters):
                            fn()
                        e.record()
                        torch.cuda.synchronize()
                        return s.elapsed_time(e) / iters

                    mine = t(lambda: flash_attn_forward(q, k, v, scale=D ** -0.5, causal=c))
                    theirs = t(lambda: stock(q, k, v, is_causal=c))
                    rows.append(dict(dtype=str(dt).replace("torch.", ""), D=D, causal=c, L=L,
                                     engine_ms=round(mine, 4), stock_ms=round(theirs, 4),
                                     speedup=round(theirs / mine, 3)))
    floor = None
    for L in sorted(lengths, reverse=True):
        if all(r["speedup"] >= 1.0 for r in rows if r["L"] >= L):
            floor = L
        else:
            break
    return rows, floor


if __name__ == "__main__":
    import json
    import sys

    res, floor = calibrate()
    for r in res:
        print(json.dumps(r))
    print(json.dumps({"fast_min_seq": floor}))
    sys.exit(0)
