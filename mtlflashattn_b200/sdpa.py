"""Gated ``F.scaled_dot_product_attention`` patch (reference: metal_flash_attn/sdpa.py:1-193).

``install()`` reroutes eligible SDPA calls on CUDA tensors to this engine; everything else, and
any kernel error, falls through to the original op, so the caller never crashes. Gates (any
one fires): correctness (max(Lq, Lk) >= MTLFLASHATTN_SDPA_MIN_SEQ, default 4096), speed (the
tcgen05 kernel would run and max(Lq, Lk) >= MTLFLASHATTN_SDPA_FAST_MIN_SEQ, default 1024) and
memory (score bytes >= MTLFLASHATTN_SDPA_MIN_GB, default 12). Independently of the gates, a
value head dim different from the query/key head dim takes a defensive exact path that keeps
SDPA's top-left causal convention. Kill switch: MTLFLASHATTN_SDPA=off.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from ._kernel import MAX_HEAD_DIM, _select_tier, flash_attn_forward

_SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)

# Kernels that beat stock SDPA even when the score matrix fits (reference: _FAST_TIERS).
_FAST_TIERS = frozenset({"tcgen05"})

_orig = None
_min_score_bytes = None
_min_seq = None
_fast_min_seq = None


def _eligibility(q, k, v, attn_mask, dropout_p, is_causal):
    """Return (eligible, reason); reason names the deciding gate (reference: sdpa.py:33-73)."""
    if q.device.type != "cuda":
        return False, "not-cuda"
    if attn_mask is not None:
        return False, "attn_mask"
    if dropout_p:
        return False, "dropout"
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        return False, f"ndim({q.dim()})"
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        return False, f"dtype({q.dtype})"
    D = q.shape[-1]
    if D > MAX_HEAD_DIM or k.shape[-1] != D or v.shape[-1] != D:
        return False, f"head_dim({D})"
    Hq, Hkv = q.shape[1], k.shape[1]
    if Hkv == 0 or Hq % Hkv != 0:
        return False, f"heads({Hq}/{Hkv})"
    if k.shape[2] != v.shape[2]:
        return False, "kv-len-mismatch"
    Lq, Lk = q.shape[2], k.shape[2]
    # SDPA's is_causal is top-left aligned; the kernel is bottom-right. Same only if Lq == Lk.
    if is_causal and Lq != Lk:
        return False, "causal-cross-length"
    maxlen = max(Lq, Lk)
    if maxlen >= _min_seq:
        return True, "correctness-large-seq"
    if maxlen >= _fast_min_seq and _select_tier(q, k, v) in _FAST_TIERS:
        return True, "fast-tier"
    score_bytes = q.shape[0] * Hq * Lq * Lk * 2
    if score_bytes >= _min_score_bytes:
        return True, "oom-rescue"
    return False, f"fits({score_bytes / 1024**3:.2f}GB)"


def _uneven_v_attention(query, key, value, attn_mask, is_causal, scale, enable_gqa=False,
                        q_chunk=4096):
    """Exact chunked-fp32 attention for value head dim != query/key head dim, with SDPA's
    top-left causal alignment and additive/boolean masks (reference: sdpa.py:76-130)."""
    Hq, Hkv = query.shape[1], key.shape[1]
    if Hq != Hkv:
        if not (enable_gqa and Hkv != 0 and Hq % Hkv == 0):
            raise ValueError(
                f"mtlflashattn_b200: SDPA query/kv head mismatch (Hq={Hq}, Hkv={Hkv}); "
                "pass enable_gqa=True for GQA/MQA"
            )
        rep = Hq // Hkv
        key = key.repeat_interleave(rep, dim=1)
        value = value.repeat_interleave(rep, dim=1)
    s = scale if scale is not None else 1.0 / math.sqrt(query.shape[-1])
    Lq, Lk = query.shape[-2], key.shape[-2]
    bias = None
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            bias = torch.zeros(attn_mask.shape, dtype=torch.float32, device=query.device)
            bias = bias.masked_fill(~attn_mask, float("-inf"))
        else:
            bias = attn_mask.float()
    key_t = key.float().transpose(-2, -1)
    value_f = value.float()
    outs = []
    for i in range(0, Lq, q_chunk):
        qi = query[..., i:i + q_chunk, :].float()
        scores = torch.matmul(qi, key_t) * s
        if bias is not None:
            scores = scores + (bias[..., i:i + qi.shape[-2], :] if bias.shape[-2] == Lq else bias)
        if is_causal:
            qpos = torch.arange(i, i + qi.shape[-2], device=query.device).unsqueeze(-1)
            kpos = torch.arange(Lk, device=query.device).unsqueeze(0)
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
        probs = torch.nan_to_num(scores.softmax(dim=-1), nan=0.0)
        outs.append(torch.matmul(probs, value_f))
    return torch.cat(outs, dim=-2).to(value.dtype)


def _sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
          **kwargs):
    eligible, _ = _eligibility(query, key, value, attn_mask, dropout_p, is_causal)
    if eligible:
        try:
            s = scale if scale is not None else 1.0 / math.sqrt(query.shape[-1])
            return flash_attn_forward(query, key, value, scale=s, causal=is_causal)
        except Exception as e:  # never crash the caller: fall back to stock SDPA
            print(f"[mtlflashattn_b200/sdpa] kernel fell back ({e}); using stock SDPA")
    if (query.device.type == "cuda" and not dropout_p and query.dim() == 4 and value.dim() == 4
            and value.shape[-1] != query.shape[-1]):
        return _uneven_v_attention(query, key, value, attn_mask, is_causal, scale,
                                   enable_gqa=kwargs.get("enable_gqa", False))
    return _orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                 is_causal=is_causal, scale=scale, **kwargs)


def install(min_score_gb=None, min_seq=None, fast_min_seq=None):
    """Patch F.scaled_dot_product_attention. Returns True if newly installed."""
    global _orig, _min_score_bytes, _min_seq, _fast_min_seq
    if _orig is not None:
        return False
    if os.environ.get("MTLFLASHATTN_SDPA", "auto").lower() in ("off", "0", "false"):
        return False
    if min_score_gb is None:
        min_score_gb = float(os.environ.get("MTLFLASHATTN_SDPA_MIN_GB", "12"))
    if min_seq is None:
        min_seq = int(os.environ.get("MTLFLASHATTN_SDPA_MIN_SEQ", "4096"))
    if fast_min_seq is None:
        fast_min_seq = int(os.environ.get("MTLFLASHATTN_SDPA_FAST_MIN_SEQ", "1024"))
    _min_score_bytes = int(min_score_gb * (1024 ** 3))
    _min_seq = min_seq
    _fast_min_seq = fast_min_seq
    _orig = F.scaled_dot_product_attention
    F.scaled_dot_product_attention = _sdpa
    torch.nn.functional.scaled_dot_product_attention = _sdpa
    return True


def uninstall():
    """Restore the original op. Returns True if a patch was removed."""
    global _orig, _min_score_bytes, _min_seq, _fast_min_seq
    if _orig is None:
        return False
    F.scaled_dot_product_attention = _orig
    torch.nn.functional.scaled_dot_product_attention = _orig
    _orig = None
    _min_score_bytes = None
    _min_seq = None
    _fast_min_seq = None
    return True
