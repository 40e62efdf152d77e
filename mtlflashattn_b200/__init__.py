"""B200-native flash-attention forward with the ``metal_flash_attn`` / CUDA ``flash_attn`` 2.x
function surface.

Inference-only (no backward). Unsupported features raise NotImplementedError so callers can
fall back, as in the reference (metal_flash_attn/__init__.py:1-5). Every public function ends
in exactly one launch of libmfa.so; ``flash_attn_varlen_func`` runs all sequences in one launch
instead of the reference's per-sequence Python loop (metal_flash_attn/__init__.py:165-182).
"""
from __future__ import annotations

import math

import torch

from ._kernel import MAX_HEAD_DIM, _BiasParams, _broadcast_alibi_slopes, flash_attn_forward
from . import _kernel
from ._version import __version__
from .host import flash_attn_host, flash_attn_varlen_host

__all__ = [
    "flash_attn_func",
    "flash_attn_varlen_func",
    "flash_attn_qkvpacked_func",
    "flash_attn_kvpacked_func",
    "flash_attn_varlen_qkvpacked_func",
    "flash_attn_varlen_kvpacked_func",
    "flash_attn_forward",
    "flash_attn_host",
    "flash_attn_varlen_host",
    "__version__",
]

_SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _check_supported(q, k, v, dropout_p, window_size, softcap, alibi_slopes,
                     deterministic, return_attn_probs):
    """Same checks, order and exception types as the reference (metal_flash_attn/__init__.py:28-59);
    the device check accepts CUDA instead of MPS."""
    if dropout_p:
        raise NotImplementedError("mtlflashattn_b200: dropout_p > 0 not supported (inference-only)")
    if (
        not isinstance(window_size, (tuple, list))
        or len(window_size) != 2
        or any(not isinstance(w, int) or isinstance(w, bool) or w < -1 for w in window_size)
    ):
        raise ValueError(
            "mtlflashattn_b200: window_size must be a (left, right) pair of ints >= -1 "
            "(-1 = unbounded on that side)"
        )
    if softcap < 0:
        raise ValueError("mtlflashattn_b200: softcap must be >= 0 (0 disables capping)")
    if alibi_slopes is not None and not torch.is_tensor(alibi_slopes):
        raise TypeError("mtlflashattn_b200: alibi_slopes must be a tensor of per-head slopes")
    if deterministic:
        raise NotImplementedError("mtlflashattn_b200: deterministic not supported")
    if return_attn_probs:
        raise NotImplementedError(
            "mtlflashattn_b200: return_attn_probs not supported (probs never materialized)")
    if q.device.type != "cuda":
        raise NotImplementedError(
            f"mtlflashattn_b200: device {q.device.type!r} not supported (CUDA only)")
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise NotImplementedError(
            f"mtlflashattn_b200: dtype {q.dtype} (q/k/v must match, fp16/bf16/fp32)")
    D = q.shape[-1]
    if D > MAX_HEAD_DIM:
        raise NotImplementedError(f"mtlflashattn_b200: head_dim {D} > {MAX_HEAD_DIM}")
    if k.shape[-1] != D or v.shape[-1] != D:
        raise ValueError("mtlflashattn_b200: q/k/v head_dim mismatch")


class _NoBackward(torch.autograd.Function):
    """Marks the output as produced by an inference-only op: backward raises."""

    @staticmethod
    def forward(ctx, out, *inputs):
        return out.view_as(out)

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("mtlflashattn_b200: backward is not supported (inference-only)")


def _guard_grad(out, *inputs):
    if torch.is_grad_enabled():
        ts = [t for t in inputs if torch.is_tensor(t)]
        if any(t.requires_grad for t in ts):
            return _NoBackward.apply(out, *ts)
    return out


def flash_attn_func(
    q,
    k,
    v,
    dropout_p=0.0,
    softmax_scale=None,
    causal=False,
    window_size=(-1, -1),
    softcap=0.0,
    alibi_slopes=None,
    deterministic=False,
    return_attn_probs=False,
):
    """Drop-in for flash_attn.flash_attn_func (forward only).

    q: [B, Lq, Hq, D]; k, v: [B, Lk, Hkv, D]. Hkv must divide Hq (GQA/MQA).
    Returns [B, Lq, Hq, D] in q.dtype (reference: metal_flash_attn/__init__.py:62-99; the
    output is written in place in this layout, so no transpose copy follows the kernel).
    """
    _check_supported(q, k, v, dropout_p, window_size, softcap, alibi_slopes,
                     deterministic, return_attn_probs)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"mtlflashattn_b200: expected 4-D [B,S,H,D] tensors, got q.dim()={q.dim()}")
    Hq, Hkv = q.shape[2], k.shape[2]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"mtlflashattn_b200: num_heads_kv ({Hkv}) must divide num_heads_q ({Hq})")
    if k.shape[1] != v.shape[1]:
        raise ValueError("mtlflashattn_b200: k/v seqlen mismatch")

    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Lq = q.shape[0], q.shape[1]
    alibi = (_broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
             if alibi_slopes is not None else None)
    bias = _BiasParams(softcap, window_size[0], window_size[1], alibi)
    out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    # the kernel reads raw pointers: no autograd graph is recorded, so no detach is needed
    _kernel.forward_bshd(q, k, v, out, scale, causal, bias)
    return _guard_grad(out, q, k, v)


def flash_attn_varlen_func(
    q,
    k,
    v,
    cu_seqlens_q,
    cu_seqlens_k,
    max_seqlen_q,
    max_seqlen_k,
    dropout_p=0.0,
    softmax_scale=None,
    causal=False,
    window_size=(-1, -1),
    softcap=0.0,
    alibi_slopes=None,
    deterministic=False,
    return_attn_probs=False,
    block_table=None,
):
    """Drop-in for flash_attn.flash_attn_varlen_func (forward only).

    q: [total_q, Hq, D]; k, v: [total_k, Hkv, D] packed without padding;
    cu_seqlens_*: [B+1] int32 cumulative sequence lengths. Returns [total_q, Hq, D] in q.dtype.
    Checks and errors follow the reference (metal_flash_attn/__init__.py:102-183), including
    its host read of cu_seqlens; all sequences then run in one launch. ``max_seqlen_*`` are
    accepted and, as in the reference, not trusted: the launch uses the lengths read from
    cu_seqlens.
    """
    _check_supported(q, k, v, dropout_p, window_size, softcap, alibi_slopes,
                     deterministic, return_attn_probs)
    if block_table is not None:
        raise NotImplementedError("mtlflashattn_b200: block_table (paged KV cache) not supported")
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError(f"mtlflashattn_b200: expected 3-D [total,H,D] tensors, got q.dim()={q.dim()}")
    if cu_seqlens_q.shape[0] != cu_seqlens_k.shape[0]:
        raise ValueError(
            f"mtlflashattn_b200: cu_seqlens_q ({cu_seqlens_q.shape[0]}) and "
            f"cu_seqlens_k ({cu_seqlens_k.shape[0]}) imply different batch sizes"
        )
    Hq, Hkv = q.shape[1], k.shape[1]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"mtlflashattn_b200: num_heads_kv ({Hkv}) must divide num_heads_q ({Hq})")
    if k.shape[0] != v.shape[0]:
        raise ValueError("mtlflashattn_b200: k/v total token count mismatch")

    cu_q = cu_seqlens_q.tolist()
    cu_k = cu_seqlens_k.tolist()
    if cu_q[-1] != q.shape[0]:
        raise ValueError(f"mtlflashattn_b200: cu_seqlens_q[-1]={cu_q[-1]} != total_q={q.shape[0]}")
    if cu_k[-1] != k.shape[0]:
        raise ValueError(f"mtlflashattn_b200: cu_seqlens_k[-1]={cu_k[-1]} != total_k={k.shape[0]}")

    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    batch = len(cu_q) - 1
    if (alibi_slopes is not None and alibi_slopes.dim() == 2
            and tuple(alibi_slopes.shape) != (batch, Hq)):
        raise ValueError(
            f"mtlflashattn_b200: alibi_slopes must be [Hq={Hq}] or [B={batch}, Hq={Hq}], "
            f"got {tuple(alibi_slopes.shape)}"
        )
    lens_q = [cu_q[i + 1] - cu_q[i] for i in range(batch)]
    lens_k = [cu_k[i + 1] - cu_k[i] for i in range(batch)]
    if batch == 0 or max(lens_q) <= 0:
        return _guard_grad(out, q, k, v)
    if any(n < 0 for n in lens_q) or any(n < 0 for n in lens_k):
        raise ValueError("mtlflashattn_b200: cu_seqlens must be nondecreasing")
    alibi = None
    if alibi_slopes is not None:
        # the reference applies [Hq] slopes per sequence (each a B=1 call), [batch, Hq] by row
        alibi = _broadcast_alibi_slopes(alibi_slopes, batch, Hq, q.device)
    bias = _BiasParams(softcap, window_size[0], window_size[1], alibi)
    cu_q_dev = _as_cu(cu_seqlens_q, q.device)
    cu_k_dev = _as_cu(cu_seqlens_k, q.device)
    _kernel.forward_varlen(q, k, v, out, cu_q_dev, cu_k_dev, max(lens_q), max(lens_k), scale,
                           causal, bias, cu_q_host=cu_q)
    return _guard_grad(out, q, k, v)


def _as_cu(cu, device):
    if cu.device == device and cu.dtype == torch.int32 and cu.is_contiguous():
        return cu
    return cu.to(device=device, dtype=torch.int32).contiguous()


def flash_attn_qkvpacked_func(qkv, *args, **kwargs):
    """Drop-in for flash_attn.flash_attn_qkvpacked_func. qkv: [B, S, 3, H, D]."""
    if qkv.dim() != 5 or qkv.shape[2] != 3:
        raise ValueError(f"mtlflashattn_b200: expected qkv [B,S,3,H,D], got {tuple(qkv.shape)}")
    q, k, v = qkv.unbind(dim=2)
    return flash_attn_func(q, k, v, *args, **kwargs)


def flash_attn_kvpacked_func(q, kv, *args, **kwargs):
    """Drop-in for flash_attn.flash_attn_kvpacked_func. kv: [B, Sk, 2, Hkv, D]."""
    if kv.dim() != 5 or kv.shape[2] != 2:
        raise ValueError(f"mtlflashattn_b200: expected kv [B,S,2,H,D], got {tuple(kv.shape)}")
    k, v = kv.unbind(dim=2)
    return flash_attn_func(q, k, v, *args, **kwargs)


def flash_attn_varlen_qkvpacked_func(qkv, cu_seqlens, max_seqlen, *args, **kwargs):
    """Drop-in for flash_attn.flash_attn_varlen_qkvpacked_func. qkv: [total, 3, H, D]."""
    if qkv.dim() != 4 or qkv.shape[1] != 3:
        raise ValueError(f"mtlflashattn_b200: expected qkv [total,3,H,D], got {tuple(qkv.shape)}")
    q, k, v = qkv.unbind(dim=1)
    return flash_attn_varlen_func(q, k, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen,
                                  *args, **kwargs)


def flash_attn_varlen_kvpacked_func(q, kv, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                    max_seqlen_k, *args, **kwargs):
    """Drop-in for flash_attn.flash_attn_varlen_kvpacked_func. kv: [total_k, 2, Hkv, D]."""
    if kv.dim() != 4 or kv.shape[1] != 2:
        raise ValueError(f"mtlflashattn_b200: expected kv [total,2,H,D], got {tuple(kv.shape)}")
    k, v = kv.unbind(dim=1)
    return flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                  max_seqlen_k, *args, **kwargs)
