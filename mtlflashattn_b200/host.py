"""Attention of host-resident tensors, with the PCIe copies overlapped with the compute.

The reference's functions take device tensors only (metal_flash_attn/__init__.py:51-52). A
caller whose q/k/v live in host memory would otherwise copy them in, run the forward and copy
the result out, one after the other. ``flash_attn_host`` / ``flash_attn_varlen_host`` do the
same work through ``mfa_fwd_staged`` (include/mfa.h): the problem is cut into pieces (runs of
query rows, each needing only the key prefix its last row can attend, or runs of whole varlen
sequences) and the copy in of one piece, the forward of the previous one and the copy out of
the one before run at the same time. Results are identical to ``flash_attn_func`` on the same
inputs; the argument semantics are the same.

Inputs should be in pinned memory (``tensor.pin_memory()``): copies from pageable memory are
correct but do not overlap. With ``synchronize=False`` the call returns once the work is
queued on the current CUDA stream; the caller then keeps the inputs alive and synchronizes the
stream before reading the result.
"""
from __future__ import annotations

import math

import torch

from . import _kernel, _lib
from ._kernel import MAX_HEAD_DIM, _BiasParams, _broadcast_alibi_slopes

__all__ = ["flash_attn_host", "flash_attn_varlen_host"]

_DT = (torch.float16, torch.bfloat16, torch.float32)


def _check(q, k, v, window_size, softcap):
    if q.device.type != "cpu" or k.device.type != "cpu" or v.device.type != "cpu":
        raise ValueError("mtlflashattn_b200: flash_attn_host takes host (CPU) tensors")
    if q.dtype not in _DT or k.dtype != q.dtype or v.dtype != q.dtype:
        raise NotImplementedError(
            f"mtlflashattn_b200: dtype {q.dtype} (q/k/v must match, fp16/bf16/fp32)")
    if q.shape[-1] > MAX_HEAD_DIM:
        raise NotImplementedError(f"mtlflashattn_b200: head_dim {q.shape[-1]} > {MAX_HEAD_DIM}")
    if k.shape[-1] != q.shape[-1] or v.shape[-1] != q.shape[-1]:
        raise ValueError("mtlflashattn_b200: q/k/v head_dim mismatch")
    if (not isinstance(window_size, (tuple, list)) or len(window_size) != 2
            or any(not isinstance(w, int) or w < -1 for w in window_size)):
        raise ValueError("mtlflashattn_b200: window_size must be a (left, right) pair of ints >= -1")
    if softcap < 0:
        raise ValueError("mtlflashattn_b200: softcap must be >= 0 (0 disables capping)")


def _staging(t, device):
    """Device buffer with the host tensor's strides (the staged copies move byte ranges)."""
    return torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device=device)


def _out(out, shape, dtype):
    if out is None:
        return torch.empty(shape, dtype=dtype, pin_memory=True)
    if out.device.type != "cpu" or tuple(out.shape) != tuple(shape) or out.dtype != dtype:
        raise ValueError("mtlflashattn_b200: out must be a host tensor of the output's shape/dtype")
    if not out.is_contiguous():
        raise ValueError("mtlflashattn_b200: out must be contiguous")
    return out


def _launch(p, io, device, synchronize, what):
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        rc = _lib.fwd_staged(p, io, stream.cuda_stream)
        if rc != _lib.OK:
            _kernel._raise_status(rc, what)
        if synchronize:
            stream.synchronize()
            _kernel.check_device_errors(device)


def flash_attn_host(q, k, v, softmax_scale=None, causal=False, window_size=(-1, -1),
                    softcap=0.0, alibi_slopes=None, device=None, out=None, chunks=0,
                    synchronize=True):
    """``flash_attn_func`` on host tensors q ``[B, Lq, Hq, D]``, k/v ``[B, Lk, Hkv, D]``.

    Returns the host output ``[B, Lq, Hq, D]`` (``out`` if given, else a new pinned tensor).
    ``device``: the CUDA device that computes (default: the current one). ``chunks``: pipeline
    pieces (0 = automatic, 1 = no overlap)."""
    _check(q, k, v, window_size, softcap)
    q, k, v = _kernel._last_dim_contig(q), _kernel._last_dim_contig(k), _kernel._last_dim_contig(v)
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    B, Lq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"mtlflashattn_b200: num_heads_kv ({Hkv}) must divide num_heads_q ({Hq})")
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    host_o = _out(out, (B, Lq, Hq, D), q.dtype)
    qd, kd, vd = _staging(q, device), _staging(k, device), _staging(v, device)
    od = torch.empty(B, Lq, Hq, D, dtype=q.dtype, device=device)
    alibi = (_broadcast_alibi_slopes(alibi_slopes.to(device), B, Hq, device)
             if alibi_slopes is not None else None)
    bias = _BiasParams(softcap, window_size[0], window_size[1], alibi)
    p = _kernel._params(qd, kd, vd, od, B=B, Hq=Hq, Hkv=Hkv, Lq=Lq, Lk=Lk, D=D,
                        q_st=q.stride()[:3], k_st=k.stride()[:3], v_st=v.stride()[:3],
                        o_st=od.stride()[:3], scale=scale, causal=causal, bias=bias,
                        kernel=_kernel._tier_mode(q.dtype))
    io = _lib.MfaHostIo(q.data_ptr(), k.data_ptr(), v.data_ptr(), host_o.data_ptr(), None, None,
                        int(chunks))
    _launch(p, io, device, synchronize, "flash_attn_host")
    return host_o


def flash_attn_varlen_host(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                           alibi_slopes=None, device=None, out=None, chunks=0, synchronize=True):
    """``flash_attn_varlen_func`` on host tensors q ``[total_q, Hq, D]``, k/v
    ``[total_k, Hkv, D]`` and host int32 ``cu_seqlens_*`` ``[batch + 1]``. Returns the host
    output ``[total_q, Hq, D]``."""
    _check(q, k, v, window_size, softcap)
    q, k, v = _kernel._last_dim_contig(q), _kernel._last_dim_contig(k), _kernel._last_dim_contig(v)
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    cu_q_h = cu_seqlens_q.to("cpu", torch.int32).contiguous()
    cu_k_h = cu_seqlens_k.to("cpu", torch.int32).contiguous()
    batch = cu_q_h.shape[0] - 1
    if cu_k_h.shape[0] != batch + 1:
        raise ValueError("mtlflashattn_b200: cu_seqlens_q and cu_seqlens_k lengths differ")
    total_q, Hq, D = q.shape
    total_k, Hkv = k.shape[0], k.shape[1]
    if int(cu_q_h[-1]) != total_q or int(cu_k_h[-1]) != total_k:
        raise ValueError("mtlflashattn_b200: cu_seqlens[-1] must equal the packed token count")
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"mtlflashattn_b200: num_heads_kv ({Hkv}) must divide num_heads_q ({Hq})")
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    host_o = _out(out, (total_q, Hq, D), q.dtype)
    qd, kd, vd = _staging(q, device), _staging(k, device), _staging(v, device)
    od = torch.empty(total_q, Hq, D, dtype=q.dtype, device=device)
    with torch.cuda.device(device):
        cu_q = cu_q_h.to(device, non_blocking=True)
        cu_k = cu_k_h.to(device, non_blocking=True)
    alibi = (_broadcast_alibi_slopes(alibi_slopes.to(device), batch, Hq, device)
             if alibi_slopes is not None else None)
    bias = _BiasParams(softcap, window_size[0], window_size[1], alibi)
    p = _kernel._params(qd, kd, vd, od, B=batch, Hq=Hq, Hkv=Hkv, Lq=total_q, Lk=total_k, D=D,
                        q_st=(0, q.stride(0), q.stride(1)), k_st=(0, k.stride(0), k.stride(1)),
                        v_st=(0, v.stride(0), v.stride(1)), o_st=(0, od.stride(0), od.stride(1)),
                        scale=scale, causal=causal, bias=bias, kernel=_kernel._tier_mode(q.dtype),
                        cu_q=cu_q, cu_k=cu_k, max_lq=int(max_seqlen_q), max_lk=int(max_seqlen_k))
    io = _lib.MfaHostIo(q.data_ptr(), k.data_ptr(), v.data_ptr(), host_o.data_ptr(),
                        cu_q_h.data_ptr(), cu_k_h.data_ptr(), int(chunks))
    _launch(p, io, device, synchronize, "flash_attn_varlen_host")
    return host_o
