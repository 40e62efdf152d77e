"""The boundary: ``flash_attn_forward`` and the launch helpers under the public API.

``flash_attn_forward`` keeps the signature, argument meaning, return layout and errors of the
reference's boundary function (metal_flash_attn/_kernel.py:1052-1153): heads-second
``[B, H, L, D]`` tensors of any strides in, a new contiguous ``[B, Hq, Lq, D]`` tensor in
``q.dtype`` out. Underneath, the reference's Metal tier dispatch is replaced by one call into
libmfa.so (include/mfa.h), which runs either the tcgen05 tensor-core kernel or the fp32
CUDA-core kernel. Tensors cross that boundary only as pointers, strides and sizes; no layout
copy is made for strided views.

Tier names. ``MTLFLASHATTN_KERNEL`` accepts ``auto`` (default), ``tcgen05`` and ``simt``, and,
for drop-in compatibility, the reference's tier names: ``v1``, ``v2``, ``v2_bf16`` map to
``tcgen05``; ``v0`` and ``v2_fp32`` map to ``simt``; ``v2_dtype`` picks by dtype. A forced tier
that cannot run the input raises RuntimeError, as in the reference (_kernel.py:1083-1139).
The reference's ``torch`` tier is not part of this engine: that chunked-fp32 algorithm lives in
``oracle/`` as the test checker only, and selecting it here raises RuntimeError.
"""
from __future__ import annotations

import array
import atexit
import collections
import ctypes
import os
import struct
import sys
import threading
from collections import namedtuple

import torch

from . import _lib

MAX_HEAD_DIM = 128

# Bias/masking knobs, as in the reference (_kernel.py:20-24): softcap (0 = off),
# window_left/window_right (-1 = open), alibi: [B*Hq] fp32 slopes already broadcast, or None.
_BiasParams = namedtuple("_BiasParams", "softcap window_left window_right alibi")

_DTYPES = {torch.float16: _lib.FP16, torch.bfloat16: _lib.BF16, torch.float32: _lib.FP32}

_TIER_ALIASES = {
    "auto": "auto", "cuda": "auto",
    "tcgen05": "tcgen05", "tc": "tcgen05", "v1": "tcgen05", "v2": "tcgen05",
    "v2_bf16": "tcgen05",
    "simt": "simt", "v0": "simt", "v2_fp32": "simt",
    "v2_dtype": "dtype", "v2_typed": "dtype",
}


_ENV_DATA = getattr(os.environ, "_data", None)


def _env(name, default=""):
    """os.environ.get for the per-call knobs, without its per-call str -> bytes encoding (the
    POSIX environ mapping keeps its data keyed by bytes); falls back to os.environ.get."""
    if _ENV_DATA is not None and os.name == "posix":
        v = _ENV_DATA.get(name.encode() if name not in _ENV_KEYS else _ENV_KEYS[name])
        return default if v is None else v.decode()
    return os.environ.get(name, default)


_ENV_KEYS = {n: n.encode() for n in ("MTLFLASHATTN_KERNEL", "MTLFLASHATTN_TRACE",
                                     "MTLFLASHATTN_SYNC_CHECK")}


def _tier_mode(dtype) -> int:
    raw = _env("MTLFLASHATTN_KERNEL", "auto").lower()
    if raw in ("torch", "pytorch"):
        raise RuntimeError(
            "mtlflashattn_b200: the chunked-fp32 torch tier is not part of this engine "
            "(it is the test oracle); use MTLFLASHATTN_KERNEL=auto|tcgen05|simt"
        )
    mode = _TIER_ALIASES.get(raw)
    if mode is None:
        raise RuntimeError(f"mtlflashattn_b200: unknown MTLFLASHATTN_KERNEL={raw!r}")
    if mode == "dtype":
        mode = "simt" if dtype == torch.float32 else "tcgen05"
    return {"auto": _lib.KERNEL_AUTO, "tcgen05": _lib.KERNEL_TCGEN05,
            "simt": _lib.KERNEL_SIMT}[mode]


# ------------------------------------------------------------------------------------ trace
class _CallTrace(collections.Counter):
    """Per-process tally of forward calls by (dtype, D, Lq, Lk, causal, kernel label), printed
    to stderr at exit when MTLFLASHATTN_TRACE is on. The line format is the reference's
    (metal_flash_attn/_kernel.py:1032-1049) because users and scripts read it."""

    def record(self, dtype, D, Lq, Lk, causal, label):
        """Count one call; a malformed entry is dropped, never raised
        (reference: _kernel.py:1022-1029)."""
        try:
            key = (str(dtype).removeprefix("torch."), int(D), int(Lq), int(Lk), bool(causal),
                   str(label))
        except (TypeError, ValueError):
            return
        self[key] += 1

    def summary(self):
        if not self:
            return []
        head = (f"[MTLFLASHATTN_TRACE] {sum(self.values())} attention call(s), "
                f"{len(self)} distinct shape/kernel combos:")
        body = [f"  calls={n:<6} {dt:<9} D={D:<4} Lq={Lq:<6} Lk={Lk:<6} "
                f"causal={'T' if causal else 'F'}  -> {label}"
                for (dt, D, Lq, Lk, causal, label), n in sorted(self.items(),
                                                                 key=lambda kv: (-kv[1], kv[0]))]
        return [head, *body]


_trace = _CallTrace()
_record_trace = _trace.record
_trace_summary_lines = _trace.summary


def _trace_enabled():
    return _env("MTLFLASHATTN_TRACE").lower() in ("1", "on", "true", "yes")


@atexit.register
def _trace_atexit():
    if _trace_enabled() and _trace:
        sys.stderr.write("\n".join(_trace.summary()) + "\n")
        sys.stderr.flush()


# ------------------------------------------------------------------------ device error word
_err_words = {}


def _err_word(device):
    t = _err_words.get(device)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _err_words[device] = t
    return t


def check_device_errors(device=None):
    """Synchronise and raise if any kernel on ``device`` reported a bounded-wait timeout."""
    dev = torch.device(device) if device is not None else torch.device("cuda")
    if dev.index is None:  # "cuda" names the current device; the words are keyed by index
        dev = torch.device("cuda", torch.cuda.current_device())
    t = _err_words.get(dev)
    if t is None:
        return
    torch.cuda.synchronize(dev)
    v = int(t.item())
    if v != 0:
        t.zero_()
        why = ("a kernel gave up on a bounded wait" if v == _lib.ERR_TIMEOUT else
               "a split launch met a varlen row at or past Lq (Lq < cu_seqlens[-1])"
               if v == _lib.ERR_INVALID else
               "a device-side bounds check (MFA_CHECKS build) failed" if v == _lib.ERR_CHECK
               else "a kernel reported an error")
        raise _lib.MfaError(v, why + "; its output is invalid")


def _sync_check_enabled():
    return _env("MTLFLASHATTN_SYNC_CHECK").lower() in ("1", "on", "true", "yes")


# --------------------------------------------------------------------------------- launch
def _broadcast_alibi_slopes(alibi_slopes, B, Hq, device):
    """Flatten slopes ``[Hq]`` or ``[B, Hq]`` to contiguous fp32 ``[B*Hq]``
    (reference: _kernel.py:1275-1285)."""
    s = alibi_slopes.to(device=device, dtype=torch.float32)
    if s.dim() == 1 and s.shape[0] == Hq:
        s = s.unsqueeze(0).expand(B, Hq)
    elif not (s.dim() == 2 and tuple(s.shape) == (B, Hq)):
        raise ValueError(
            f"mtlflashattn_b200: alibi_slopes must be [Hq={Hq}] or [B={B}, Hq={Hq}], "
            f"got {tuple(s.shape)}"
        )
    return s.reshape(-1).contiguous()


def _last_dim_contig(t):
    return t if t.stride(-1) == 1 else t.contiguous()


def _raise_status(rc, what):
    if rc == _lib.ERR_INVALID:
        raise ValueError(f"mtlflashattn_b200: {what}: {_lib.status_string(rc)}")
    if rc == _lib.ERR_UNSUPPORTED:
        raise NotImplementedError(f"mtlflashattn_b200: {what}: {_lib.status_string(rc)}")
    raise _lib.MfaError(rc, what)


_PACK = struct.Struct(_lib.PARAMS_FORMAT)
_WS = struct.Struct("<QQ")
_tls = threading.local()


def _values(q, k, v, o, B, Hq, Hkv, Lq, Lk, D, q_st, k_st, v_st, o_st, scale, causal, bias,
            kernel, lse, lse_st, cu_q, cu_k, max_lq, max_lk, k_pos_offset, lk_total,
            cu_q_host=0):
    """The fields of ``struct mfa_fwd_params`` in declaration order (workspace left empty)."""
    return (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
            lse.data_ptr() if lse is not None else 0,
            *q_st, *k_st, *v_st, *o_st, *lse_st,
            B, Hq, Hkv, Lq, Lk, D,
            cu_q.data_ptr() if cu_q is not None else 0,
            cu_k.data_ptr() if cu_k is not None else 0,
            max_lq, max_lk, float(scale), float(bias.softcap), 1 if causal else 0,
            int(bias.window_left), int(bias.window_right),
            bias.alibi.data_ptr() if bias.alibi is not None else 0,
            _DTYPES[q.dtype], _DTYPES[o.dtype], int(k_pos_offset), int(lk_total), kernel,
            _err_word(q.device).data_ptr(), 0, 0, cu_q_host)


def _params(q, k, v, o, *, B, Hq, Hkv, Lq, Lk, D, q_st, k_st, v_st, o_st, scale, causal,
            bias: _BiasParams, kernel, lse=None, lse_st=(0, 0), cu_q=None, cu_k=None,
            max_lq=0, max_lk=0, k_pos_offset=0, lk_total=0):
    """An ``MfaFwdParams`` (ctypes) for these tensors: for callers that inspect or edit fields
    (the host-staged path, the plan queries, tests). The forward itself uses ``_packed``."""
    vals = _values(q, k, v, o, B, Hq, Hkv, Lq, Lk, D, q_st, k_st, v_st, o_st, scale, causal,
                   bias, kernel, lse, lse_st, cu_q, cu_k, max_lq, max_lk, k_pos_offset, lk_total)
    return _lib.MfaFwdParams.from_buffer_copy(_PACK.pack(*vals))


_tls_host = threading.local()


def _host_i32(values):
    """Address of a host int32 copy of ``values`` (0 for None), valid until the next call on
    this thread."""
    if values is None:
        return 0
    arr = array.array("i", values)
    _tls_host.keep = arr
    return arr.buffer_info()[0]


def _packed(*args):
    """The same params packed into this thread's reusable buffer (valid until the next call on
    this thread; libmfa reads it only during the call)."""
    buf = getattr(_tls, "buf", None)
    if buf is None:
        buf = _tls.buf = ctypes.create_string_buffer(_PACK.size)
    _PACK.pack_into(buf, 0, *_values(*args))
    return buf


_workspaces = {}  # (device, stream) -> uint8 tensor


def _workspace(dev, stream, need):
    """Split-KV scratch for launches on ``stream``: one buffer per (device, stream), grown on
    demand and reused by every later call. Work on one stream runs in order, so a call never
    overwrites partials an earlier call still reads; a replaced buffer goes back to torch's
    caching allocator, which keeps it until the work queued on its stream is done. Saves a
    torch.empty per decode-sized call."""
    key = (dev, stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws


def _run(p, q, what, causal, trace_shape, kernel, D):
    dev = q.device
    ctx = torch.cuda.device(dev) if dev.index != torch.cuda.current_device() else None
    if ctx is not None:
        ctx.__enter__()
    try:
        if _trace_enabled():
            sel = _lib.select_kernel(p)
            label = "cuda/" + _lib.KERNEL_NAMES.get(sel, "rejected")
            _record_trace(q.dtype, trace_shape[0], trace_shape[1], trace_shape[2], causal, label)
        stream = torch._C._cuda_getCurrentRawStream(dev.index)  # the current stream's handle
        need = _lib.workspace_size(p)
        if need > 0:  # few query rows: let the library split the keys over more CTAs
            ws = _workspace(dev, stream, need)
            _WS.pack_into(p, _lib.WORKSPACE_OFFSET, ws.data_ptr(), need)
        rc = _lib.fwd(p, stream)
        if rc != _lib.OK:
            if rc == _lib.ERR_UNSUPPORTED and kernel != _lib.KERNEL_AUTO:
                raise RuntimeError(
                    f"mtlflashattn_b200: {_lib.KERNEL_NAMES.get(kernel)} kernel forced but "
                    f"ineligible (dtype={q.dtype}, D={D}; needs fp16/bf16, D%8==0, "
                    f"16-byte aligned strides, sm_100 device)"
                )
            _raise_status(rc, what)
    finally:
        if ctx is not None:
            ctx.__exit__(None, None, None)
    if _sync_check_enabled():
        check_device_errors(dev)


def _check_tensors(q, k, v):
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("mtlflashattn_b200 requires CUDA tensors (B200 / sm_100a)")
    if k.device != q.device or v.device != q.device:
        raise ValueError("mtlflashattn_b200: q/k/v must be on the same device")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise NotImplementedError(f"mtlflashattn_b200: dtype {q.dtype} (q/k/v must match, fp16/bf16/fp32)")


def forward_bshd(q, k, v, out, scale, causal, bias: _BiasParams, lse=None, k_pos_offset=0,
                 lk_total=0):
    """Attention on heads-third ``[B, L, H, D]`` tensors of any strides, writing into ``out``
    (``[B, Lq, Hq, D]``, any strides, fp16/bf16/fp32). ``lse`` is an optional fp32
    ``[B, Hq, Lq]`` tensor. Launches exactly one kernel; no layout copies."""
    _check_tensors(q, k, v)
    qs, ks, vs, os_ = q.stride(), k.stride(), v.stride(), out.stride()
    if qs[3] != 1:
        q = q.contiguous()
        qs = q.stride()
    if ks[3] != 1:
        k = k.contiguous()
        ks = k.stride()
    if vs[3] != 1:
        v = v.contiguous()
        vs = v.stride()
    B, Lq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"mtlflashattn_b200: num_heads_kv ({Hkv}) must divide num_heads_q ({Hq})")
    if D > MAX_HEAD_DIM:
        raise NotImplementedError(f"mtlflashattn_b200: head_dim {D} > {MAX_HEAD_DIM}")
    if os_[3] != 1:
        raise ValueError("mtlflashattn_b200: out must have a contiguous last dimension")
    kernel = _tier_mode(q.dtype)
    p = _packed(q, k, v, out, B, Hq, Hkv, Lq, Lk, D, qs[:3], ks[:3], vs[:3], os_[:3], scale,
                causal, bias, kernel, lse, lse.stride()[:2] if lse is not None else (0, 0), None,
                None, 0, 0, k_pos_offset, lk_total)
    _run(p, q, "flash_attn_forward", causal, (D, Lq, Lk), kernel, D)
    return out


def forward_varlen(q, k, v, out, cu_q, cu_k, max_lq, max_lk, scale, causal, bias: _BiasParams,
                   lse=None, cu_q_host=None):
    """Packed varlen attention in ONE launch: q ``[total_q, Hq, D]``, k/v ``[total_k, Hkv, D]``,
    device int32 ``cu_q``/``cu_k`` ``[batch+1]``; ``bias.alibi`` is ``[batch*Hq]`` or None.
    ``lse`` is an optional fp32 ``[Hq, total_q]`` tensor. ``cu_q_host``, the same offsets as a
    host list, lets the library launch exactly the CTAs the sequences need."""
    _check_tensors(q, k, v)
    q, k, v = _last_dim_contig(q), _last_dim_contig(k), _last_dim_contig(v)
    total_q, Hq, D = q.shape
    total_k, Hkv = k.shape[0], k.shape[1]
    batch = cu_q.shape[0] - 1
    kernel = _tier_mode(q.dtype)
    p = _packed(q, k, v, out, batch, Hq, Hkv, total_q, total_k, D, (0, q.stride(0), q.stride(1)),
                (0, k.stride(0), k.stride(1)), (0, v.stride(0), v.stride(1)),
                (0, out.stride(0), out.stride(1)), scale, causal, bias, kernel, lse,
                (0, lse.stride(0)) if lse is not None else (0, 0), cu_q, cu_k, max_lq, max_lk,
                0, 0, _host_i32(cu_q_host))
    _run(p, q, "flash_attn_varlen_func", causal, (D, max_lq, max_lk), kernel, D)
    return out


def flash_attn_forward(q, k, v, scale, causal, softcap=0.0, window_left=-1, window_right=-1,
                       alibi_slopes=None):
    """q: [B,Hq,Lq,D], k/v: [B,Hkv,Lk,D] (heads-second, any strides).

    Returns [B,Hq,Lq,D] contiguous, in q.dtype (reference: _kernel.py:1052-1153).
    """
    if softcap < 0:
        raise ValueError("mtlflashattn_b200: softcap must be >= 0 (0 disables capping)")
    _check_tensors(q, k, v)
    B, Hq, Lq, D = q.shape
    alibi = (_broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
             if alibi_slopes is not None else None)
    bias = _BiasParams(softcap, window_left, window_right, alibi)
    out = torch.empty(B, Hq, Lq, D, device=q.device, dtype=q.dtype)
    forward_bshd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), out.transpose(1, 2),
                 scale, causal, bias)
    return out


def _select_tier(q, k, v):
    """Kernel ``auto`` would run for heads-second tensors: 'tcgen05', 'simt' or 'rejected'."""
    try:
        qb, kb, vb = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        B, Lq, Hq, D = qb.shape
        p = _params(qb, kb, vb, qb, B=B, Hq=Hq, Hkv=kb.shape[2], Lq=Lq, Lk=kb.shape[1], D=D,
                    q_st=(qb.stride(0), qb.stride(1), qb.stride(2)),
                    k_st=(kb.stride(0), kb.stride(1), kb.stride(2)),
                    v_st=(vb.stride(0), vb.stride(1), vb.stride(2)),
                    o_st=(qb.stride(0), qb.stride(1), qb.stride(2)),
                    scale=1.0, causal=False, bias=_BiasParams(0.0, -1, -1, None),
                    kernel=_lib.KERNEL_AUTO)
        with torch.cuda.device(q.device):
            return _lib.KERNEL_NAMES.get(_lib.select_kernel(p), "rejected")
    except Exception:
        return "rejected"
