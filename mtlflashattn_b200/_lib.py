"""ctypes binding of libmfa.so (C ABI declared in include/mfa.h).

The shared library is built in-tree by ``mtlflashattn_b200.build`` and loaded from this
package's directory (or from ``MTLFLASHATTN_LIB``, the path of another build of it). Nothing here falls back to another implementation: if the library is
missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmfa.so")

MFA_ABI_VERSION = 8

# mfa_status
OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_NO_DEVICE = 5
ERR_FAULT_INJECTED = 6
ERR_SCRATCH_TOO_SMALL = 7
ERR_CHECK = 8

# mfa_dtype
FP16, BF16, FP32 = 0, 1, 2

# mfa_kernel
KERNEL_AUTO, KERNEL_TCGEN05, KERNEL_SIMT = 0, 1, 2
KERNEL_NAMES = {KERNEL_TCGEN05: "tcgen05", KERNEL_SIMT: "simt"}

# Every symbol include/mfa.h declares.
EXPORTED_SYMBOLS = (
    "mfa_fwd",
    "mfa_fwd_noalloc",
    "mfa_fwd_staged",
    "mfa_fwd_workspace_size",
    "mfa_fwd_num_splits",
    "mfa_fwd_packed_heads",
    "mfa_select_kernel",
    "mfa_lse_combine",
    "mfa_lse_rescale_sum",
    "mfa_fwd_scatter",
    "mfa_lse_merge",
    "mfa_lse_merge_rows",
    "mfa_peer_alloc",
    "mfa_peer_open",
    "mfa_peer_close",
    "mfa_peer_free",
    "mfa_selftest_wait_timeout",
    "mfa_status_string",
    "mfa_abi_version",
)


class MfaFwdParams(ctypes.Structure):
    """Mirror of ``struct mfa_fwd_params`` (include/mfa.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("lse_stride", ctypes.c_int64 * 2),
        ("B", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32),
        ("Lq", ctypes.c_int32),
        ("Lk", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("cu_q", ctypes.c_void_p),
        ("cu_k", ctypes.c_void_p),
        ("max_lq", ctypes.c_int32),
        ("max_lk", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("softcap", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("win_left", ctypes.c_int32),
        ("win_right", ctypes.c_int32),
        ("alibi", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("o_dtype", ctypes.c_int32),
        ("k_pos_offset", ctypes.c_int32),
        ("lk_total", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("err", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("cu_q_host", ctypes.c_void_p),
    ]


# The same layout as one struct.pack format (native little-endian sizes, explicit padding), so
# the hot path fills a reusable buffer with one pack_into call instead of ~40 ctypes field
# assignments (about 1.5 us against 8 us per forward). The offsets of the two workspace fields
# let a caller patch them after sizing the workspace.
PARAMS_FORMAT = "<5Q12q2q6i2Q2i2f3i4xQ5i4xQQQQ"
WORKSPACE_OFFSET = 264  # workspace pointer, then workspace_bytes


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class MfaPeerScatter(ctypes.Structure):
    """Mirror of ``struct mfa_peer_scatter`` (include/mfa.h)."""

    _fields_ = [
        ("n_peers", ctypes.c_int32),
        ("rows_per_peer", ctypes.c_int32),
        ("slot", ctypes.c_int32),
        ("o_recv", ctypes.c_void_p * MAX_PEERS),
        ("lse_recv", ctypes.c_void_p * MAX_PEERS),
    ]


class MfaHostIo(ctypes.Structure):
    """Mirror of ``struct mfa_host_io`` (include/mfa.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("cu_q", ctypes.c_void_p),
        ("cu_k", ctypes.c_void_p),
        ("chunks", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()


class MfaError(RuntimeError):
    """A libmfa call returned a non-OK status."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = f"libmfa: {status_string(status)} (status {status})"
        if what:
            msg = f"{msg}: {what}"
        super().__init__(msg)


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libmfa.so (once) and declare the C signatures. Raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or os.environ.get("MTLFLASHATTN_LIB") or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"libmfa.so not found at {p}; build it with `python -m mtlflashattn_b200.build`"
            )
        lib = ctypes.CDLL(p)
        lib.mfa_fwd.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.mfa_fwd.restype = ctypes.c_int
        lib.mfa_fwd_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.mfa_fwd_noalloc.restype = ctypes.c_int
        lib.mfa_fwd_staged.argtypes = [ctypes.POINTER(MfaFwdParams), ctypes.POINTER(MfaHostIo),
                                        ctypes.c_void_p]
        lib.mfa_fwd_staged.restype = ctypes.c_int
        lib.mfa_fwd_workspace_size.argtypes = [ctypes.c_void_p]
        lib.mfa_fwd_workspace_size.restype = ctypes.c_size_t
        lib.mfa_fwd_num_splits.argtypes = [ctypes.c_void_p]
        lib.mfa_fwd_num_splits.restype = ctypes.c_int
        lib.mfa_fwd_packed_heads.argtypes = [ctypes.c_void_p]
        lib.mfa_fwd_packed_heads.restype = ctypes.c_int
        lib.mfa_select_kernel.argtypes = [ctypes.c_void_p]
        lib.mfa_select_kernel.restype = ctypes.c_int
        lib.mfa_lse_combine.argtypes = [
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
            ctypes.c_void_p, ctypes.c_void_p,
        ]
        lib.mfa_lse_combine.restype = ctypes.c_int
        lib.mfa_lse_rescale_sum.argtypes = [
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int32, ctypes.c_void_p,
        ]
        lib.mfa_lse_rescale_sum.restype = ctypes.c_int
        lib.mfa_fwd_scatter.argtypes = [ctypes.c_void_p, ctypes.POINTER(MfaPeerScatter),
                                        ctypes.c_void_p]
        lib.mfa_fwd_scatter.restype = ctypes.c_int
        lib.mfa_lse_merge.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                      ctypes.c_void_p]
        lib.mfa_lse_merge.restype = ctypes.c_int
        lib.mfa_lse_merge_rows.argtypes = [
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
            ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
        lib.mfa_lse_merge_rows.restype = ctypes.c_int
        lib.mfa_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.c_void_p]
        lib.mfa_peer_alloc.restype = ctypes.c_int
        lib.mfa_peer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.mfa_peer_open.restype = ctypes.c_int
        lib.mfa_peer_close.argtypes = [ctypes.c_void_p]
        lib.mfa_peer_close.restype = ctypes.c_int
        lib.mfa_peer_free.argtypes = [ctypes.c_void_p]
        lib.mfa_peer_free.restype = ctypes.c_int
        lib.mfa_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        lib.mfa_selftest_wait_timeout.restype = ctypes.c_int
        lib.mfa_status_string.argtypes = [ctypes.c_int]
        lib.mfa_status_string.restype = ctypes.c_char_p
        lib.mfa_abi_version.argtypes = []
        lib.mfa_abi_version.restype = ctypes.c_int
        if lib.mfa_abi_version() != MFA_ABI_VERSION:
            raise RuntimeError(
                f"libmfa ABI version {lib.mfa_abi_version()} != expected {MFA_ABI_VERSION}"
            )
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().mfa_status_string(status).decode()
    except Exception:  # the library itself may be what failed to load
        return f"status {status}"


def _addr(params) -> int:
    """Address of a params block: an MfaFwdParams or a packed buffer (see _kernel.pack)."""
    return ctypes.addressof(params)


def fwd(params, stream: int) -> int:
    return load().mfa_fwd(_addr(params), stream)


def fwd_noalloc(params, stream: int) -> int:
    return load().mfa_fwd_noalloc(_addr(params), stream)


def fwd_staged(params: MfaFwdParams, io: MfaHostIo, stream: int) -> int:
    return load().mfa_fwd_staged(ctypes.byref(params), ctypes.byref(io), ctypes.c_void_p(stream))


def workspace_size(params) -> int:
    return load().mfa_fwd_workspace_size(_addr(params))


def num_splits(params) -> int:
    return load().mfa_fwd_num_splits(_addr(params))


def packed_heads(params) -> int:
    return load().mfa_fwd_packed_heads(_addr(params))


def select_kernel(params) -> int:
    return load().mfa_select_kernel(_addr(params))


def lse_combine(o_ptrs, lse_ptrs, rows, H, D, o_ptr, o_dtype, lse_ptr, stream) -> int:
    n = len(o_ptrs)
    oa = (ctypes.c_void_p * n)(*o_ptrs)
    la = (ctypes.c_void_p * n)(*lse_ptrs)
    return load().mfa_lse_combine(oa, la, n, rows, H, D, ctypes.c_void_p(o_ptr), o_dtype,
                                  ctypes.c_void_p(lse_ptr or 0), ctypes.c_void_p(stream))


def lse_rescale_sum(o_ptrs, lse_ptrs, rows, H, D, lse_ref_ptr, o_ptr, o_dtype, stream) -> int:
    n = len(o_ptrs)
    oa = (ctypes.c_void_p * n)(*o_ptrs)
    la = (ctypes.c_void_p * n)(*lse_ptrs)
    return load().mfa_lse_rescale_sum(oa, la, n, rows, H, D, ctypes.c_void_p(lse_ref_ptr),
                                      ctypes.c_void_p(o_ptr), o_dtype, ctypes.c_void_p(stream))


def fwd_scatter(params, scatter: MfaPeerScatter, stream: int) -> int:
    return load().mfa_fwd_scatter(_addr(params), ctypes.byref(scatter), stream)


def lse_merge(o_parts_ptr, lse_parts_ptr, n, rows, H, D, o_ptr, o_dtype, lse_ptr, stream) -> int:
    return load().mfa_lse_merge(o_parts_ptr, lse_parts_ptr, n, rows, H, D, o_ptr, o_dtype,
                                lse_ptr or None, stream)


def peer_alloc(nbytes: int):
    """(device pointer, IPC handle bytes) of a new receive buffer on the current GPU."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    rc = load().mfa_peer_alloc(nbytes, ctypes.byref(ptr), handle)
    if rc != OK:
        raise MfaError(rc, "mfa_peer_alloc")
    return ptr.value, handle.raw


def peer_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    rc = load().mfa_peer_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr))
    if rc != OK:
        raise MfaError(rc, "mfa_peer_open")
    return ptr.value


def peer_close(ptr: int) -> int:
    return load().mfa_peer_close(ptr)


def peer_free(ptr: int) -> int:
    return load().mfa_peer_free(ptr)


def lse_merge_rows(o_ptrs, lse_ptrs, rows_total, row0, nrows, H, D, o_ptr, o_dtype, lse_ptr,
                   stream) -> int:
    n = len(o_ptrs)
    oa = (ctypes.c_void_p * n)(*o_ptrs)
    la = (ctypes.c_void_p * n)(*lse_ptrs)
    return load().mfa_lse_merge_rows(oa, la, n, rows_total, row0, nrows, H, D, o_ptr, o_dtype,
                                     lse_ptr or None, stream)
