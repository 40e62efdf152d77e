"""The C ABI (include/mfa.h) as seen from Python, without a GPU: the library loads, exports every
declared symbol, the ctypes mirror of mfa_fwd_params matches the C layout, and the host-side
checks and fault injection answer before any CUDA call is made."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from mtlflashattn_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mfa.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(mfa_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTED_SYMBOLS), names
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.mfa_abi_version() == _lib.MFA_ABI_VERSION
    for s in range(8):
        assert _lib.status_string(s)
    assert _lib.status_string(0) == "ok"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("cls,cname", [(_lib.MfaFwdParams, "mfa_fwd_params"),
                                       (_lib.MfaPeerScatter, "mfa_peer_scatter"),
                                       (_lib.MfaHostIo, "mfa_host_io")])
def test_ctypes_struct_matches_c_layout(tmp_path, cls, cname):
    fields = [f[0] for f in cls._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
           f'printf("%zu\\n", sizeof({cname}));']
    src += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    src += ["return 0;}"]
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(c), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got[0] == ctypes.sizeof(cls)
    for name, off in zip(fields, got[1:]):
        assert getattr(cls, name).offset == off, name


def test_packed_params_format_matches_struct():
    """The hot path's struct.pack format has the C struct's size and workspace offset."""
    import struct
    assert struct.calcsize(_lib.PARAMS_FORMAT) == ctypes.sizeof(_lib.MfaFwdParams)
    assert _lib.MfaFwdParams.workspace.offset == _lib.WORKSPACE_OFFSET


def test_invalid_params_rejected_on_host():
    p = _lib.MfaFwdParams()
    p.B, p.Hq, p.Hkv, p.Lq, p.Lk, p.D = 1, 4, 3, 8, 8, 64  # Hkv does not divide Hq
    assert _lib.fwd(p, 0) == _lib.ERR_INVALID
    p.Hkv, p.D = 4, 160
    assert _lib.fwd(p, 0) == _lib.ERR_UNSUPPORTED
    p.D, p.softcap = 64, -1.0
    assert _lib.fwd(p, 0) == _lib.ERR_INVALID
    p.softcap, p.win_left = 0.0, -2
    assert _lib.fwd(p, 0) == _lib.ERR_INVALID
    p.win_left = -1
    assert _lib.fwd(p, 0) == _lib.ERR_INVALID  # null pointers with a non-empty problem
    p.Lq = 0
    assert _lib.fwd(p, 0) == _lib.OK  # empty problem: nothing to launch


def test_fault_injection_fires_before_launch(monkeypatch):
    monkeypatch.setenv("MFA_FAULT", "combine,fwd")
    p = _lib.MfaFwdParams()
    assert _lib.fwd(p, 0) == _lib.ERR_FAULT_INJECTED
    assert _lib.lse_combine([0], [0], 1, 1, 1, 0, 0, 0, 0) == _lib.ERR_FAULT_INJECTED
    monkeypatch.setenv("MFA_FAULT", "other")
    assert _lib.fwd(p, 0) != _lib.ERR_FAULT_INJECTED


def test_combine_argument_checks():
    assert _lib.lse_combine([0] * 65, [0] * 65, 1, 1, 1, 0, 0, 0, 0) == _lib.ERR_INVALID
    assert _lib.lse_combine([0], [0], 0, 1, 1, 0, 0, 0, 0) == _lib.OK


def test_wait_selftest_argument_checks():
    lib = _lib.load()
    assert lib.mfa_selftest_wait_timeout(None, 1000, None) == _lib.ERR_INVALID
    assert lib.mfa_selftest_wait_timeout(None, 0, None) == _lib.ERR_INVALID


def test_staged_entry_checks_before_any_cuda_call(monkeypatch):
    lib = _lib.load()
    p = _lib.MfaFwdParams()
    io = _lib.MfaHostIo()
    assert lib.mfa_fwd_staged(ctypes.byref(p), None, None) == _lib.ERR_INVALID
    p.D, p.Hq, p.Hkv, p.dtype, p.o_dtype = 160, 1, 1, _lib.BF16, -1
    assert lib.mfa_fwd_staged(ctypes.byref(p), ctypes.byref(io), None) == _lib.ERR_UNSUPPORTED
    monkeypatch.setenv("MFA_FAULT", "fwd")
    assert lib.mfa_fwd_staged(ctypes.byref(p), ctypes.byref(io), None) == _lib.ERR_FAULT_INJECTED
