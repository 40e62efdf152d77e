"""Failure detection on the GPU without a GPU fault: a bounded in-kernel wait that can never be
satisfied gives up after its limit and reports MFA_ERR_TIMEOUT to the host, and the context
stays usable (a forward right after it is correct). Host-side fault injection (MFA_FAULT) on a
real device leaves outputs untouched and raises the mapped exception."""
import time

import pytest
import torch

import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import _lib
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_bounded_wait_times_out_and_context_survives():
    err = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    t0 = time.perf_counter()
    rc = _lib.load().mfa_selftest_wait_timeout(err.data_ptr(), 200000,
                                               torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert int(err.item()) == _lib.ERR_TIMEOUT
    assert time.perf_counter() - t0 < 30
    q, k, v = ref.make_qkv(1, 200, 300, 2, 2, 64, torch.bfloat16, seed=9)
    out = mfa.flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), causal=True)
    torch.testing.assert_close(out.float().cpu(), ref.flash_attn_func(q, k, v, causal=True),
                               atol=2e-2, rtol=2e-2)


def test_injected_fault_raises_and_launches_nothing(monkeypatch):
    q, k, v = (torch.randn(1, 64, 2, 64, device=DEV, dtype=torch.float16) for _ in range(3))
    monkeypatch.setenv("MFA_FAULT", "fwd")
    with pytest.raises(_lib.MfaError, match="fault injected"):
        mfa.flash_attn_func(q, k, v)
