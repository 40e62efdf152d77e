"""mfa_fwd_noalloc, the entry point for callers that cannot allocate device memory during a
forward (an allocator that owns all device memory, a custom pool, a loop that must not take
the allocator's locks): it keeps the split-KV partials in the library's fixed 16 MiB device
array instead of a caller workspace. This file is collected last on purpose, so a run that stops
at its first failure has already run every other test.

Checked through the C ABI against the regular mfa_fwd (with a torch-allocated workspace) on
two consecutive calls, within the reference's bf16/fp16 tolerances, on shapes whose keys are
split (so the scratch is really used); and a problem too big for the scratch is refused."""
import math

import pytest
import torch

from mtlflashattn_b200 import _kernel, _lib
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float16: dict(atol=1.5e-2, rtol=2e-2), torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}


def params(q, k, v, o, causal, lse=None):
    B, Lq, Hq, D = q.shape
    return _kernel._params(q, k, v, o, B=B, Hq=Hq, Hkv=k.shape[2], Lq=Lq, Lk=k.shape[1], D=D,
                           q_st=q.stride()[:3], k_st=k.stride()[:3], v_st=v.stride()[:3],
                           o_st=o.stride()[:3], scale=1 / math.sqrt(D), causal=causal,
                           bias=_kernel._BiasParams(0.0, -1, -1, None), kernel=_lib.KERNEL_AUTO,
                           lse=lse, lse_st=((lse.stride(0), lse.stride(1)) if lse is not None else (0, 0)))


@pytest.mark.parametrize("shape,dtype,causal", [
    ((1, 1, 32768, 32, 8, 128), torch.bfloat16, False),
    ((2, 64, 9000, 4, 2, 64), torch.float16, True),
])
def test_noalloc_matches_regular_entry_twice(shape, dtype, causal):
    B, Lq, Lk, Hq, Hkv, D = shape
    q, k, v = (t.to(DEV) for t in ref.make_qkv(B, Lq, Lk, Hq, Hkv, D, dtype, seed=Lk))
    stream = torch.cuda.current_stream().cuda_stream

    # regular entry point, caller-owned workspace
    o_ref = torch.empty_like(q)
    p = params(q, k, v, o_ref, causal)
    need = _lib.workspace_size(p)
    assert 0 < need <= 16 << 20, need  # the keys are split and the scratch is big enough
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), need
    assert _lib.num_splits(p) > 1
    assert _lib.fwd(p, stream) == _lib.OK

    # no-allocation entry point, two calls in a row (the second reuses the shared scratch)
    for _ in range(2):
        o = torch.empty_like(q)
        p2 = params(q, k, v, o, causal)
        assert _lib.fwd_noalloc(p2, stream) == _lib.OK
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float(), o_ref.float(), **TOL[dtype])
    _kernel.check_device_errors(DEV)


def test_noalloc_refuses_problems_beyond_its_scratch():
    # 255 query rows x 16 heads over 65536 keys would need ~40 MB of split partials
    q = torch.zeros(1, 255, 16, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(1, 65536, 16, 128, device=DEV, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    p = params(q, k, k, o, False)
    assert _lib.workspace_size(p) > 16 << 20
    rc = _lib.fwd_noalloc(p, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_SCRATCH_TOO_SMALL
    assert "16 MiB" in _lib.status_string(rc)


def varlen_params(q, k, v, o, cu_q, cu_k, max_lq, max_lk):
    return _kernel._params(q, k, v, o, B=cu_q.shape[0] - 1, Hq=q.shape[1], Hkv=k.shape[1],
                           Lq=q.shape[0], Lk=k.shape[0], D=q.shape[2],
                           q_st=(0, q.stride(0), q.stride(1)), k_st=(0, k.stride(0), k.stride(1)),
                           v_st=(0, v.stride(0), v.stride(1)), o_st=(0, o.stride(0), o.stride(1)),
                           scale=1 / math.sqrt(q.shape[2]), causal=True,
                           bias=_kernel._BiasParams(0.0, -1, -1, None), kernel=_lib.KERNEL_AUTO,
                           cu_q=cu_q, cu_k=cu_k, max_lq=max_lq, max_lk=max_lk)


def test_noalloc_varlen_split_two_calls_with_different_sequences():
    """Batched decode through the varlen path: two no-allocation calls in a row with different
    cu_seqlens share the scratch; each must match mfa_fwd with its own workspace (stale partials
    of the first call must not leak into the second)."""
    stream = torch.cuda.current_stream().cuda_stream
    for seed, lq, lk in ((1, [1, 2, 1, 1], [9000, 15000, 300, 20000]),
                         (2, [3, 1, 1], [4000, 22000, 11000])):
        q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, 16, 4, 128, torch.bfloat16, seed=seed)
        qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
        o_ref = torch.empty_like(qd)
        p = varlen_params(qd, kd, vd, o_ref, cqd, ckd, max(lq), max(lk))
        need = _lib.workspace_size(p)
        assert 0 < need <= 16 << 20, need
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        p.workspace, p.workspace_bytes = ws.data_ptr(), need
        assert _lib.num_splits(p) > 1
        assert _lib.fwd(p, stream) == _lib.OK
        o = torch.empty_like(qd)
        assert _lib.fwd_noalloc(varlen_params(qd, kd, vd, o, cqd, ckd, max(lq), max(lk)),
                                stream) == _lib.OK
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float(), o_ref.float(), **TOL[torch.bfloat16])
    _kernel.check_device_errors(DEV)
