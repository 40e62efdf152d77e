"""Key split within one launch for decode-like shapes (few query rows, many keys): the library
cuts each CTA's keys over several CTAs writing fp32 partials into a workspace and merges them
by log-sum-exp. Checked against the oracle with the reference's tolerances, for every feature
(causal, window, softcap, ALiBi, GQA, fp16/bf16, D 64/128), including the row log-sum-exp."""
import math

import pytest
import torch

import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import _kernel, _lib
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float16: dict(atol=1.5e-2, rtol=2e-2), torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}


def plan(q, k, v):
    """(workspace bytes, splits) the library chooses for flash_attn_func(q, k, v)."""
    B, Lq, Hq, D = q.shape
    o = torch.empty_like(q)
    p = _kernel._params(q, k, v, o, B=B, Hq=Hq, Hkv=k.shape[2], Lq=Lq, Lk=k.shape[1], D=D,
                        q_st=q.stride()[:3], k_st=k.stride()[:3], v_st=v.stride()[:3],
                        o_st=o.stride()[:3], scale=1.0, causal=False,
                        bias=_kernel._BiasParams(0.0, -1, -1, None), kernel=_lib.KERNEL_AUTO)
    need = _lib.workspace_size(p)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), need
    return need, _lib.num_splits(p)


CASES = [
    # B, Lq, Lk, Hq, Hkv, D, dtype, kwargs
    (1, 1, 4096, 8, 8, 128, torch.bfloat16, dict()),
    (2, 1, 33000, 8, 2, 128, torch.bfloat16, dict(causal=True)),
    (1, 7, 5000, 4, 1, 64, torch.float16, dict(causal=True)),
    (1, 64, 16384, 16, 4, 128, torch.bfloat16, dict(window_size=(3000, 0))),
    (1, 16, 8192, 4, 4, 64, torch.float16, dict(softcap=30.0)),
    (1, 33, 6000, 4, 4, 128, torch.bfloat16, dict(alibi_slopes=torch.tensor([0.01, 0.02, 0.05, 0.1]))),
    (3, 300, 9000, 2, 1, 64, torch.bfloat16, dict(causal=True, window_size=(700, 64))),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}h{c[3]}d{c[5]}" for c in CASES])
def test_split_matches_oracle(case):
    B, Lq, Lk, Hq, Hkv, D, dtype, kw = case
    q, k, v = ref.make_qkv(B, Lq, Lk, Hq, Hkv, D, dtype, seed=Lq + Lk)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    need, splits = plan(qd, kd, vd)
    assert need > 0 and splits > 1, (need, splits)
    kwd = {a: (b.to(DEV) if torch.is_tensor(b) else b) for a, b in kw.items()}
    out = mfa.flash_attn_func(qd, kd, vd, **kwd)
    want = ref.flash_attn_func(q, k, v, **kw)
    torch.testing.assert_close(out.float().cpu(), want, **TOL[dtype])


def test_split_writes_row_lse():
    q, k, v = ref.make_qkv(1, 5, 7000, 4, 2, 128, torch.bfloat16, seed=3)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o = torch.empty(1, 5, 4, 128, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(1, 4, 5, device=DEV, dtype=torch.float32)
    _kernel.forward_bshd(qd, kd, vd, o, 1 / math.sqrt(128), True,
                         _kernel._BiasParams(0.0, -1, -1, None), lse=lse)
    want, want_lse = ref.attention_heads_second(q.transpose(1, 2), k.transpose(1, 2),
                                                v.transpose(1, 2), 1 / math.sqrt(128), True,
                                                return_lse=True)
    torch.testing.assert_close(o.float().cpu(), want.transpose(1, 2), **TOL[torch.bfloat16])
    torch.testing.assert_close(lse.cpu(), want_lse, atol=1e-3, rtol=1e-4)


def test_no_split_when_grid_is_full():
    q, k, v = (torch.empty(1, 8192, 16, 128, device=DEV, dtype=torch.bfloat16) for _ in range(3))
    assert plan(q, k, v) == (0, 1)
