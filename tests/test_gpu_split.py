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


def varlen_plan(q, k, v, cu_q, cu_k, max_lq, max_lk):
    """(workspace bytes, splits) the library chooses for a varlen call."""
    o = torch.empty_like(q)
    p = _kernel._params(q, k, v, o, B=cu_q.shape[0] - 1, Hq=q.shape[1], Hkv=k.shape[1],
                        Lq=q.shape[0], Lk=k.shape[0], D=q.shape[2],
                        q_st=(0, q.stride(0), q.stride(1)), k_st=(0, k.stride(0), k.stride(1)),
                        v_st=(0, v.stride(0), v.stride(1)), o_st=(0, o.stride(0), o.stride(1)),
                        scale=1.0, causal=True, bias=_kernel._BiasParams(0.0, -1, -1, None),
                        kernel=_lib.KERNEL_AUTO, cu_q=cu_q, cu_k=cu_k, max_lq=max_lq,
                        max_lk=max_lk)
    need = _lib.workspace_size(p)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), need
    return need, _lib.num_splits(p)


VARLEN_CASES = [
    # lens_q, lens_k, Hq, Hkv, D, dtype, kwargs
    ([1] * 8, [8192, 300, 5000, 1, 8192, 2048, 7000, 4096], 32, 8, 128, torch.bfloat16,
     dict(causal=True)),
    ([1, 2, 0, 1], [30000, 0, 100, 12000], 16, 2, 128, torch.float16, dict(causal=True)),
    ([4, 1, 3], [20000, 20000, 9000], 8, 8, 64, torch.bfloat16,
     dict(causal=True, window_size=(4000, 0))),
    ([1, 1], [16000, 9000], 8, 2, 128, torch.bfloat16, dict(softcap=25.0)),
    ([2, 1, 1], [10000, 600, 15000], 8, 2, 128, torch.bfloat16, dict(alibi_slopes="per-seq")),
]


@pytest.mark.parametrize("case", VARLEN_CASES, ids=[f"v{i}" for i in range(len(VARLEN_CASES))])
def test_varlen_split_matches_oracle(case):
    lq, lk, Hq, Hkv, D, dtype, kw = case
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, Hq, Hkv, D, dtype, seed=sum(lk) % 1000)
    if kw.get("alibi_slopes") == "per-seq":
        kw = dict(kw, alibi_slopes=torch.rand(len(lq), Hq, generator=torch.Generator().manual_seed(1)) * 0.05)
    qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    need, splits = varlen_plan(qd, kd, vd, cqd, ckd, max(lq), max(lk))
    assert need > 0 and splits > 1, (need, splits)
    kwd = {a: (b.to(DEV) if torch.is_tensor(b) else b) for a, b in kw.items()}
    out = mfa.flash_attn_varlen_func(qd, kd, vd, cqd, ckd, max(lq), max(lk), **kwd)
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, **kw)
    torch.testing.assert_close(out.float().cpu(), want, **TOL[dtype])


def test_varlen_split_row_lse_and_understated_max_lk():
    """The row log-sum-exp of a split varlen launch, and a max_lk below the true longest key
    length (the last split takes every remaining key, so nothing is lost)."""
    lq, lk = [1, 3, 2], [9000, 20000, 4000]
    Hq, Hkv, D = 16, 4, 128
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, Hq, Hkv, D, torch.bfloat16, seed=21)
    qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    scale = 1 / math.sqrt(D)
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, causal=True)
    for max_lk in (max(lk), 12000):
        assert varlen_plan(qd, kd, vd, cqd, ckd, max(lq), max_lk)[1] > 1
        o = torch.empty_like(qd)
        lse = torch.empty(Hq, q.shape[0], device=DEV, dtype=torch.float32)
        _kernel.forward_varlen(qd, kd, vd, o, cqd, ckd, max(lq), max_lk, scale, True,
                               _kernel._BiasParams(0.0, -1, -1, None), lse=lse)
        torch.testing.assert_close(o.float().cpu(), want, **TOL[torch.bfloat16])
        for i in range(len(lq)):
            qs = slice(int(cu_q[i]), int(cu_q[i + 1]))
            ks = slice(int(cu_k[i]), int(cu_k[i + 1]))
            _, wl = ref.attention_heads_second(q[qs].permute(1, 0, 2)[None], k[ks].permute(1, 0, 2)[None],
                                               v[ks].permute(1, 0, 2)[None], scale, True,
                                               return_lse=True)
            torch.testing.assert_close(lse[:, qs].cpu(), wl[0], atol=1e-3, rtol=1e-4)


def _varlen_params(q, k, v, o, cu_q, cu_k, max_lq, max_lk, lse=None):
    return _kernel._params(q, k, v, o, B=cu_q.shape[0] - 1, Hq=q.shape[1], Hkv=k.shape[1],
                           Lq=q.shape[0], Lk=k.shape[0], D=q.shape[2],
                           q_st=(0, q.stride(0), q.stride(1)), k_st=(0, k.stride(0), k.stride(1)),
                           v_st=(0, v.stride(0), v.stride(1)), o_st=(0, o.stride(0), o.stride(1)),
                           scale=1 / math.sqrt(q.shape[2]), causal=True,
                           bias=_kernel._BiasParams(0.0, -1, -1, None), kernel=_lib.KERNEL_AUTO,
                           lse=lse, lse_st=((0, lse.stride(0)) if lse is not None else (0, 0)),
                           cu_q=cu_q, cu_k=cu_k, max_lq=max_lq, max_lk=max_lk)


def test_varlen_split_over_part_of_a_batch_leaves_other_rows_alone():
    """Two split launches, each over half of the sequences of one packed batch, into the same
    output through the same (dirty) workspace: each writes only its own packed rows, and
    together they give the whole batch's result."""
    lq, lk = [1, 2, 1, 3], [12000, 9000, 15000, 7000]
    Hq, Hkv, D = 16, 4, 128
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, Hq, Hkv, D, torch.bfloat16, seed=33)
    qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, causal=True)
    sentinel = 123.0
    o = torch.full_like(qd, sentinel)
    lse = torch.full((Hq, q.shape[0]), sentinel, device=DEV, dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.full((64 << 20,), 0x7F, dtype=torch.uint8, device=DEV)  # stale, non-zero bytes
    halves = [(0, 2), (2, 4)]
    for n, (s0, s1) in enumerate(halves):
        p = _varlen_params(qd, kd, vd, o, cqd[s0:s1 + 1], ckd[s0:s1 + 1], max(lq), max(lk), lse)
        need = _lib.workspace_size(p)
        assert 0 < need <= ws.numel()
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        assert _lib.num_splits(p) > 1
        assert _lib.fwd(p, stream) == _lib.OK
        torch.cuda.synchronize()
        r0, r1 = int(cu_q[s0]), int(cu_q[s1])
        # rows of sequences not yet run are untouched
        later = int(cu_q[halves[n][1]])
        assert torch.all(o[later:] == sentinel)
        assert torch.all(lse[:, later:] == sentinel)
        torch.testing.assert_close(o[r0:r1].float().cpu(), want[r0:r1], **TOL[torch.bfloat16])
    torch.testing.assert_close(o.float().cpu(), want, **TOL[torch.bfloat16])
    _kernel.check_device_errors(DEV)


def test_varlen_split_with_understated_lq_reports_instead_of_writing_past_workspace():
    """A C caller whose Lq (total_q) is below cu_q[B] gets MFA_ERR_INVALID in the error word;
    the rows past Lq are not stored into the workspace."""
    lq, lk = [1, 1, 2], [12000, 9000, 15000]
    Hq, Hkv, D = 8, 2, 128
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, Hq, Hkv, D, torch.bfloat16, seed=34)
    qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    o = torch.zeros_like(qd)
    p = _varlen_params(qd, kd, vd, o, cqd, ckd, max(lq), max(lk))
    p.Lq = q.shape[0] - 2  # understated total_q
    need = _lib.workspace_size(p)
    ws = torch.zeros(need + (1 << 20), dtype=torch.uint8, device=DEV)
    guard = ws[need:].clone()
    p.workspace, p.workspace_bytes = ws.data_ptr(), need
    assert _lib.num_splits(p) > 1
    assert _lib.fwd(p, torch.cuda.current_stream().cuda_stream) == _lib.OK
    with pytest.raises(_lib.MfaError) as ei:
        _kernel.check_device_errors(DEV)
    assert ei.value.status == _lib.ERR_INVALID
    assert torch.equal(ws[need:], guard)  # nothing written past the planned workspace


@pytest.mark.parametrize("lens,kw", [
    ([6040, 3336, 945, 4133, 1, 0, 7422, 257], dict(causal=True)),
    ([1, 2, 1, 3, 1], dict(causal=True)),  # decode-like: packed heads and a key split
    ([700, 1300, 90], dict(window_size=(200, 0), softcap=20.0)),
])
def test_varlen_exact_cta_list_matches_padded_grid(lens, kw):
    """The exact, longest-first CTA list (host cu_seqlens known) computes every row exactly as
    the padded grid with early-exit CTAs does: each CTA's rows, keys and order of work are the
    same, only the CTAs' order in the grid differs, so the outputs are bitwise equal."""
    lk = [max(n, 1) * 3 for n in lens]
    q, k, v, cu_q, cu_k = ref.make_varlen(lens, lk, 16, 4, 128, torch.bfloat16, seed=len(lens))
    qd, kd, vd, cqd, ckd = (t.to(DEV) for t in (q, k, v, cu_q, cu_k))
    bias = _kernel._BiasParams(kw.get("softcap", 0.0), *kw.get("window_size", (-1, -1)), None)
    outs = []
    for host in (None, cu_q.tolist()):
        o = torch.empty_like(qd)
        _kernel.forward_varlen(qd, kd, vd, o, cqd, ckd, max(lens), max(lk), 1 / math.sqrt(128),
                               kw.get("causal", False), bias, cu_q_host=host)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, **kw)
    torch.testing.assert_close(outs[1].float().cpu(), want, **TOL[torch.bfloat16])
