"""Query heads of a KV group packed into the rows of one tile (decode-like GQA/MQA shapes).

For fewer than 128 query rows per sequence and a power-of-two group of at most 16 query heads
per KV head, the tcgen05 kernel runs one CTA per (batch, KV head) whose tile row r is query
position r / group of query head hk * group + r % group, so every K/V block is loaded once per
group. Every feature reads per row (mask position, ALiBi slope, output and log-sum-exp address),
so each is checked against the oracle with the reference's tolerances, with and without the key
split, across row counts that leave the second tile of a CTA empty, partly full and full."""
import math

import pytest
import torch

import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import _kernel, _lib
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float16: dict(atol=1.5e-2, rtol=2e-2), torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}


def params(q, k, v, causal=False, window=(-1, -1), softcap=0.0):
    B, Lq, Hq, D = q.shape
    o = torch.empty_like(q)
    return _kernel._params(q, k, v, o, B=B, Hq=Hq, Hkv=k.shape[2], Lq=Lq, Lk=k.shape[1], D=D,
                           q_st=q.stride()[:3], k_st=k.stride()[:3], v_st=v.stride()[:3],
                           o_st=o.stride()[:3], scale=1.0 / math.sqrt(D), causal=causal,
                           bias=_kernel._BiasParams(softcap, window[0], window[1], None),
                           kernel=_lib.KERNEL_AUTO)


def slopes(h):
    return torch.tensor([2.0 ** (-8.0 * (i + 1) / h) for i in range(h)])


CASES = [
    # B, Lq, Lk, Hq, Hkv, D, dtype, kwargs
    (1, 1, 32768, 32, 8, 128, torch.bfloat16, dict()),
    (2, 1, 5000, 16, 2, 128, torch.bfloat16, dict(causal=True)),
    (1, 3, 4000, 32, 2, 64, torch.float16, dict(causal=True)),
    (1, 17, 3000, 8, 4, 128, torch.bfloat16, dict(causal=True, window_size=(100, 0))),
    (1, 33, 2000, 16, 4, 128, torch.bfloat16, dict(causal=True)),         # 132 rows: tile 1 has 4
    (1, 64, 9000, 16, 4, 64, torch.float16, dict(causal=True)),           # 256 rows
    (1, 127, 1000, 8, 1, 128, torch.bfloat16, dict(causal=True)),         # MQA, 1016 rows
    (1, 100, 3000, 16, 8, 128, torch.bfloat16, dict(causal=True)),        # group 2, 200 rows
    (1, 5, 6000, 8, 2, 128, torch.bfloat16, dict(causal=True, alibi_slopes=slopes(8))),
    (1, 20, 3000, 16, 4, 64, torch.bfloat16, dict(alibi_slopes=slopes(16))),  # two-sided ALiBi
    (2, 9, 2500, 8, 2, 128, torch.float16, dict(window_size=(700, 40), alibi_slopes=slopes(8))),
    (1, 2, 7000, 8, 2, 128, torch.float16, dict(softcap=30.0)),
    (1, 6, 5000, 16, 4, 64, torch.bfloat16, dict(softcap=20.0, causal=True)),
    (3, 1, 300, 8, 2, 128, torch.bfloat16, dict(causal=True)),            # too few keys to split
    (2, 4, 5, 8, 4, 64, torch.bfloat16, dict()),                          # tiny Lk
    (1, 40, 20, 8, 2, 64, torch.bfloat16, dict(causal=True)),             # Lq > Lk: zero rows
    (1, 8, 1000, 4, 2, 128, torch.float16, dict(softmax_scale=0.0)),      # uniform weights
]


def _id(c):
    return "-".join([f"{c[0]}x{c[1]}x{c[2]}h{c[3]}/{c[4]}d{c[5]}", *sorted(c[7])])


@pytest.mark.parametrize("case", CASES, ids=[_id(c) for c in CASES])
def test_packed_matches_oracle(case):
    B, Lq, Lk, Hq, Hkv, D, dtype, kw = case
    q, k, v = ref.make_qkv(B, Lq, Lk, Hq, Hkv, D, dtype, seed=Lq * 7 + Lk)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    p = params(qd, kd, vd, kw.get("causal", False), kw.get("window_size", (-1, -1)),
               kw.get("softcap", 0.0))
    assert _lib.packed_heads(p) == Hq // Hkv
    kwd = {a: (b.to(DEV) if torch.is_tensor(b) else b) for a, b in kw.items()}
    out = mfa.flash_attn_func(qd, kd, vd, **kwd)
    want = ref.flash_attn_func(q, k, v, **kw)
    torch.testing.assert_close(out.float().cpu(), want, **TOL[dtype])


@pytest.mark.parametrize("hq,hkv,lq", [(12, 4, 2), (64, 2, 1), (8, 2, 128), (8, 8, 1)])
def test_unpacked_groups_still_match(hq, hkv, lq):
    """Groups that are not packed (not a power of two, above 16, 128+ rows, no GQA)."""
    q, k, v = ref.make_qkv(1, lq, 3000, hq, hkv, 128, torch.bfloat16, seed=hq + lq)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    assert _lib.packed_heads(params(qd, kd, vd, True)) == 1
    out = mfa.flash_attn_func(qd, kd, vd, causal=True)
    torch.testing.assert_close(out.float().cpu(), ref.flash_attn_func(q, k, v, causal=True),
                               **TOL[torch.bfloat16])


def test_packed_strided_query_heads():
    """q a strided view (every other head of a wider tensor): the packed map walks head strides."""
    g = torch.Generator().manual_seed(5)
    wide = torch.randn(1, 3, 32, 128, generator=g).to(torch.bfloat16)
    q = wide[:, :, ::2]
    _, k, v = ref.make_qkv(1, 3, 4000, 16, 4, 128, torch.bfloat16, seed=6)
    qd = wide.to(DEV)[:, :, ::2]
    kd, vd = k.to(DEV), v.to(DEV)
    assert _lib.packed_heads(params(qd, kd, vd, True)) == 4
    out = mfa.flash_attn_func(qd, kd, vd, causal=True)
    torch.testing.assert_close(out.float().cpu(), ref.flash_attn_func(q, k, v, causal=True),
                               **TOL[torch.bfloat16])


def test_packed_row_lse():
    q, k, v = ref.make_qkv(2, 5, 3000, 16, 4, 128, torch.bfloat16, seed=11)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o = torch.empty(2, 5, 16, 128, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(2, 16, 5, device=DEV, dtype=torch.float32)
    _kernel.forward_bshd(qd, kd, vd, o, 1 / math.sqrt(128), True,
                         _kernel._BiasParams(0.0, -1, -1, None), lse=lse)
    want, want_lse = ref.attention_heads_second(q.transpose(1, 2), k.transpose(1, 2),
                                                v.transpose(1, 2), 1 / math.sqrt(128), True,
                                                return_lse=True)
    torch.testing.assert_close(o.float().cpu(), want.transpose(1, 2), **TOL[torch.bfloat16])
    torch.testing.assert_close(lse.cpu(), want_lse, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("alibi", [False, True])
def test_packed_varlen_decode(alibi):
    """Batched decode through varlen: one to a few new tokens per sequence, ragged key
    lengths, an empty query sequence, GQA group 8."""
    lq = [1, 3, 0, 1, 2, 1]
    lk = [700, 4100, 50, 1, 9000, 129]
    Hq, Hkv = 32, 4
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, Hq, Hkv, 128, torch.bfloat16, seed=9)
    kw = dict(causal=True)
    if alibi:
        kw["alibi_slopes"] = torch.rand(len(lq), Hq, generator=torch.Generator().manual_seed(2)) * 0.2
    out = mfa.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu_q.to(DEV), cu_k.to(DEV),
                                     max(lq), max(lk),
                                     **{a: (b.to(DEV) if torch.is_tensor(b) else b) for a, b in kw.items()})
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, **kw)
    torch.testing.assert_close(out.float().cpu(), want, **TOL[torch.bfloat16])


SHORT_CASES = [
    # one-tile CTAs without packing: at most 128 query rows, no GQA group to pack
    (1, 1, 8192, 16, 16, 128, torch.bfloat16, dict(causal=True)),
    (2, 50, 3000, 4, 4, 128, torch.float16, dict(softcap=30.0)),
    (1, 77, 2000, 8, 8, 128, torch.bfloat16, dict(causal=True, alibi_slopes=slopes(8))),
    (1, 128, 4096, 4, 4, 128, torch.bfloat16, dict(causal=True)),         # exactly one tile
    (1, 96, 1500, 6, 2, 128, torch.bfloat16, dict(window_size=(300, 300))),  # group 3
    (1, 3, 9000, 4, 4, 64, torch.float16, dict(softcap=15.0, causal=True)),
    (1, 64, 2000, 32, 16, 128, torch.bfloat16, dict(causal=True)),        # packed to 128 rows
]


@pytest.mark.parametrize("case", SHORT_CASES, ids=[_id(c) for c in SHORT_CASES])
def test_one_tile_ctas_match_oracle(case):
    B, Lq, Lk, Hq, Hkv, D, dtype, kw = case
    q, k, v = ref.make_qkv(B, Lq, Lk, Hq, Hkv, D, dtype, seed=Lq * 3 + Lk)
    kwd = {a: (b.to(DEV) if torch.is_tensor(b) else b) for a, b in kw.items()}
    out = mfa.flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), **kwd)
    torch.testing.assert_close(out.float().cpu(), ref.flash_attn_func(q, k, v, **kw), **TOL[dtype])


def test_one_tile_varlen_mixed_lengths():
    """Varlen with max_seqlen_q <= 128: every sequence runs in one-tile CTAs, GQA group 3."""
    lq = [128, 1, 0, 77, 5]
    lk = [128, 3000, 10, 900, 4000]
    q, k, v, cu_q, cu_k = ref.make_varlen(lq, lk, 12, 4, 128, torch.float16, seed=4)
    out = mfa.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu_q.to(DEV), cu_k.to(DEV),
                                     max(lq), max(lk), causal=True)
    torch.testing.assert_close(out.float().cpu(), ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k,
                                                                             causal=True),
                               **TOL[torch.float16])
