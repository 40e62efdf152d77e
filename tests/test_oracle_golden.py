"""The oracle (oracle/flash_torch.py) reproduces the reference's own outputs, stored in
tests/golden/golden.pt by tests/golden/make_golden.py, on every golden case."""
import pytest
import torch

from golden.cases import load_cases
from oracle import flash_torch as ref

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(case):
    kw = dict(softmax_scale=case["scale"], causal=case["causal"], window_size=case["window"],
              softcap=case["softcap"], alibi_slopes=case["alibi"])
    if case["kind"] == "dense":
        got = ref.flash_attn_func(case["q"], case["k"], case["v"], chunk=case.get("chunk"), **kw)
    else:
        got = ref.flash_attn_varlen_func(case["q"], case["k"], case["v"], case["cu_q"],
                                         case["cu_k"], **kw)
    want = case["out_f32"] if case["out_f32"] is not None else case["out"]
    # same algorithm, same torch CPU kernels: agreement to fp32 rounding
    torch.testing.assert_close(got, want.float(), atol=2e-6, rtol=1e-5)
    # the reference's q.dtype output is its fp32 result cast once
    assert torch.equal(want.float().to(case["dtype"]), case["out"])


def test_golden_covers_reference_test_shapes():
    names = {c["name"] for c in CASES}
    for needed in ("lq_gt_lk_causal_f32", "tiny_3_5_f16", "tiny_lk5_bf16", "chunk13_gqa_f32",
                   "window_wide_f32", "alibi_batched_f32", "varlen_ragged_f32",
                   "unaligned_causal_bfloat16", "headdim33_bf16"):
        assert needed in names


def test_lse_matches_logsumexp_definition():
    q, k, v = ref.make_qkv(1, 33, 47, 2, 1, 16, torch.float32, seed=4)
    o, lse = ref.attention_heads_second(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                        0.3, True, return_lse=True)
    s = (q.transpose(1, 2) @ k.transpose(1, 2).repeat_interleave(2, 1).transpose(-1, -2)) * 0.3
    i = torch.arange(33)[:, None] + (47 - 33)
    j = torch.arange(47)[None, :]
    s = s.masked_fill(j > i, float("-inf"))
    torch.testing.assert_close(lse, torch.logsumexp(s, -1))


def test_split_keys_merge_equals_full():
    """Splitting the keys into chunks and merging by log-sum-exp reproduces the full result:
    the identity the multi-GPU split-KV path relies on."""
    q, k, v = ref.make_qkv(1, 40, 97, 2, 2, 16, torch.float32, seed=9)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    full = ref.attention_heads_second(qh, kh, vh, 0.25, True, softcap=5.0, window_left=30,
                                      alibi=torch.tensor([0.1, 0.2]))
    parts = []
    for a, b in ((0, 30), (30, 64), (64, 97)):
        parts.append(ref.attention_heads_second(qh, kh[:, :, a:b], vh[:, :, a:b], 0.25, True,
                                                softcap=5.0, window_left=30,
                                                alibi=torch.tensor([0.1, 0.2]), return_lse=True,
                                                key_offset=a, lk_total=97))
    lses = torch.stack([p[1] for p in parts])
    tot = torch.logsumexp(lses, 0)
    w = torch.nan_to_num(torch.exp(lses - tot), nan=0.0)
    merged = sum(w[g][..., None] * parts[g][0] for g in range(3))
    torch.testing.assert_close(merged, full, atol=1e-6, rtol=1e-5)
