"""GPU tests of the surface around the kernel: the SDPA patch (routing, gates, bitwise stock
fallback, uneven-V shield; reference tests/test_sdpa_patch.py), the flash_attn shim serving this
engine, and the multi-GPU helpers run as a single NCCL rank (head shard = whole problem,
split-KV over zigzag chunks merged = unsplit)."""
import math
import os
import socket

import pytest
import torch
import torch.nn.functional as F

import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import _finder, sdpa
from mtlflashattn_b200 import distributed as mfd
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bhld(B, H, Lq, Lk, D, dtype=torch.float16, Hkv=None, seed=0, Dv=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, Lq, D, generator=g).to(DEV, dtype)
    k = torch.randn(B, Hkv or H, Lk, D, generator=g).to(DEV, dtype)
    v = torch.randn(B, Hkv or H, Lk, Dv or D, generator=g).to(DEV, dtype)
    return q, k, v


def ref_bhld(q, k, v, causal=False, scale=None):
    return ref.attention_heads_second(q.float().cpu(), k.float().cpu(), v.float().cpu(),
                                      scale if scale is not None else 1 / math.sqrt(q.shape[-1]),
                                      causal)


@pytest.fixture
def patched():
    assert sdpa.install(min_score_gb=1e-9)
    yield sdpa
    sdpa.uninstall()


def test_sdpa_routes_and_matches(patched):
    q, k, v = bhld(1, 4, 128, 128, 64)
    out = F.scaled_dot_product_attention(q, k, v)
    torch.testing.assert_close(out.float().cpu(), ref_bhld(q, k, v), atol=1.5e-2, rtol=2e-2)
    q, k, v = bhld(1, 2, 96, 96, 64, dtype=torch.float32)
    out = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=0.5)
    torch.testing.assert_close(out.cpu(), ref_bhld(q, k, v, True, 0.5), atol=2e-5, rtol=1e-4)


def test_sdpa_gqa_routes(patched):
    q, k, v = bhld(1, 8, 64, 64, 64, Hkv=2)
    out = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
    torch.testing.assert_close(out.float().cpu(), ref_bhld(q, k, v), atol=1.5e-2, rtol=2e-2)


def test_sdpa_stock_fallbacks_are_bitwise(patched):
    q, k, v = bhld(1, 2, 64, 64, 64)
    mask = torch.zeros(64, 64, device=DEV, dtype=torch.float16)
    mask[:, 32:] = float("-inf")
    assert torch.equal(F.scaled_dot_product_attention(q, k, v, attn_mask=mask),
                       patched._orig(q, k, v, attn_mask=mask))
    q, k, v = bhld(1, 2, 32, 96, 64)
    assert torch.equal(F.scaled_dot_product_attention(q, k, v, is_causal=True),
                       patched._orig(q, k, v, is_causal=True))


def test_sdpa_gates():
    assert sdpa.install()
    try:
        q, k, v = bhld(1, 2, 64, 64, 64)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert not ok and reason.startswith("fits")
        q, k, v = bhld(1, 4, 2048, 2048, 64)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert ok and reason == "fast-tier"
        q, k, v = bhld(1, 1, 4096, 4096, 100)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert ok and reason == "correctness-large-seq"
    finally:
        sdpa.uninstall()


def test_sdpa_uneven_v(patched):
    q, k, v = bhld(1, 4, 128, 128, 64, dtype=torch.float32, Dv=128)
    out = F.scaled_dot_product_attention(q, k, v)
    assert out.shape == (1, 4, 128, 128)
    want = torch.softmax(q.cpu() @ k.cpu().transpose(-1, -2) / 8.0, -1) @ v.cpu()
    torch.testing.assert_close(out.cpu(), want, atol=2e-5, rtol=1e-4)
    with pytest.raises(ValueError, match="enable_gqa"):
        q, k, v = bhld(1, 8, 32, 32, 64, dtype=torch.float32, Hkv=2, Dv=128)
        F.scaled_dot_product_attention(q, k, v)


def test_shim_serves_engine_functions():
    import importlib.util
    finder = _finder._MtlFlashAttnB200Finder()
    for name in ("flash_attn", "flash_attn.flash_attn_interface"):
        spec = finder.find_spec(name)
        assert spec is not None
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        assert mod.flash_attn_func is mfa.flash_attn_func
        assert mod.flash_attn_varlen_kvpacked_func is mfa.flash_attn_varlen_kvpacked_func
        if name == "flash_attn":
            assert mod.__version__ == "2.7.4"
    q, k, v = (torch.randn(1, 64, 4, 64, device=DEV, dtype=torch.float16) for _ in range(3))
    out = mod.flash_attn_func(q, k, v, causal=True)
    assert out.shape == q.shape and torch.isfinite(out).all()


@pytest.fixture(scope="module")
def nccl_single_rank():
    import torch.distributed as dist
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device(DEV, 0))
    yield
    dist.destroy_process_group()


def test_head_sharded_single_rank(nccl_single_rank):
    q, k, v = ref.make_qkv(1, 300, 300, 8, 2, 64, torch.bfloat16, seed=4)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out, (h0, h1) = mfd.flash_attn_head_sharded(qd, kd, vd, causal=True)
    assert (h0, h1) == (0, 8)
    torch.testing.assert_close(out, mfa.flash_attn_func(qd, kd, vd, causal=True), atol=0, rtol=0)


def test_split_kv_single_rank_equals_unsplit(nccl_single_rank):
    q, k, v = ref.make_qkv(1, 700, 1000, 4, 4, 128, torch.bfloat16, seed=12)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    ranges = [(0, 300), (300, 1000)]
    out = mfd.flash_attn_split_kv(qd, [kd[:, a:b] for a, b in ranges],
                                  [vd[:, a:b] for a, b in ranges], ranges, 1000, causal=True,
                                  softcap=20.0, alibi_slopes=torch.tensor([0.1] * 4, device=DEV))
    want = ref.flash_attn_func(q, k, v, causal=True, softcap=20.0,
                               alibi_slopes=torch.tensor([0.1] * 4))
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-2, rtol=2e-2)
