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


def test_sdpa_gates(monkeypatch):
    assert sdpa.install()
    try:
        q, k, v = bhld(1, 2, 64, 64, 64)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert not ok and reason.startswith("fits")
        # default: no speed routing unless calibrate() found a crossover on this platform
        q, k, v = bhld(1, 4, 2048, 2048, 64)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert ok == (sdpa.DEFAULT_FAST_MIN_SEQ is not None and 2048 >= sdpa.DEFAULT_FAST_MIN_SEQ)
        # stock SDPA is exact on CUDA and faster than the CUDA-core kernel: a long call the
        # tensor-core kernel cannot take stays on stock unless the all-tier floor is set
        q, k, v = bhld(1, 1, 4096, 4096, 100)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert not ok and reason.startswith("fits")
    finally:
        sdpa.uninstall()
    monkeypatch.setenv("MTLFLASHATTN_SDPA_MIN_SEQ", "256")
    assert sdpa.install()
    try:
        q, k, v = bhld(1, 1, 512, 512, 100)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert ok and reason == "correctness-large-seq"
    finally:
        sdpa.uninstall()
    monkeypatch.delenv("MTLFLASHATTN_SDPA_MIN_SEQ")
    monkeypatch.setenv("MTLFLASHATTN_SDPA_FAST_MIN_SEQ", "256")
    assert sdpa.install()
    try:
        q, k, v = bhld(1, 2, 512, 512, 64)
        ok, reason = sdpa._eligibility(q, k, v, None, 0.0, False)
        assert ok and reason == "fast-tier"
    finally:
        sdpa.uninstall()


def test_sdpa_uneven_v(patched):
    # fp32: routed by the memory gate (installed with a tiny budget), padded to D = 128
    q, k, v = bhld(1, 4, 128, 128, 64, dtype=torch.float32, Dv=128)
    out = F.scaled_dot_product_attention(q, k, v)
    assert out.shape == (1, 4, 128, 128)
    want = torch.softmax(q.cpu() @ k.cpu().transpose(-1, -2) / 8.0, -1) @ v.cpu()
    torch.testing.assert_close(out.cpu(), want, atol=2e-5, rtol=1e-4)
    # bf16, value narrower than query/key, causal: the tensor-core kernel on padded inputs
    q, k, v = bhld(1, 4, 300, 300, 128, dtype=torch.bfloat16, Dv=48)
    out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert out.shape == (1, 4, 300, 48)
    qf, kf, vf = q.float().cpu(), k.float().cpu(), v.float().cpu()
    s_ = (qf @ kf.transpose(-1, -2)) / math.sqrt(128)
    s_ = s_.masked_fill(torch.ones(300, 300, dtype=torch.bool).triu(1), float("-inf"))
    want = torch.softmax(s_, -1) @ vf
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-2, rtol=2e-2)
    # GQA without enable_gqa is not routed: stock SDPA decides (and refuses it)
    q, k, v = bhld(1, 8, 32, 32, 64, dtype=torch.float32, Hkv=2, Dv=128)
    ok, reason = sdpa._decide(q, k, v, None, 0.0, False, enable_gqa=False)
    assert not ok and reason.startswith("heads")
    with pytest.raises(Exception):
        F.scaled_dot_product_attention(q, k, v)


def test_sdpa_calibrate_runs():
    rows, floor = sdpa.calibrate(lengths=(256, 1024), dims=(64,), causal=(True,), iters=2)
    assert len(rows) == 2 and all(r["engine_ms"] > 0 and r["stock_ms"] > 0 for r in rows)
    assert floor in (None, 256, 1024)


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
    out, rows = mfd.flash_attn_split_kv(qd, [kd[:, a:b] for a, b in ranges],
                                        [vd[:, a:b] for a, b in ranges], ranges, 1000,
                                        causal=True, softcap=20.0,
                                        alibi_slopes=torch.tensor([0.1] * 4, device=DEV))
    assert rows == (0, 700)
    want = ref.flash_attn_func(q, k, v, causal=True, softcap=20.0,
                               alibi_slopes=torch.tensor([0.1] * 4))
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-2, rtol=2e-2)


def test_lse_rescale_sum_kernel_matches_torch():
    """mfa_lse_rescale_sum (the per-GPU half of the multi-GPU merge) against its statement in
    torch, including -inf rows, an unaligned output (scalar path) and a bf16 output."""
    from mtlflashattn_b200 import _lib
    g = torch.Generator(device=DEV).manual_seed(5)
    rows, H, D, n = 300, 6, 128, 3
    o = [torch.randn(rows, H, D, device=DEV, generator=g) for _ in range(n)]
    lse = [torch.randn(H, rows, device=DEV, generator=g) * 3 for _ in range(n)]
    lse[1][2, :50] = float("-inf")
    ref_lse = torch.logsumexp(torch.stack(lse), 0) + 0.25  # another GPU's share: +log(1.28)
    ref_lse[0, :7] = float("-inf")
    want = torch.zeros(rows, H, D, device=DEV)
    for og, lg in zip(o, lse):
        w = torch.exp(lg - ref_lse).nan_to_num(0.0)
        w[torch.isinf(lg) | torch.isinf(ref_lse)] = 0
        want += w.t()[..., None] * og
    st = torch.cuda.current_stream().cuda_stream
    for dt, code, off in ((torch.float32, _lib.FP32, 0), (torch.float32, _lib.FP32, 1),
                          (torch.bfloat16, _lib.BF16, 0)):
        buf = torch.empty(rows * H * D + off, device=DEV, dtype=dt)
        out = buf[off:].view(rows, H, D)
        rc = _lib.lse_rescale_sum([t.data_ptr() for t in o], [t.data_ptr() for t in lse], rows,
                                  H, D, ref_lse.data_ptr(), out.data_ptr(), code, st)
        assert rc == _lib.OK
        torch.testing.assert_close(out.float(), want, atol=1e-5 if dt == torch.float32 else 2e-2,
                                   rtol=1e-5 if dt == torch.float32 else 1e-2)


@pytest.mark.parametrize("ranges", [[(0, 300), (300, 1000)], [(0, 1000)]])
def test_split_kv_peer_merge_single_rank(nccl_single_rank, ranges):
    """The peer-memory merges on one rank: "peer" scatters partial rows from the forward into
    the (local) receive buffer, one slot per key chunk, and mfa_lse_merge combines the slots;
    "pull" writes the partials to the rank's own buffer and mfa_lse_merge_rows merges its rows
    through the peer pointers; checked against the oracle and against the NCCL merge."""
    q, k, v = ref.make_qkv(1, 700, 1000, 4, 2, 128, torch.bfloat16, seed=13)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kp, vp = [kd[:, a:b] for a, b in ranges], [vd[:, a:b] for a, b in ranges]
    want = ref.flash_attn_func(q, k, v, causal=True, window_size=(500, -1))
    outs = {}
    for merge in ("pull", "peer", "nccl"):
        for _ in range(2):  # the second call reuses the receive buffers
            out, rows = mfd.flash_attn_split_kv(qd, kp, vp, ranges, 1000, causal=True,
                                                window_size=(500, -1), merge=merge)
        assert rows == (0, 700)
        torch.testing.assert_close(out.float().cpu(), want, atol=2e-2, rtol=2e-2)
        outs[merge] = out.float()
    torch.testing.assert_close(outs["peer"], outs["nccl"], atol=8e-3, rtol=1e-2)
    torch.testing.assert_close(outs["pull"], outs["peer"], atol=8e-3, rtol=1e-2)


def test_lse_merge_kernel_matches_torch():
    from mtlflashattn_b200 import _lib
    g = torch.Generator(device=DEV).manual_seed(6)
    n, rows, H, D = 5, 77, 6, 64
    o = torch.randn(n, rows, H, D, device=DEV, generator=g)
    lse = torch.randn(n, H, rows, device=DEV, generator=g) * 4
    lse[1, :, :10] = float("-inf")
    lse[:, 3, 5] = float("-inf")  # a row no partial attends
    tot = torch.logsumexp(lse, 0)
    w = torch.exp(lse - tot).nan_to_num(0.0)
    want = (w.permute(0, 2, 1)[..., None] * o).sum(0)
    for dt, code in ((torch.float32, _lib.FP32), (torch.bfloat16, _lib.BF16)):
        out = torch.empty(rows, H, D, device=DEV, dtype=dt)
        lo = torch.empty(H, rows, device=DEV)
        rc = _lib.lse_merge(o.data_ptr(), lse.data_ptr(), n, rows, H, D, out.data_ptr(), code,
                            lo.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.OK
        torch.testing.assert_close(out.float(), want, atol=1e-5 if dt == torch.float32 else 2e-2,
                                   rtol=1e-5 if dt == torch.float32 else 1e-2)
        fin = torch.isfinite(tot)
        torch.testing.assert_close(lo[fin], tot[fin])
        assert torch.isinf(lo[3, 5]) and out[5, 3].abs().max() == 0


def test_trace_disabled_records_nothing(monkeypatch):
    from mtlflashattn_b200 import _kernel
    monkeypatch.delenv("MTLFLASHATTN_TRACE", raising=False)
    _kernel._trace.clear()
    q = torch.randn(1, 2, 64, 64, device=DEV, dtype=torch.float16)
    _kernel.flash_attn_forward(q, q, q, scale=0.125, causal=False)
    assert not _kernel._trace


def test_trace_records_shape_and_kernel_label(monkeypatch):
    """Same accounting as the reference's trace (tests/test_trace.py there): one key per
    (dtype, D, Lq, Lk, causal, kernel), counts accumulate, labels name the kernel that ran."""
    from mtlflashattn_b200 import _kernel
    monkeypatch.setenv("MTLFLASHATTN_TRACE", "1")
    _kernel._trace.clear()
    q = torch.randn(1, 4, 128, 64, device=DEV, dtype=torch.float16)
    _kernel.flash_attn_forward(q, q, q, scale=0.125, causal=False)
    _kernel.flash_attn_forward(q, q, q, scale=0.125, causal=False)
    qf = torch.randn(1, 2, 96, 32, device=DEV, dtype=torch.float32)
    _kernel.flash_attn_forward(qf, qf, qf, scale=0.2, causal=True)
    assert _kernel._trace[("float16", 64, 128, 128, False, "cuda/tcgen05")] == 2
    assert _kernel._trace[("float32", 32, 96, 96, True, "cuda/simt")] == 1
    lines = _kernel._trace_summary_lines()
    assert lines[0].startswith("[MTLFLASHATTN_TRACE] 3 attention call(s), 2 distinct")
    _kernel._trace.clear()


def test_trace_summary_printed_at_exit():
    import subprocess
    import sys
    root = os.path.dirname(HERE) if "HERE" in globals() else os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))
    code = ("import torch, mtlflashattn_b200 as m\n"
            "q = torch.randn(1, 256, 4, 64, device='cuda', dtype=torch.bfloat16)\n"
            "m.flash_attn_func(q, q, q, causal=True); torch.cuda.synchronize()\n")
    env = dict(os.environ, MTLFLASHATTN_TRACE="1",
               PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "[MTLFLASHATTN_TRACE] 1 attention call(s)" in r.stderr
    assert "-> cuda/tcgen05" in r.stderr
