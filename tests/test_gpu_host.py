"""Host-staged forward (flash_attn_host / flash_attn_varlen_host through mfa_fwd_staged):
pieces of query rows or of whole sequences, copies overlapped with the compute. Each result
must match the oracle like the device path does, for causal / windowed / softcap / ALiBi
inputs, Lq != Lk (rows with no key), every chunk count, fp32 (CUDA-core kernel) and varlen
with empty sequences."""
import pytest
import torch

import mtlflashattn_b200 as mfa
from oracle import flash_torch as ref

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(atol=2e-5, rtol=1e-4), torch.float16: dict(atol=1.5e-2, rtol=2e-2),
       torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}


def _close(out, want, dtype, what):
    assert out.device.type == "cpu" and out.dtype == dtype
    torch.testing.assert_close(out.float(), want.float(), **TOL[dtype], msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("case", [
    # B, Lq, Lk, Hq, Hkv, D, dtype, causal, kwargs, chunks
    (1, 1000, 1000, 4, 2, 64, torch.bfloat16, True, {}, 0),
    (2, 777, 777, 2, 2, 128, torch.float16, True, {}, 3),
    (1, 1024, 1024, 4, 4, 128, torch.float16, False,
     dict(softcap=30.0, window_size=(100, 50)), 4),
    (1, 900, 900, 4, 1, 64, torch.bfloat16, True, dict(alibi_slopes=torch.tensor([.1, .2, .3, .4])), 5),
    (1, 300, 1000, 2, 2, 64, torch.bfloat16, True, {}, 2),
    (1, 1000, 300, 2, 2, 64, torch.bfloat16, True, {}, 4),   # first 700 rows see no key
    (1, 1000, 300, 2, 2, 64, torch.bfloat16, False, dict(window_size=(20, 30)), 4),
    (1, 600, 600, 2, 2, 40, torch.float32, True, {}, 2),    # CUDA-core kernel
    (1, 512, 512, 2, 2, 64, torch.bfloat16, False, {}, 1),
    (1, 2048, 2048, 2, 2, 64, torch.bfloat16, True, {}, 64),
])
def test_host_dense_matches_oracle(case):
    B, Lq, Lk, Hq, Hkv, D, dtype, causal, kw, chunks = case
    q, k, v = ref.make_qkv(B, Lq, Lk, Hq, Hkv, D, dtype, seed=Lq + Lk + D)
    want = ref.flash_attn_func(q, k, v, causal=causal, **kw)
    qp, kp, vp = q.pin_memory(), k.pin_memory(), v.pin_memory()
    out = mfa.flash_attn_host(qp, kp, vp, causal=causal, chunks=chunks, **kw)
    _close(out, want, dtype, f"{case}")
    dev = mfa.flash_attn_func(q.cuda(), k.cuda(), v.cuda(), causal=causal,
                              **{a: (b.cuda() if torch.is_tensor(b) else b) for a, b in kw.items()})
    torch.testing.assert_close(out.float(), dev.float().cpu(), **TOL[dtype])


def test_host_out_buffer_and_async_two_calls():
    q, k, v = ref.make_qkv(1, 1500, 1500, 4, 2, 128, torch.bfloat16, seed=11)
    qp, kp, vp = q.pin_memory(), k.pin_memory(), v.pin_memory()
    out = torch.empty(1, 1500, 4, 128, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):  # the second call reuses the staging and host buffers
        r = mfa.flash_attn_host(qp, kp, vp, causal=True, out=out, synchronize=False)
        assert r is out
    torch.cuda.current_stream().synchronize()
    _close(out, ref.flash_attn_func(q, k, v, causal=True), torch.bfloat16, "async")


def test_host_varlen_matches_oracle():
    seqs = [300, 0, 1, 700, 129, 1000]
    q, k, v, cu_q, cu_k = ref.make_varlen(seqs, seqs, 4, 2, 64, torch.bfloat16, seed=4)
    slopes = torch.tensor([0.05, 0.1, 0.2, 0.4])
    want = ref.flash_attn_varlen_func(q, k, v, cu_q, cu_k, causal=True, alibi_slopes=slopes)
    for chunks in (0, 1, 3):
        out = mfa.flash_attn_varlen_host(q.pin_memory(), k.pin_memory(), v.pin_memory(), cu_q,
                                         cu_k, max(seqs), max(seqs), causal=True,
                                         alibi_slopes=slopes, chunks=chunks)
        _close(out, want, torch.bfloat16, f"varlen chunks={chunks}")


def test_host_rejects_device_tensors():
    q = torch.zeros(1, 8, 2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        mfa.flash_attn_host(q, q, q)
