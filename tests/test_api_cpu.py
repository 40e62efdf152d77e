"""The Python surface without a GPU: argument checks in the reference's order and exception
types (metal_flash_attn/__init__.py:28-59), packed-wrapper shape checks, SDPA gating and
install/uninstall, the guarded flash_attn import shim, and the call trace."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch
import torch.nn.functional as F

import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import _kernel, sdpa

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def qkv(D=64, dtype=torch.float16):
    t = torch.zeros(1, 8, 2, D, dtype=dtype)
    return t, t.clone(), t.clone()


@pytest.mark.parametrize("kwargs,exc", [
    (dict(dropout_p=0.1), NotImplementedError),
    (dict(window_size=(-2, 0)), ValueError),
    (dict(window_size=(1, 2, 3)), ValueError),
    (dict(window_size=(True, 0)), ValueError),
    (dict(softcap=-1.0), ValueError),
    (dict(alibi_slopes=[0.5, 0.25]), TypeError),
    (dict(deterministic=True), NotImplementedError),
    (dict(return_attn_probs=True), NotImplementedError),
    (dict(), NotImplementedError),  # CPU tensors: device check (CUDA only)
])
def test_check_order_and_types(kwargs, exc):
    q, k, v = qkv()
    with pytest.raises(exc):
        mfa.flash_attn_func(q, k, v, **kwargs)


def test_dropout_checked_before_device_and_window():
    q, k, v = qkv()
    with pytest.raises(NotImplementedError, match="dropout"):
        mfa.flash_attn_func(q, k, v, dropout_p=0.5, window_size=(-5, 0))


def test_varlen_block_table_and_shape_errors():
    q = torch.zeros(8, 2, 64, dtype=torch.float16)
    cu = torch.tensor([0, 8], dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        mfa.flash_attn_varlen_func(q, q, q, cu, cu, 8, 8, dropout_p=0.3)


def test_packed_shape_validation():
    with pytest.raises(ValueError):
        mfa.flash_attn_qkvpacked_func(torch.zeros(1, 4, 2, 2, 64))
    with pytest.raises(ValueError):
        mfa.flash_attn_kvpacked_func(torch.zeros(1, 4, 2, 64), torch.zeros(1, 4, 3, 2, 64))
    with pytest.raises(ValueError):
        mfa.flash_attn_varlen_qkvpacked_func(torch.zeros(4, 2, 2, 64), torch.tensor([0, 4]), 4)
    with pytest.raises(ValueError):
        mfa.flash_attn_varlen_kvpacked_func(torch.zeros(4, 2, 64), torch.zeros(4, 3, 2, 64),
                                            torch.tensor([0, 4]), torch.tensor([0, 4]), 4, 4)


def test_boundary_rejects_negative_softcap_and_cpu():
    q = torch.zeros(1, 2, 8, 64)
    with pytest.raises(ValueError):
        mfa.flash_attn_forward(q, q, q, scale=0.1, causal=False, softcap=-1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        mfa.flash_attn_forward(q, q, q, scale=0.1, causal=False)


def test_torch_tier_is_not_part_of_the_engine(monkeypatch):
    monkeypatch.setenv("MTLFLASHATTN_KERNEL", "torch")
    with pytest.raises(RuntimeError, match="oracle"):
        _kernel._tier_mode(torch.float16)
    monkeypatch.setenv("MTLFLASHATTN_KERNEL", "v0")
    assert _kernel._tier_mode(torch.float16) == 2
    monkeypatch.setenv("MTLFLASHATTN_KERNEL", "v2_bf16")
    assert _kernel._tier_mode(torch.bfloat16) == 1
    monkeypatch.setenv("MTLFLASHATTN_KERNEL", "v2_dtype")
    assert _kernel._tier_mode(torch.float32) == 2


def test_alibi_broadcast():
    s = _kernel._broadcast_alibi_slopes(torch.tensor([1.0, 2.0]), 3, 2, "cpu")
    assert s.tolist() == [1.0, 2.0] * 3
    with pytest.raises(ValueError):
        _kernel._broadcast_alibi_slopes(torch.ones(3), 1, 2, "cpu")


def test_sdpa_install_uninstall_and_cpu_passthrough(monkeypatch):
    orig = F.scaled_dot_product_attention
    assert sdpa.install(min_score_gb=1e-9)
    try:
        assert F.scaled_dot_product_attention is not orig
        assert not sdpa.install()
        q = torch.randn(1, 2, 16, 8)
        out = F.scaled_dot_product_attention(q, q, q)  # CPU: not eligible -> stock, bitwise
        assert torch.equal(out, orig(q, q, q))
        ok, reason = sdpa._eligibility(q, q, q, None, 0.0, False)
        assert not ok and reason == "not-cuda"
    finally:
        assert sdpa.uninstall()
    assert F.scaled_dot_product_attention is orig
    monkeypatch.setenv("MTLFLASHATTN_SDPA", "off")
    assert not sdpa.install()


def test_sdpa_uneven_v_padding_is_exact(monkeypatch):
    """A routed call whose value head dim differs from the query/key one runs on q/k/v
    zero-padded to the larger dim and slices the output: exact, checked here with the oracle
    standing in for the kernel."""
    from oracle import flash_torch as ref

    seen = []

    def fake_forward(q, k, v, scale, causal):
        seen.append(q.shape[-1])
        return ref.attention_heads_second(q, k, v, scale, causal)

    monkeypatch.setattr(sdpa, "flash_attn_forward", fake_forward)
    g = torch.Generator().manual_seed(3)
    for Dqk, Dv in ((40, 64), (64, 24), (100, 128)):
        q = torch.randn(1, 2, 20, Dqk, generator=g)
        k = torch.randn(1, 2, 24, Dqk, generator=g)
        v = torch.randn(1, 2, 24, Dv, generator=g)
        for causal in (False, True):
            if causal:
                k, v = k[:, :, :20], v[:, :, :20]
            out = sdpa._engine(q, k, v, causal, None)
            want = torch.softmax((q @ k.transpose(-1, -2)) / Dqk ** 0.5 + (
                torch.full((20, k.shape[2]), float("-inf")).triu(1) if causal else 0), -1) @ v
            assert out.shape == (1, 2, 20, Dv)
            torch.testing.assert_close(out, want, atol=1e-5, rtol=1e-5)
    assert all(d % 8 == 0 for d in seen)


def test_trace_records_and_summarises(monkeypatch):
    _kernel._trace.clear()
    _kernel._record_trace(torch.bfloat16, 64, 128, 128, True, "cuda/tcgen05")
    _kernel._record_trace(torch.bfloat16, 64, 128, 128, True, "cuda/tcgen05")
    key = ("bfloat16", 64, 128, 128, True, "cuda/tcgen05")
    assert _kernel._trace[key] == 2
    assert any("cuda/tcgen05" in line for line in _kernel._trace_summary_lines())
    _kernel._record_trace(object(), "bad", None, None, None, None)  # never raises
    _kernel._trace.clear()


def run_py(code, env_extra=None):
    env = os.environ.copy()
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    env.update(env_extra or {})
    return subprocess.run([sys.executable, "-c", textwrap.dedent(code)], capture_output=True,
                          text=True, env=env, timeout=120)


def test_shim_kill_switch_and_idempotent_install():
    r = run_py("""
        import mtlflashattn_b200._shim as s
        print(s.install(), s.install())
    """, {"MTLFLASHATTN_SHIM": "off"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["False", "False"]
    r = run_py("""
        import mtlflashattn_b200._shim as s
        print(s.install(), s.install())
        import importlib.metadata as md
        print("flash_attn" in md.packages_distributions())
    """)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["True", "False", "True"]


def test_shim_real_install_wins(tmp_path):
    pkg = tmp_path / "flash_attn"
    pkg.mkdir()
    (pkg / "__init__.py").write_text('__version__ = "9.9.9-real"\n')
    r = run_py("""
        import mtlflashattn_b200._shim as s; s.install()
        import flash_attn; print(flash_attn.__version__)
    """, {"PYTHONPATH": f"{tmp_path}{os.pathsep}{ROOT}"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "9.9.9-real"


def test_shim_finder_gated_on_cuda():
    """The finder never serves flash_attn on a machine without CUDA (reference: fires only when
    the accelerator is available, _mtlflashattn_finder.py:33-40)."""
    from mtlflashattn_b200 import _finder

    spec = _finder._MtlFlashAttnB200Finder().find_spec("flash_attn")
    assert (spec is not None) == torch.cuda.is_available()
    assert _finder._MtlFlashAttnB200Finder().find_spec("numpy") is None


def test_host_api_argument_errors():
    q = torch.zeros(1, 8, 2, 64, dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        mfa.flash_attn_host(q, q, q)
    q = torch.zeros(1, 8, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        mfa.flash_attn_host(q, q, q, window_size=(-2, 0))
    with pytest.raises(ValueError):
        mfa.flash_attn_host(q, q, q, softcap=-1.0)
    with pytest.raises(NotImplementedError):
        mfa.flash_attn_host(torch.zeros(1, 8, 2, 160, dtype=torch.bfloat16), q, q)
