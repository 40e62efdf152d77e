"""The debug build with device-side bounds checks (libmfa_checks.so, -DMFA_CHECKS=1): every
TMA tile coordinate and output row address is checked before use and a failure is reported in
the error word instead of faulting. Runs a sweep of small and ragged shapes through it (in a
subprocess, since one process loads one libmfa) and requires no check to fire and every output
to match the oracle at the reference's tolerances."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "mtlflashattn_b200", "libmfa_checks.so")


@pytest.mark.skipif(not os.path.exists(LIB), reason="libmfa_checks.so not built")
def test_bounds_checked_build_sweep():
    code = textwrap.dedent("""
        import itertools, torch
        import mtlflashattn_b200 as mfa
        from mtlflashattn_b200 import _kernel
        from oracle import flash_torch as ref
        TOL = {torch.float16: dict(atol=1.5e-2, rtol=2e-2), torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}
        n = 0
        for L, D, dt in itertools.product((1, 3, 5, 17, 67, 133, 255, 257), (32, 64, 80, 128),
                                          (torch.bfloat16, torch.float16)):
            for Lq, Lk, kw in ((L, L, dict(causal=True)), (L, 2 * L + 3, dict(causal=True)),
                               (2 * L + 1, L, dict(causal=True)),
                               (L, L + 40, dict(window_size=(7, 3), softcap=5.0))):
                q, k, v = ref.make_qkv(1, Lq, Lk, 4, 2, D, dt, seed=L + D + Lq)
                out = mfa.flash_attn_func(q.cuda(), k.cuda(), v.cuda(), **kw)
                torch.testing.assert_close(out.float().cpu(), ref.flash_attn_func(q, k, v, **kw), **TOL[dt])
                n += 1
        lens = [1, 130, 0, 257, 64]
        q, k, v, cq, ck = ref.make_varlen(lens, [x + 5 for x in lens], 8, 2, 64, torch.bfloat16, seed=3)
        out = mfa.flash_attn_varlen_func(q.cuda(), k.cuda(), v.cuda(), cq.cuda(), ck.cuda(),
                                         max(lens), max(lens) + 5, causal=True)
        torch.testing.assert_close(out.float().cpu(), ref.flash_attn_varlen_func(q, k, v, cq, ck, causal=True),
                                   **TOL[torch.bfloat16])
        torch.cuda.synchronize()
        _kernel.check_device_errors("cuda")
        print("checked", n + 1, "launches")
    """)
    env = dict(os.environ, MTLFLASHATTN_LIB=LIB, MTLFLASHATTN_SYNC_CHECK="1",
               PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "checked" in r.stdout
