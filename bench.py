"""Benchmark: attention forward throughput (causal-adjusted TFLOP/s) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5|target] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

One step = one forward of the workload over inputs already resident in HBM (``value``), and,
separately, the same workload through the public host-memory API (``flash_attn_host``) with
pinned host inputs copied in and the output copied back inside the timed region (``e2e``).
The default workload is BASELINE config 2 (B=1, H=16, L=8192, D=64, bf16, causal). With N ranks
each rank runs its own instance (batch-sharded, no collective: weak scaling), except config 5
(one 131072-token sequence), whose heads are sharded over the ranks (strong scaling); the
reported time is the max over ranks.

``--impl reference`` times the reference's own CPU algorithm (the chunked-fp32 torch tier,
restated in oracle/flash_torch.py) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from mtlflashattn_b200.flops import attention_flops, compulsory_bytes, varlen_flops  # noqa: E402

METRIC = "attn fwd causal-adjusted TFLOP/s at 1/2/4/8 B200; % of dense TC peak"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return dict(bf16=float(d["bf16_tflops"]), bf16_sustained=float(d["bf16_tflops_sustained"]),
                    hbm=float(d["hbm_gbs"]), source="measured")
    except Exception:
        return dict(bf16=1590.0, bf16_sustained=1400.0, hbm=6650.0, source="fallback")


# ------------------------------------------------------------------------------ workloads
def workload(cfg, device, rank=0, world=1):
    """Synthetic inputs with the BASELINE config's shapes and distributions (N(0,1), seeded).
    Returns (call(q, k, v) launching exactly one kernel, host inputs, algorithmic FLOPs,
    compulsory HBM bytes, description)."""
    import mtlflashattn_b200 as mfa

    g = torch.Generator().manual_seed(1000 + rank)
    if cfg in ("2", "3", "target", "5"):
        if cfg == "2":
            B, L, H, D, dt, causal, kw = 1, 8192, 16, 64, torch.bfloat16, True, {}
        elif cfg == "3":
            B, L, H, D, dt, causal, kw = 1, 8192, 16, 128, torch.float16, False, dict(
                softcap=30.0, window_size=(1024, 1024))
        elif cfg == "target":
            B, L, H, D, dt, causal, kw = 1, 8192, 16, 128, torch.bfloat16, True, {}
        else:
            B, L, H, D, dt, causal, kw = 1, 131072, 16, 128, torch.bfloat16, True, {}
        sc = 0.5 if cfg == "5" else 1.0
        # config 5 on N ranks: one sequence, head-sharded (each rank its KV-group-aligned heads,
        # no communication): strong scaling of the whole problem
        strong = cfg == "5" and world > 1
        Hr = H
        if strong:
            from mtlflashattn_b200.distributed import head_shard

            h0, h1 = head_shard(H, H, world, rank)
            Hr = h1 - h0
        q = (torch.randn(B, L, Hr, D, generator=g) * sc).to(dt)
        k = (torch.randn(B, L, Hr, D, generator=g) * sc).to(dt)
        v = (torch.randn(B, L, Hr, D, generator=g) * sc).to(dt)
        flops = attention_flops(B, Hr, L, L, D, causal, kw.get("window_size", (-1, -1)))
        nbytes = compulsory_bytes(B, Hr, Hr, L, L, D)

        def call(q, k, v):
            return mfa.flash_attn_func(q, k, v, causal=causal, **kw)

        def host_call(q, k, v, out):  # pinned host tensors in and out
            return mfa.flash_attn_host(q, k, v, causal=causal, device=device, out=out,
                                       synchronize=False, **kw)

        call.host = host_call

        desc = dict(workload=f"config{cfg}" if cfg != "target" else "target", batch_per_rank=B,
                    seq_len=L, heads=H, head_dim=D, dtype=str(dt).replace("torch.", ""),
                    causal=causal, **{k_: list(v_) if isinstance(v_, tuple) else v_
                                      for k_, v_ in kw.items()})
        if strong:
            desc.update(heads_per_rank=Hr, strong=True,
                        total_flops=attention_flops(B, H, L, L, D, causal, (-1, -1)))
        return call, (q, k, v), flops, nbytes, desc
    if cfg == "4":
        lens = torch.randint(256, 8193, (16,), generator=torch.Generator().manual_seed(0)).tolist()
        tot = sum(lens)
        q = torch.randn(tot, 32, 128, generator=g).bfloat16()
        k = torch.randn(tot, 8, 128, generator=g).bfloat16()
        v = torch.randn(tot, 8, 128, generator=g).bfloat16()
        cu = torch.tensor([0] + lens, dtype=torch.int32).cumsum(0, dtype=torch.int32).to(device)
        slopes = torch.tensor([2 ** (-8 * (i + 1) / 32) for i in range(32)], device=device)
        flops = varlen_flops(lens, lens, 32, 128, True)
        nbytes = tot * 128 * 2 * (32 + 8 + 8 + 32)
        mx = max(lens)

        def call(q, k, v):
            return mfa.flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, causal=True,
                                              alibi_slopes=slopes)

        cu_h = cu.cpu()

        def host_call(q, k, v, out):  # pinned host tensors in and out
            return mfa.flash_attn_varlen_host(q, k, v, cu_h, cu_h, mx, mx, causal=True,
                                              alibi_slopes=slopes, device=device, out=out,
                                              synchronize=False)

        call.host = host_call

        desc = dict(workload="config4", sequences=16, total_tokens=tot, heads_q=32, heads_kv=8,
                    head_dim=128, dtype="bfloat16", causal=True, alibi=True)
        return call, (q, k, v), flops, nbytes, desc
    raise ValueError(f"unknown config {cfg}")


# ------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every few ms on a thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            pass

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self):
        if not self._ok:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvml unavailable"], samples=0)
        reasons = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return dict(sm_mhz=statistics.median(self.samples) if self.samples else None,
                    sm_max_mhz=self.max_mhz, reasons=reasons, samples=len(self.samples))


# ------------------------------------------------------------------------------- CPU leg
def cpu_sample_run(reps_budget_s=10.0, steps=None, rows=512):
    """Time the reference's CPU algorithm (oracle port of the chunked-fp32 torch tier) on a
    bounded sample of config 2: one head, ``rows`` query rows centred in the middle of the
    sequence (their mean causal key count equals the full problem's), all 8192 keys, bf16
    inputs. Returns (TFLOP/s over the sample's algorithmic FLOPs, seconds per sample,
    description)."""
    from oracle import flash_torch as ref

    L, D, r = 8192, 64, rows
    r0 = L // 2 - r // 2
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, r, 1, D, generator=g).bfloat16()
    k = torch.randn(1, L, 1, D, generator=g).bfloat16()
    v = torch.randn(1, L, 1, D, generator=g).bfloat16()
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    flops = 4 * D * sum(r0 + i + 1 for i in range(r))

    def one():
        ref.attention_heads_second(qh, kh, vh, 1 / math.sqrt(D), True, row_offset=r0,
                                   lq_total=L).to(torch.bfloat16)

    one()  # warm-up
    times = []
    t_end = time.perf_counter() + reps_budget_s
    n = 0
    while (steps is None and time.perf_counter() < t_end) or (steps is not None and n < steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        n += 1
    t = statistics.median(times)
    desc = (f"config2 sample: 1 of 16 heads, query rows [{r0},{r0 + r}) of 8192 (mean causal "
            f"key count = full problem's), all 8192 keys; {n} timed repetitions, median")
    return flops / t / 1e12, t, desc


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # size the per-step sample so the whole --steps/--warmup run stays within ~2 minutes
    _, t512, _ = cpu_sample_run(steps=1, rows=512)
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(16, min(512, 512 * budget / max(t512, 1e-6))) // 16 * 16)
    for _ in range(args.warmup):
        cpu_sample_run(steps=1, rows=rows)
    tf, t, desc = cpu_sample_run(steps=args.steps, rows=rows)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tf, 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": dict(workload="config2", seq_len=8192, heads=16, head_dim=64, causal=True,
                       dtype_inputs="bfloat16", parallelism="host CPU"),
        "cpu_baseline": {"value": round(tf, 6), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(tf, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- GPU leg
def timed_steps(fn, steps, flush_buf, stream):
    """Run fn() `steps` times, flushing L2 before each, timing each call with CUDA events on
    `stream`. Returns the per-step times (ms)."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for s, e in evs:
        flush_buf.zero_()
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def run_gpu(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    call, host_in, flops, nbytes, desc = workload(args.config, dev, rank, world)
    strong = bool(desc.pop("strong", False))
    total_flops = desc.pop("total_flops", world * flops)
    dev_in = [t.to(dev) for t in host_in]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        call(*dev_in)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        times = timed_steps(step, args.steps, flush, stream)
    torch.cuda.synchronize()
    barrier()
    t = torch.tensor([sum(times)], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = t.item() / args.steps
    value = total_flops / (ms_step * 1e-3) / 1e12

    # end-to-end through the public host-memory API (flash_attn_host): pinned host inputs in,
    # the output back in pinned host memory; the library overlaps the copies with the compute
    pinned = [h.pin_memory() for h in host_in]
    out_host = torch.empty(host_in[0].shape, dtype=host_in[0].dtype, pin_memory=True)
    h2d = sum(h.numel() * h.element_size() for h in pinned)

    def e2e_step():
        call.host(*pinned, out_host)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e_times = timed_steps(e2e_step, args.e2e_steps, flush, stream)
    torch.cuda.synchronize()
    te = torch.tensor([sum(e_times)], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = te.item() / args.e2e_steps
    d2h = out_host.numel() * out_host.element_size()

    pk = peaks()
    achieved = flops / (statistics.mean(times) * 1e-3) / 1e12
    traffic = None
    tr_path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tr_path):
        try:
            with open(tr_path) as f:
                traffic = json.load(f).get(desc["workload"])
        except Exception:
            traffic = None
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": desc.get("dtype", "bfloat16").replace("bfloat16", "bf16").replace(
                "float16", "fp16"),
            "data": "synthetic (seeded N(0,1), BASELINE shapes)",
            "config": dict(desc, global_batch=(desc.get("batch_per_rank", 1) if strong else
                                              world * desc.get("batch_per_rank", 1)),
                           parallelism=(f"heads{world} (one sequence, KV-group-aligned head "
                                        "shards, no collective)" if strong else
                                        f"dp{world} (batch shards, no collective)"),
                           l2="flushed (256 MiB write) before every timed step"),
            "pct_of_peak": round(100 * value / world / pk["bf16"], 2),
            "hbm_gbs_compulsory": round(nbytes / (ms_step * 1e-3) / 1e9, 1),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3),
                         "peak": pk["bf16"], "unit": "TFLOP/s",
                         "frac": round(achieved / pk["bf16"], 4),
                         "peak_source": f"bf16_tflops (burst) of {pk['source']} peaks",
                         "traffic": traffic},
            "e2e": {"value": round(total_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4),
                    "api": "flash_attn_host / flash_attn_varlen_host (host tensors in and out; "
                           "copies of one piece overlap the forward of another)"},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            tf, _, sdesc = cpu_sample_run(reps_budget_s=args.cpu_seconds)
            line["cpu_baseline"] = {"value": round(tf, 6), "unit": "TFLOP/s",
                                    "cores": torch.get_num_threads(), "kind": "port",
                                    "sample": sdesc}
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--config", default="2", choices=["2", "3", "4", "5", "target"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
