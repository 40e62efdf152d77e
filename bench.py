"""Benchmark: attention forward throughput (causal-adjusted TFLOP/s) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1|2|3|4|5|target] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

The default workload is BASELINE config 5, the one the metric quotes at 1/2/4/8 GPUs: one
131072-token sequence, B=1 H=16 D=128 bf16 causal, inputs 0.5*N(0,1). One step = one forward of
the whole problem over inputs already resident in HBM (``value``). With N ranks the heads are
sharded over the ranks (KV-group-aligned, no communication): strong scaling, ``value`` = the
whole problem's FLOPs over the max-over-ranks device time. At N > 1 the same line carries a
``split_kv`` leg: every rank holds one contiguous key range of all heads with equal causal
work and computes partials for every query row into its own buffer; each rank then merges its
own rows reading every rank's partials over NVLink (peer loads, one kernel). The same leg with
the forward pushing rows to their owners (``push_merge``) and with the NCCL merge (all-gather
of the row log-sum-exp, rescale kernel, reduce-scatter by query rows; ``nccl_merge``) is
reported beside it. Phases are timed with CUDA
events. Every run checks sampled row windows of its
output against a single-GPU forward of the same rows (``parity``).

``e2e`` is the same workload through the public host-memory API (``flash_attn_host``): pinned
host inputs copied in and the output copied back inside the timed region.

At N = 1 the line also carries ``configs``: BASELINE configs 1, 2, 3, 4 and the D=128 target,
each timed on the device the same way, and ``cpu_baseline``: the reference's CPU algorithm (the
chunked-fp32 torch tier, restated in oracle/flash_torch.py) on a bounded sample of config 5 and
on all of config 1.

``--impl reference`` times the reference's own CPU algorithm on the host cores, on a bounded
sample of the same workload.
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
SUB_CONFIGS = ("2", "target", "3", "4", "1")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return dict(bf16=float(d["bf16_tflops"]), bf16_sustained=float(d["bf16_tflops_sustained"]),
                    hbm=float(d["hbm_gbs"]), source="measured")
    except Exception:
        return dict(bf16=1590.0, bf16_sustained=1400.0, hbm=6650.0, source="fallback")


# ------------------------------------------------------------------------------ workloads
DENSE = {
    # name: (B, L, H, D, dtype, causal, kwargs, input scale)
    "1": (1, 1024, 4, 64, torch.float32, False, {}, 1.0),
    "2": (1, 8192, 16, 64, torch.bfloat16, True, {}, 1.0),
    "3": (1, 8192, 16, 128, torch.float16, False, dict(softcap=30.0, window_size=(1024, 1024)), 1.0),
    "target": (1, 8192, 16, 128, torch.bfloat16, True, {}, 1.0),
    "5": (1, 131072, 16, 128, torch.bfloat16, True, {}, 0.5),
}


def workload(cfg, device, rank=0, world=1):
    """Synthetic inputs with the BASELINE config's shapes and distributions (N(0,1), seeded).
    Returns (call(q, k, v) launching exactly one kernel, host inputs, algorithmic FLOPs,
    compulsory HBM bytes, description). Config 5 at world > 1 gives this rank its heads."""
    import mtlflashattn_b200 as mfa

    g = torch.Generator().manual_seed(1000 + rank)
    if cfg in DENSE:
        B, L, H, D, dt, causal, kw, sc = DENSE[cfg]
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
        nbytes = compulsory_bytes(B, Hr, Hr, L, L, D, elem=q.element_size())

        def call(q, k, v):
            return mfa.flash_attn_func(q, k, v, causal=causal, **kw)

        def host_call(q, k, v, out):  # pinned host tensors in and out
            return mfa.flash_attn_host(q, k, v, causal=causal, device=device, out=out,
                                       synchronize=False, **kw)

        call.host = host_call
        name = "target" if cfg == "target" else f"config{cfg}"
        desc = dict(workload=name, batch_per_rank=B, seq_len=L, heads=H, head_dim=D,
                    dtype=str(dt).replace("torch.", ""), causal=causal,
                    **{k_: list(v_) if isinstance(v_, tuple) else v_ for k_, v_ in kw.items()})
        if sc != 1.0:
            desc["input_scale"] = sc
        if strong:
            desc.update(heads_per_rank=Hr, strong=True, head_range=[h0, h1],
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

# ------------------------------------------------------------------------------- CPU leg
def cpu_sample_run(reps_budget_s=10.0, steps=None, rows=512):
    """Time the reference's CPU algorithm (oracle port of the chunked-fp32 torch tier) on a
    bounded sample of config 5: one head, ``rows`` query rows centred in the middle of the
    131072-token sequence (their mean causal key count equals the full problem's), bf16 inputs
    0.5*N(0,1). Returns (TFLOP/s over the sample's algorithmic FLOPs, seconds per sample,
    description)."""
    from oracle import flash_torch as ref

    L, D, r = 131072, 128, rows
    r0 = L // 2 - r // 2
    g = torch.Generator().manual_seed(0)
    q = (torch.randn(1, r, 1, D, generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, r0 + r, 1, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, r0 + r, 1, D, generator=g) * 0.5).bfloat16()
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    flops = 4 * D * sum(r0 + i + 1 for i in range(r))

    def one():
        # rows [r0, r0 + r) of the full problem: bottom-right causal over keys [0, r0 + r)
        ref.attention_heads_second(qh, kh, vh, 1 / math.sqrt(D), True).to(torch.bfloat16)

    one()  # warm-up
    times = []
    t_end = time.perf_counter() + reps_budget_s
    n = 0
    while (steps is None and (time.perf_counter() < t_end or n == 0)) or (steps is not None and n < steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        n += 1
    t = statistics.median(times)
    desc = (f"config5 sample: 1 of 16 heads, query rows [{r0},{r0 + r}) of 131072 against their "
            f"causal key prefix (mean key count = the full problem's, so the rate extrapolates to "
            f"the full problem; the full problem is 16 heads x 131072 rows); {n} timed "
            f"repetitions, median")
    return flops / t / 1e12, t, desc


def cpu_config1_run(reps_budget_s=5.0):
    """The reference's stated CPU run, whole and unsampled: BASELINE config 1 (B=1 H=4
    Lq=Lk=1024 D=64 fp32, q/k/v N(0,1) from seed 0, non-causal, scale 1/8) through the chunked
    fp32 torch tier (oracle port), timed like the reference's bench loop (bench/bench_attn.py:
    14-22: warm-up, then the median of timed repetitions)."""
    from oracle import flash_torch as ref

    q, k, v = ref.make_qkv(1, 1024, 1024, 4, 4, 64, torch.float32, seed=0)
    flops = attention_flops(1, 4, 1024, 1024, 64, False)
    for _ in range(3):
        ref.flash_attn_func(q, k, v, softmax_scale=0.125)
    times = []
    t_end = time.perf_counter() + reps_budget_s
    while time.perf_counter() < t_end or len(times) < 5:
        t0 = time.perf_counter()
        ref.flash_attn_func(q, k, v, softmax_scale=0.125)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return dict(value=round(flops / t / 1e12, 6), unit="TFLOP/s", ms=round(t * 1e3, 3),
                reps=len(times), sample="all of config 1 (B=1 H=4 L=1024 D=64 fp32, non-causal)")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # a fixed sample (the same 256 middle rows the GPU line's cpu_baseline uses), so the work per
    # step does not depend on the host: ~0.1 s per step on 16 cores
    rows = 256
    for _ in range(args.warmup):
        cpu_sample_run(steps=1, rows=rows)
    tf, t, desc = cpu_sample_run(steps=args.steps, rows=rows)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tf, 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded 0.5*N(0,1))",
        "config": dict(workload="config5", seq_len=131072, heads=16, head_dim=128, causal=True,
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


def window_diff(q, k, v, out, windows, row0=0):
    """Largest |out - reference| over sampled query-row windows of a bottom-right causal
    problem with Lq == Lk. Rows [r0, r1) of the full problem equal a forward with Lq = r1 - r0
    over keys [0, r1), run here as a separate single-GPU forward. ``out`` holds the rows from
    ``row0`` on (a rank's own rows after a split-KV merge)."""
    import mtlflashattn_b200 as mfa

    worst = 0.0
    for r0, r1 in windows:
        w = mfa.flash_attn_func(q[:, r0:r1], k[:, :r1], v[:, :r1], causal=True)
        got = out[:, r0 - row0:r1 - row0]
        worst = max(worst, (w.float() - got.float()).abs().max().item())
    return worst


def sample_windows(lo, hi, width=512, n=5):
    """n windows of `width` rows spread over [lo, hi), first and last included."""
    if hi - lo <= width:
        return [(lo, hi)] if hi > lo else []
    starts = sorted({lo + (hi - width - lo) * i // (n - 1) for i in range(n)})
    return [(a, a + width) for a in starts]


def measure(cfg, dev, steps, warmup, flush, stream, rank=0, world=1):
    """Device time of `steps` forwards of workload `cfg` (inputs resident). Returns (per-step
    ms list, flops, nbytes, desc, call, device inputs, host inputs, last output)."""
    call, host_in, flops, nbytes, desc = workload(cfg, dev, rank, world)
    dev_in = [t.to(dev) for t in host_in]
    last = []

    def step():
        last[:] = [call(*dev_in)]

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    times = timed_steps(step, steps, flush, stream)
    return times, flops, nbytes, desc, call, dev_in, host_in, last[0]


def split_kv_leg(steps, warmup, dev, rank, world, flush, stream, dist, merge):
    """Config 5 as split-KV over the ranks: rank g holds one contiguous key range of all heads
    with equal causal work (balanced_ranges; all ranks draw the same seeded q/k/v on the
    device), computes partials for all 131072 query rows, and the merge leaves each rank its
    own rows. merge = "pull": each rank's forward writes its partials to its own buffer and
    each rank merges its rows reading all ranks' buffers over NVLink (one kernel); "peer": the
    forward scatters partial rows into their owners' receive buffers over NVLink, then one
    local merge kernel; "nccl": all-gather of the row log-sum-exp, rescale kernel,
    reduce-scatter. Per step, CUDA events on the launching stream
    time the phases; every figure is the max over ranks."""
    from mtlflashattn_b200 import distributed as mfd

    B, L, H, D, dt, causal, _, sc = DENSE["5"]
    gen = torch.Generator(device=dev).manual_seed(2024)
    q = (torch.randn(B, L, H, D, device=dev, generator=gen) * sc).to(dt)
    k = (torch.randn(B, L, H, D, device=dev, generator=gen) * sc).to(dt)
    v = (torch.randn(B, L, H, D, device=dev, generator=gen) * sc).to(dt)
    rng = mfd.balanced_ranges(L, world, rank, causal=True)
    kp = [k[:, a:b].contiguous() for a, b in rng]
    vp = [v[:, a:b].contiguous() for a, b in rng]
    last = []

    def one(ev=None):
        last[:] = [mfd.flash_attn_split_kv(q, kp, vp, rng, L, causal=True, events=ev,
                                           merge=merge)]

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    dist.barrier()
    parts = []
    for _ in range(steps):
        flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        ev = {}
        s.record(stream)
        one(ev)
        e.record(stream)
        parts.append((s, e, ev))
    torch.cuda.synchronize()
    acc = {}
    for s, e, ev in parts:
        fwd = ev["forward_done"]
        ph = {"total": s.elapsed_time(e), "forward": s.elapsed_time(fwd)}
        if merge in ("peer", "pull"):
            ph["exchange_wait"] = fwd.elapsed_time(ev["exchange_done"])
            ph["merge"] = ev["exchange_done"].elapsed_time(e)
        else:
            ph["lse_allgather"] = ev["lse_gather"][0].elapsed_time(ev["lse_gather"][1])
            ph["rescale"] = ev["lse_gather"][1].elapsed_time(ev["reduce_scatter"][0])
            ph["reduce_scatter"] = ev["reduce_scatter"][0].elapsed_time(ev["reduce_scatter"][1])
        for name, val in ph.items():
            acc[name] = acc.get(name, 0.0) + val / steps
    names = sorted(acc)
    t = torch.tensor([acc[n] for n in names], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    acc = dict(zip(names, t.tolist()))
    out, (r0, r1) = last[0]
    diff = window_diff(q, k, v, out, sample_windows(r0, r1), row0=r0)
    dd = torch.tensor([diff], device=dev, dtype=torch.float64)
    dist.all_reduce(dd, op=dist.ReduceOp.MAX)
    flops = attention_flops(B, H, L, L, D, causal)
    tot = acc["total"]
    res = {
        "value": round(flops / (tot * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
        "ms_per_step": round(tot, 4), "steps": steps, "merge": merge,
        "phases_ms": {n: round(acc[n], 4) for n in names if n != "total"},
        "merge_share": round((tot - acc["forward"]) / tot, 4),
        "key_ranges": "one contiguous range per rank with equal causal work",
        "parity": {"max_abs_diff_vs_single_gpu": round(dd.item(), 6), "ok": dd.item() <= 2e-2,
                   "windows_per_rank": len(sample_windows(r0, r1))},
    }
    if merge == "nccl":
        res["collective_share"] = round((acc["lse_allgather"] + acc["reduce_scatter"]) / tot, 4)
    return res


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

        import datetime

        # a short collective timeout: a rank that fails in the split-KV leg must not leave the
        # others waiting for NCCL's default of ten minutes
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    call, host_in, flops, nbytes, desc = workload(args.config, dev, rank, world)
    strong = bool(desc.pop("strong", False))
    total_flops = desc.pop("total_flops", world * flops)
    dev_in = [t.to(dev) for t in host_in]
    last = []

    def step():
        last[:] = [call(*dev_in)]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        times = timed_steps(step, args.steps, flush, stream)
    torch.cuda.synchronize()
    barrier()
    ms_step = max_over_ranks(sum(times)) / args.steps
    value = total_flops / (ms_step * 1e-3) / 1e12

    # parity: sampled row windows of this rank's output against a single-GPU forward of the
    # same rows (exact restatement for bottom-right causal Lq == Lk)
    parity = None
    if args.config in ("5", "2", "target"):
        L = desc["seq_len"]
        diff = max_over_ranks(window_diff(*dev_in, last[0], sample_windows(0, L)))
        parity = {"max_abs_diff_vs_single_gpu": round(diff, 6), "ok": diff <= 2e-2,
                  "windows": [list(w) for w in sample_windows(0, L)],
                  "what": "rows [r0, r1) of every head this rank ran vs a separate forward of "
                          "Lq = r1 - r0 over keys [0, r1)"}
    del last[:]

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
    e2e_ms = max_over_ranks(sum(e_times)) / args.e2e_steps
    d2h = out_host.numel() * out_host.element_size()
    del pinned, out_host, dev_in

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
    launches = args.steps  # the main timed region: one forward kernel per step

    split = None
    split_failed = False
    if world > 1 and args.config == "5" and not args.no_split_kv:
        # the headline is already measured: a failure here is reported in the line, not raised
        for merge in ("pull", "peer", "nccl"):
            torch.cuda.empty_cache()
            try:
                leg = split_kv_leg(min(args.steps, args.split_steps), args.warmup, dev, rank,
                                   world, flush, stream, dist, merge)
            except Exception as e:  # noqa: BLE001
                leg = {"merge": merge, "error": f"{type(e).__name__}: {e}"[:300]}
                split_failed = True
            if split is None:
                split = leg
            else:
                split["push_merge" if merge == "peer" else "nccl_merge"] = leg
            if split_failed:
                break
        torch.cuda.empty_cache()

    configs = None
    if world == 1 and not args.no_sub_configs:
        configs = {}
        for c in SUB_CONFIGS:
            if c == args.config:
                continue
            torch.cuda.empty_cache()
            n = min(args.steps, args.sub_steps)
            t_c, f_c, b_c, d_c, *_ = measure(c, dev, n, args.warmup, flush, stream)
            ms = statistics.mean(t_c)
            tf = f_c / (ms * 1e-3) / 1e12
            configs[d_c["workload"]] = {
                "value": round(tf, 3), "unit": "TFLOP/s", "ms_per_step": round(ms, 5),
                "steps": n, "frac_of_bf16_peak": round(tf / pk["bf16"], 4),
                "config": d_c,
                **({"note": "fp32 inputs: CUDA-core kernel, not a tensor-core rate"}
                   if c == "1" else {}),
            }

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong" if strong or args.config == "5" else "weak",
            "vs_baseline": None,
            "dtype": desc.get("dtype", "bfloat16").replace("bfloat16", "bf16").replace(
                "float16", "fp16").replace("float32", "f32"),
            "data": "synthetic (seeded N(0,1) scaled as BASELINE states, BASELINE shapes)",
            "config": dict(desc, global_batch=(desc.get("batch_per_rank", 1) if strong or world == 1
                                              else world * desc.get("batch_per_rank", 1)),
                           parallelism=(f"heads{world} (one sequence, KV-group-aligned head "
                                        "shards, no collective)" if strong else
                                        "single GPU" if world == 1 else
                                        f"dp{world} (batch shards, no collective)"),
                           l2="flushed (256 MiB write) before every timed step; inputs > L2"),
            "pct_of_peak": round(100 * value / world / pk["bf16"], 2),
            "hbm_gbs_compulsory": round(nbytes / (ms_step * 1e-3) / 1e9, 1),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3),
                         "peak": pk["bf16"], "unit": "TFLOP/s",
                         "frac": round(achieved / pk["bf16"], 4),
                         "peak_source": f"bf16_tflops (burst) of {pk['source']} peaks",
                         "frac_of_sustained": round(achieved / pk["bf16_sustained"], 4),
                         "traffic": traffic},
            "e2e": {"value": round(total_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4),
                    "api": "flash_attn_host / flash_attn_varlen_host (host tensors in and out; "
                           "copies of one piece overlap the forward of another)"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if parity is not None:
            line["parity"] = parity
        if split is not None:
            line["split_kv"] = split
        if configs is not None:
            line["configs"] = configs
    if dist is not None and not split_failed:  # after a failed collective the group is unusable
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            tf, _, sdesc = cpu_sample_run(reps_budget_s=args.cpu_seconds, rows=256)
            line["cpu_baseline"] = {"value": round(tf, 6), "unit": "TFLOP/s",
                                    "cores": torch.get_num_threads(), "kind": "port",
                                    "sample": sdesc,
                                    "config1_full": cpu_config1_run()}
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--split-steps", type=int, default=10)
    ap.add_argument("--sub-steps", type=int, default=30)
    ap.add_argument("--config", default="5", choices=["1", "2", "3", "4", "5", "target"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-split-kv", action="store_true")
    ap.add_argument("--no-sub-configs", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
