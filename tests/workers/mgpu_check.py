"""Worker launched by tests/test_gpu_multi.py under torch.distributed.run (one rank per GPU).

Checks, on every rank, against the oracle (the reference's chunked-fp32 algorithm, run on this
GPU in fp32) with the bf16 bar of 1e-2 beyond output rounding:
  * head sharding: this rank's heads of the full problem;
  * gather_heads reassembles the head shards exactly;
  * split-KV over zigzag key chunks and over balanced contiguous key ranges, merged through
    peer memory (the forward scatters partial rows to their owners, then a local merge) and
    by all-gather of the row log-sum-exp + rescale + reduce-scatter by query rows: this rank's
    rows, and with gather=True every row."""
import math, os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from mtlflashattn_b200 import distributed as mfd
from oracle import flash_torch as ref
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"]); local = int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local); dev = torch.device("cuda", local)
dist.init_process_group("nccl", device_id=dev)
L, Hq, Hkv, D = 4096, 16, 4, 128
q, k, v = ref.make_qkv(1, L, L, Hq, Hkv, D, torch.bfloat16, seed=7)
qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
want = ref.flash_attn_func(qd.float(), kd.float(), vd.float(), causal=True)  # oracle, fp32


def bar(got, exp):
    """max |got - exp| beyond half an output ulp (bf16 rounding of the exact value)."""
    half_ulp = exp.abs().clamp_min(2 ** -126) * 2 ** -8
    return ((got.float() - exp).abs() - half_ulp).max().item()


loc, (h0, h1) = mfd.flash_attn_head_sharded(qd, kd, vd, causal=True)
hs_err = bar(loc, want[:, :, h0:h1])
assert hs_err <= 1e-2, f"head shard vs oracle: {hs_err}"
g = mfd.gather_heads(loc, Hq, Hkv)
parts = [torch.empty_like(loc) for _ in range(world)]
dist.all_gather(parts, loc.contiguous())
assert torch.equal(g, torch.cat(parts, dim=2))
msgs = []
balanced = lambda L_, w, r: mfd.balanced_ranges(L_, w, r, causal=True)  # noqa: E731
for ranges_of, merge in ((mfd.zigzag_ranges, "nccl"), (mfd.zigzag_ranges, "peer"),
                         (mfd.zigzag_ranges, "pull"), (balanced, "peer"), (balanced, "pull")):
    rng = ranges_of(L, world, rank)
    kp, vp = [kd[:, a:b] for a, b in rng], [vd[:, a:b] for a, b in rng]
    for _ in range(2):  # a second call reuses the peer receive buffers
        rows, (r0, r1) = mfd.flash_attn_split_kv(qd, kp, vp, rng, L, causal=True, merge=merge)
    assert (r0, r1) == mfd.row_shard(L, world, rank)
    sk_err = bar(rows, want[:, r0:r1])
    assert sk_err <= 1e-2, f"split-kv ({merge}) rows vs oracle: {sk_err}"
    full = mfd.flash_attn_split_kv(qd, kp, vp, rng, L, causal=True, gather=True, merge=merge)
    fe = bar(full, want)
    assert fe <= 1e-2, f"split-kv ({merge}) gathered vs oracle: {fe}"
    msgs.append(f"{merge} {len(rng)} chunk(s) rows [{r0},{r1}) {sk_err:.3e}/{fe:.3e}")
print(f"rank {rank}: head-shard ok ({hs_err:.3e}), split-kv ok: " + "; ".join(msgs), flush=True)
dist.destroy_process_group()
