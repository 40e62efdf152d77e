"""Worker launched by tests/test_gpu_multi.py under torch.distributed.run (one rank per GPU):
head sharding must reproduce the single-GPU result (within bf16 rounding: with half the heads a
launch has fewer CTAs than SMs and splits its keys over more CTAs, which changes the summation
order), gathering the heads must reassemble it exactly, and split-KV over zigzag key chunks
merged over NCCL must match it within bf16 tolerance."""
import os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import mtlflashattn_b200 as mfa
from mtlflashattn_b200 import distributed as mfd
from oracle import flash_torch as ref
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"]); local = int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local); dev = torch.device("cuda", local)
dist.init_process_group("nccl", device_id=dev)
q, k, v = ref.make_qkv(1, 4096, 4096, 16, 4, 128, torch.bfloat16, seed=7)
qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
full = mfa.flash_attn_func(qd, kd, vd, causal=True)
loc, (h0, h1) = mfd.flash_attn_head_sharded(qd, kd, vd, causal=True)
hs_err = (loc.float() - full[:, :, h0:h1].float()).abs().max().item()
assert hs_err < 2e-2, f"head shard differs: {hs_err}"
g = mfd.gather_heads(loc, 16, 4)
parts = [torch.empty_like(loc) for _ in range(world)]
dist.all_gather(parts, loc.contiguous())
assert torch.equal(g, torch.cat(parts, dim=2))
rng = mfd.zigzag_ranges(4096, world, rank)
o = mfd.flash_attn_split_kv(qd, [kd[:, a:b] for a, b in rng], [vd[:, a:b] for a, b in rng], rng, 4096, causal=True)
err = (o.float() - full.float()).abs().max().item()
assert err < 2e-2, err
print(f"rank {rank}: head-shard ok ({hs_err:.3e}), split-kv max diff vs single GPU {err:.3e}", flush=True)
dist.destroy_process_group()
