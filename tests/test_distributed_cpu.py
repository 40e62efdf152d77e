"""Multi-rank logic on CPU with gloo (world size 2 and 3): head sharding covers every head once,
zigzag key ranges partition the keys with equal causal work, the split-KV log-sum-exp merge over
ranks reproduces the unsplit oracle result, and a rank that leaves surfaces as an error."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mtlflashattn_b200 import distributed as mfd
from mtlflashattn_b200.flops import attention_pairs


def test_head_shard_partition():
    for Hq, Hkv in ((16, 16), (32, 8), (8, 1), (5, 5)):
        for world in (1, 2, 3, 4, 8):
            got = [mfd.head_shard(Hq, Hkv, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == Hq
            for (_, b), (c, _) in zip(got, got[1:]):
                assert b == c
            for a, b in got:
                assert a % (Hq // Hkv) == 0 and b % (Hq // Hkv) == 0


def test_zigzag_ranges_partition_and_balance():
    L = 8192
    for world in (2, 4, 8):
        ranges = [mfd.zigzag_ranges(L, world, r) for r in range(world)]
        keys = sorted(x for rr in ranges for (a, b) in rr for x in range(a, b))
        assert keys == list(range(L))
        work = [sum(attention_pairs(L, b - a, True, key_offset=a, lk_total=L) for a, b in rr)
                for rr in ranges]
        assert max(work) / min(work) < 1.01


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _merge_worker(rank, world, port, q, k, v, causal, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import flash_torch as ref
        L = k.shape[2]
        parts = []
        for a, b in mfd.zigzag_ranges(L, world, rank):
            parts.append(ref.attention_heads_second(q, k[:, :, a:b], v[:, :, a:b], 0.2, causal,
                                                    softcap=7.0, alibi=torch.tensor([0.1, 0.3]),
                                                    return_lse=True, key_offset=a, lk_total=L))
        lses = torch.stack([p[1] for p in parts])
        lse_loc = torch.logsumexp(lses, 0)
        w = torch.nan_to_num(torch.exp(lses - lse_loc), nan=0.0)
        o_loc = sum(w[i][..., None] * parts[i][0] for i in range(len(parts)))
        o, lse = mfd.merge_partials(o_loc.transpose(1, 2).contiguous(), lse_loc)
        result_q.put((rank, o, lse))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("causal", [True, False])
def test_split_kv_merge_over_gloo_matches_unsplit(world, causal):
    from oracle import flash_torch as ref
    q, k, v = ref.make_qkv(1, 50, 96, 2, 2, 16, torch.float32, seed=5)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    full, full_lse = ref.attention_heads_second(qh, kh, vh, 0.2, causal, softcap=7.0,
                                                alibi=torch.tensor([0.1, 0.3]), return_lse=True)
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_merge_worker, args=(r, world, port, qh, kh, vh, causal, rq))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [rq.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, o, lse in results:
        torch.testing.assert_close(o, full.transpose(1, 2), atol=1e-5, rtol=1e-5)
        fin = torch.isfinite(full_lse)
        torch.testing.assert_close(lse[fin], full_lse[fin], atol=1e-5, rtol=1e-5)


def _dead_rank_worker(rank, world, port, result_q):
    """Rank 1 leaves before the merge; rank 0's collective must end with an error, not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if rank == 1:
            os._exit(0)
        mfd.merge_partials(torch.zeros(1, 4, 2, 8), torch.zeros(1, 2, 4))
        result_q.put("no-error")
    except Exception as e:  # noqa: BLE001 - init or the collective saw the missing rank
        if rank == 0:
            result_q.put(type(e).__name__)
    result_q.close()
    result_q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, rq)) for r in range(2)]
    for p in procs:
        p.start()
    res = rq.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res != "no-error"
