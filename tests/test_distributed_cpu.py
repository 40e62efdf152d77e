"""Multi-rank logic on CPU with gloo (world size 2 and 3): head sharding covers every head once,
zigzag key ranges partition the keys with equal causal work, the split-KV log-sum-exp merge
(all-gather of the row log-sum-exp, rescale, reduce-scatter by query rows) gives every rank
exactly its rows of the unsplit oracle result, and a rank that leaves surfaces as an error."""
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


def cpu_rescale(o_parts, lse_parts, lse_ref, out):
    """CPU statement of the library's mfa_lse_rescale_sum (the GPU kernel), for the host-logic
    test: out[:Lq] = sum_g exp(lse_g - lse_ref) o_g, 0 where either is -inf."""
    Lq = o_parts[0].shape[0]
    acc = torch.zeros_like(o_parts[0])
    for o, lse in zip(o_parts, lse_parts):
        w = torch.exp(lse - lse_ref)
        w = torch.where(torch.isinf(lse) | torch.isinf(lse_ref), torch.zeros_like(w), w)
        acc += w.t()[..., None] * o
    out[:Lq] = acc


def _merge_worker(rank, world, port, q, k, v, causal, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import flash_torch as ref
        L = k.shape[2]
        o_parts, lse_parts = [], []
        for a, b in mfd.zigzag_ranges(L, world, rank):
            o, lse = ref.attention_heads_second(q, k[:, :, a:b], v[:, :, a:b], 0.2, causal,
                                                softcap=7.0, alibi=torch.tensor([0.1, 0.3]),
                                                return_lse=True, key_offset=a, lk_total=L)
            B, H, Lq, D = o.shape
            # the forward's output strides put partial rows in [Lq, B*H, D]
            o_parts.append(o.permute(2, 0, 1, 3).reshape(Lq, B * H, D).contiguous())
            lse_parts.append(lse.reshape(B * H, Lq))
        o, lse, rows = mfd.merge_partials(o_parts, lse_parts, rescale=cpu_rescale)
        result_q.put((rank, o, lse, rows))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("causal", [True, False])
def test_split_kv_merge_over_gloo_matches_unsplit(world, causal):
    """Each rank ends with exactly its own query rows of the merged output (reduce-scatter by
    rows), equal to the unsplit oracle result; together the ranks cover every row once."""
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
    want = full[0].transpose(0, 1)  # [Lq, H, D]
    covered = []
    for rank, o, lse, (r0, r1) in results:
        assert (r0, r1) == mfd.row_shard(50, world, rank)
        covered += list(range(r0, r1))
        torch.testing.assert_close(o, want[r0:r1], atol=1e-5, rtol=1e-5)
        wl = full_lse[0][:, r0:r1]
        fin = torch.isfinite(wl)
        torch.testing.assert_close(lse[fin], wl[fin], atol=1e-5, rtol=1e-5)
    assert sorted(covered) == list(range(50))


def test_balanced_ranges_equal_causal_work():
    for L, Lq in ((8192, 8192), (131072, 131072), (5000, 300)):
        for world in (1, 2, 3, 8):
            rr = [mfd.balanced_ranges(L, world, r, causal=True, Lq=Lq)[0] for r in range(world)]
            assert rr[0][0] == 0 and rr[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(rr, rr[1:]))
            work = [attention_pairs(Lq, b - a, True, key_offset=a, lk_total=L) for a, b in rr]
            assert max(work) - min(work) <= 2 * Lq, (L, world, work)  # a key column per boundary
        nc = [mfd.balanced_ranges(L, 4, r, causal=False)[0] for r in range(4)]
        assert [b - a for a, b in nc] == [L // 4] * 4 or sum(b - a for a, b in nc) == L


def test_row_shard_partition():
    for Lq in (1, 7, 50, 131072):
        for world in (1, 2, 3, 8):
            got = [mfd.row_shard(Lq, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == Lq
            for (_, b), (c, _) in zip(got, got[1:]):
                assert b == c


def _dead_rank_worker(rank, world, port, result_q):
    """Rank 1 leaves before the merge; rank 0's collective must end with an error, not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if rank == 1:
            os._exit(0)
        mfd.merge_partials([torch.zeros(4, 2, 8)], [torch.zeros(2, 4)], rescale=cpu_rescale)
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
