"""Multi-GPU attention: one process per GPU, torch.distributed (NCCL on GPUs) for plumbing.

Two decompositions, neither present in the reference (its tiers run on one Apple GPU):

* Head sharding, no communication. ``head_shard`` splits the query heads into contiguous,
  KV-group-aligned ranges; each rank runs the forward on its heads only. ``gather_heads``
  reassembles the full output only for a caller that wants it on every rank.

* Split-KV for one long sequence. Each rank holds a subset of the keys (``zigzag_ranges`` gives
  rank g the key chunks g and 2W-1-g, so causal work is equal) and computes, for every query
  row, a partial output normalised by its own softmax sum plus the row log-sum-exp. The merge is
  built for NVLink, not for a full-size all-reduce:

  1. each rank folds its own partials' log-sum-exp into one ``[B*H, Lq]`` fp32 row vector and
     the ranks all-gather it (``W x 4 B`` per row and head: 8 MB per rank at 131072 x 16);
  2. from the gathered vectors every rank knows the exact total log-sum-exp of every row, and
     one kernel (``mfa_lse_rescale_sum``) writes its partials' contribution
     ``sum_g exp(lse_g - lse) o_g`` into a row-major fp32 ``[Lq, B*H, D]`` buffer;
  3. one ``reduce_scatter`` by query rows sums the contributions: rank r receives its own rows
     ``row_shard(Lq, W, r)`` of the merged output, already normalised. Each rank sends and
     receives ``(W-1)/W`` of one fp32 output instead of all-reducing a whole one, and nobody
     holds rows it does not own unless it asks (``gather=True``).

  The rank's two zigzag chunks are two launches of the forward kernel writing their partials
  straight into the row-major layout (output strides), so no transpose or eager merge runs over
  the partials.

The collectives are plain torch.distributed calls and run on any backend; the rescale is the
library's CUDA kernel. Tests of the host logic on CPU (gloo) inject a CPU rescale instead.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _kernel, _lib


def head_shard(Hq, Hkv, world, rank):
    """Query-head range [h0, h1) of ``rank``: whole KV groups, as even as possible."""
    group = Hq // Hkv
    g0 = (Hkv * rank) // world
    g1 = (Hkv * (rank + 1)) // world
    return g0 * group, g1 * group


def zigzag_ranges(L, world, rank):
    """Key ranges of ``rank`` when L keys are cut into 2*world chunks and rank g takes chunks
    g and 2*world-1-g (balanced causal work). Returns a list of (start, end)."""
    n = 2 * world
    bounds = [(L * i) // n for i in range(n + 1)]
    out = []
    for c in (rank, n - 1 - rank):
        if bounds[c + 1] > bounds[c]:
            out.append((bounds[c], bounds[c + 1]))
    return out


def row_shard(Lq, world, rank):
    """Query rows [r0, r1) that ``rank`` owns after a split-KV merge: ceil(Lq / world) rows per
    rank (the reduce-scatter needs equal pieces; the last rank's piece may be short or empty)."""
    per = -(-Lq // world)
    r0 = min(Lq, per * rank)
    return r0, min(Lq, r0 + per)


def flash_attn_head_sharded(q, k, v, softmax_scale=None, causal=False, window_size=(-1, -1),
                            softcap=0.0, alibi_slopes=None, group=None, out=None):
    """This rank's heads of flash_attn_func(q, k, v, ...) on full [B, L, H, D] tensors (sliced
    here as views, no copy). Returns ([B, Lq, h1-h0, D], (h0, h1))."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    Hq, Hkv = q.shape[2], k.shape[2]
    h0, h1 = head_shard(Hq, Hkv, world, rank)
    grp = Hq // Hkv
    k0, k1 = h0 // grp, h1 // grp
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Lq = q.shape[0], q.shape[1]
    alibi = None
    if alibi_slopes is not None:
        alibi = _kernel._broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
        alibi = alibi.view(B, Hq)[:, h0:h1].contiguous().view(-1)
    bias = _kernel._BiasParams(softcap, window_size[0], window_size[1], alibi)
    if out is None:
        out = torch.empty(B, Lq, h1 - h0, q.shape[3], device=q.device, dtype=q.dtype)
    if h1 > h0:
        _kernel.forward_bshd(q[:, :, h0:h1], k[:, :, k0:k1], v[:, :, k0:k1], out, scale, causal,
                             bias)
    return out, (h0, h1)


def gather_heads(local, Hq, Hkv, group=None):
    """All-gather head shards into the full [B, L, Hq, D] on every rank (only for callers that
    want the whole output)."""
    world = dist.get_world_size(group)
    parts = []
    for r in range(world):
        h0, h1 = head_shard(Hq, Hkv, world, r)
        parts.append(torch.empty(local.shape[0], local.shape[1], h1 - h0, local.shape[3],
                                 device=local.device, dtype=local.dtype))
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=2)


def _rescale_sum_cuda(o_parts, lse_parts, lse_ref, out):
    """out[:Lq] = sum_g exp(lse_g - lse_ref) o_g with the library kernel (one launch)."""
    Lq, BH, D = o_parts[0].shape
    rc = _lib.lse_rescale_sum([t.data_ptr() for t in o_parts], [t.data_ptr() for t in lse_parts],
                              Lq, BH, D, lse_ref.data_ptr(), out.data_ptr(), _lib.FP32,
                              torch.cuda.current_stream(out.device).cuda_stream)
    if rc != _lib.OK:
        _kernel._raise_status(rc, "mfa_lse_rescale_sum")


def merge_partials(o_parts, lse_parts, group=None, rescale=None, events=None):
    """Exact log-sum-exp merge of split-KV partials held by every rank, scattered by query rows.

    o_parts: this rank's partials, each fp32 ``[Lq, BH, D]`` (row-major over query rows; BH =
    batch x heads), normalised by its own softmax sum (0 where it saw no key of a row);
    lse_parts: the matching fp32 ``[BH, Lq]`` row log-sum-exp (-inf where it saw none).
    Returns (o_rows fp32 ``[r1 - r0, BH, D]``, lse_rows fp32 ``[BH, r1 - r0]``, (r0, r1)) for
    this rank's rows ``row_shard(Lq, W, rank)``. ``rescale(o_parts, lse_parts, lse_ref, out)``
    overrides the CUDA kernel (host-logic tests on CPU). ``events``, if given, is a dict that
    receives CUDA events recorded before and after each collective (keys ``lse_gather`` and
    ``reduce_scatter``, each a (start, end) pair) so a caller can time the communication."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Lq, BH, D = o_parts[0].shape
    dev = o_parts[0].device

    def mark(name, i):
        if events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            events.setdefault(name, [None, None])[i] = ev

    lse_loc = lse_parts[0] if len(lse_parts) == 1 else torch.logsumexp(torch.stack(lse_parts), 0)
    lse_all = torch.empty(world * BH, Lq, device=dev, dtype=torch.float32)
    mark("lse_gather", 0)
    dist.all_gather_into_tensor(lse_all, lse_loc.contiguous(), group=group)
    mark("lse_gather", 1)
    lse_tot = torch.logsumexp(lse_all.view(world, BH, Lq), 0)  # -inf where no rank attends
    per = -(-Lq // world)
    contrib = torch.empty(per * world, BH, D, device=dev, dtype=torch.float32)
    if per * world > Lq:
        contrib[Lq:].zero_()
    (rescale or _rescale_sum_cuda)(o_parts, lse_parts, lse_tot, contrib)
    mine = torch.empty(per, BH, D, device=dev, dtype=torch.float32)
    mark("reduce_scatter", 0)
    dist.reduce_scatter_tensor(mine, contrib, op=dist.ReduceOp.SUM, group=group)
    mark("reduce_scatter", 1)
    r0, r1 = row_shard(Lq, world, rank)
    return mine[: r1 - r0], lse_tot[:, r0:r1], (r0, r1)


def flash_attn_split_kv(q, k_parts, v_parts, key_ranges, lk_total, softmax_scale=None,
                        causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                        group=None, out_dtype=None, gather=False, events=None):
    """Attention of the full query set against keys spread over ranks.

    q: [B, Lq, Hq, D] (every rank); k_parts/v_parts: this rank's key chunks, each
    [B, n_i, Hkv, D], holding global key positions key_ranges[i] = (start, end) of lk_total.
    Returns (o_rows [B, r1 - r0, Hq, D] in out_dtype (default q.dtype), (r0, r1)): this rank's
    query rows of the merged output. With ``gather=True`` the rows of every rank are
    all-gathered and the full [B, Lq, Hq, D] output is returned on every rank instead."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Lq, Hq, D = q.shape
    alibi = (_kernel._broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
             if alibi_slopes is not None else None)
    bias = _kernel._BiasParams(softcap, window_size[0], window_size[1], alibi)
    o_parts, lse_parts = [], []
    for kp, vp, (a, _) in zip(k_parts, v_parts, key_ranges):
        # partial rows straight into the row-major [Lq, B*Hq, D] layout the merge scatters
        o = torch.empty(Lq, B, Hq, D, device=q.device, dtype=torch.float32)
        lse = torch.empty(B, Hq, Lq, device=q.device, dtype=torch.float32)
        _kernel.forward_bshd(q, kp, vp, o.transpose(0, 1), scale, causal, bias, lse=lse,
                             k_pos_offset=a, lk_total=lk_total)
        o_parts.append(o.view(Lq, B * Hq, D))
        lse_parts.append(lse.view(B * Hq, Lq))
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events["forward_done"] = ev
    rows, _, (r0, r1) = merge_partials(o_parts, lse_parts, group=group, events=events)
    out = rows.view(r1 - r0, B, Hq, D).transpose(0, 1).to(out_dtype or q.dtype)
    if not gather:
        return out, (r0, r1)
    world = dist.get_world_size(group)
    per = -(-Lq // world)
    full = torch.zeros(world * per, B, Hq, D, device=q.device, dtype=out.dtype)
    mine = torch.zeros(per, B, Hq, D, device=q.device, dtype=out.dtype)
    mine[: r1 - r0] = out.transpose(0, 1)
    dist.all_gather_into_tensor(full, mine, group=group)
    return full[:Lq].transpose(0, 1).contiguous()
