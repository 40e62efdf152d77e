"""Multi-GPU attention: one process per GPU, torch.distributed (NCCL on GPUs) for plumbing.

Two decompositions, neither present in the reference (its tiers run on one Apple GPU):

* Head sharding, no communication. ``head_shard`` splits the query heads into contiguous,
  KV-group-aligned ranges; each rank runs the forward on its heads only. ``gather_heads``
  reassembles the full output only for a caller that wants it on every rank.

* Split-KV for one long sequence. Each rank holds a subset of the keys (contiguous ranges;
  ``zigzag_ranges`` gives rank g the chunks g and 2W-1-g so causal work is equal), computes a
  partial output normalised by its own softmax sum plus the row log-sum-exp, and the partials
  are merged exactly: lse = log sum_g exp(lse_g), o = sum_g exp(lse_g - lse) o_g.
  ``merge_partials`` does that with one all_gather of the (small) lse and one all_reduce of the
  rescaled fp32 output. It runs on any backend, so the merge is tested on CPU with gloo.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _kernel


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


def flash_attn_head_sharded(q, k, v, softmax_scale=None, causal=False, window_size=(-1, -1),
                            softcap=0.0, alibi_slopes=None, group=None):
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


def merge_partials(o_part, lse_part, group=None):
    """Exact log-sum-exp merge of per-rank partials over disjoint key sets.

    o_part: fp32 [B, Lq, H, D], normalised by this rank's own softmax sum (0 where the rank saw
    no key of a row); lse_part: fp32 [B, H, Lq] (-inf where it saw none). Returns the merged
    fp32 [B, Lq, H, D] and lse [B, H, Lq] on every rank."""
    world = dist.get_world_size(group)
    lses = [torch.empty_like(lse_part) for _ in range(world)]
    dist.all_gather(lses, lse_part.contiguous(), group=group)
    lse_tot = torch.logsumexp(torch.stack(lses), dim=0)
    w = torch.nan_to_num(torch.exp(lse_part - lse_tot), nan=0.0)  # rows nobody attends
    o = o_part * w.transpose(1, 2).unsqueeze(-1)
    dist.all_reduce(o, op=dist.ReduceOp.SUM, group=group)
    return o, lse_tot


def flash_attn_split_kv(q, k_parts, v_parts, key_ranges, lk_total, softmax_scale=None,
                        causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                        group=None, out_dtype=None):
    """Attention of the full query set against keys spread over ranks.

    q: [B, Lq, Hq, D] (every rank); k_parts/v_parts: this rank's key chunks, each
    [B, n_i, Hkv, D], holding global key positions key_ranges[i] = (start, end) of lk_total.
    Returns the merged output [B, Lq, Hq, D] in out_dtype (default q.dtype) on every rank."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Lq, Hq, D = q.shape
    alibi = (_kernel._broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
             if alibi_slopes is not None else None)
    bias = _kernel._BiasParams(softcap, window_size[0], window_size[1], alibi)
    o_acc = torch.zeros(B, Lq, Hq, D, device=q.device, dtype=torch.float32)
    lse_acc = torch.full((B, Hq, Lq), float("-inf"), device=q.device, dtype=torch.float32)
    for kp, vp, (a, _) in zip(k_parts, v_parts, key_ranges):
        o = torch.empty(B, Lq, Hq, D, device=q.device, dtype=torch.float32)
        lse = torch.empty(B, Hq, Lq, device=q.device, dtype=torch.float32)
        _kernel.forward_bshd(q, kp, vp, o, scale, causal, bias, lse=lse, k_pos_offset=a,
                             lk_total=lk_total)
        tot = torch.logsumexp(torch.stack([lse_acc, lse]), dim=0)
        wa = torch.nan_to_num(torch.exp(lse_acc - tot), nan=0.0).transpose(1, 2).unsqueeze(-1)
        wb = torch.nan_to_num(torch.exp(lse - tot), nan=0.0).transpose(1, 2).unsqueeze(-1)
        o_acc = o_acc * wa + o * wb
        lse_acc = tot
    o, _ = merge_partials(o_acc, lse_acc, group=group)
    return o.to(out_dtype or q.dtype)
