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

  The rank's key chunks are launches of the forward kernel writing their partials straight
  into the row-major layout (output strides), so no transpose or eager merge runs over them.

* Split-KV merged by pulling through peer memory (``merge="pull"``, the default on CUDA).
  Each rank's forward writes its partial rows and log-sum-exp into its own buffer (local
  stores at full speed; the buffer is libmfa-allocated so it carries a CUDA IPC handle and is
  mapped on every other rank). After an ordering point, each rank merges its own rows with one
  kernel (``mfa_lse_merge_rows``) that reads the rows from every rank's buffer with plain loads
  over NVLink and writes the final rows in the output dtype.

* Split-KV merged by pushing through peer memory (``merge="peer"``). The forward
  kernel's epilogue stores every partial row directly into the receive buffer of the GPU that
  owns the row (``mfa_fwd_scatter``: plain stores over NVLink into buffers mapped with CUDA
  IPC), so the exchange runs while the attention runs, tile by tile; each GPU then merges its
  own rows with one local kernel (``mfa_lse_merge``) that writes the final rows in the output
  dtype. No all-gather, rescale pass or reduce-scatter remains. On 4 GPUs the remote stores
  slowed the forward by ~19 % (3/4 of the rows are remote), which is why pulling is the default.
  For both, ordering between GPUs comes from two one-element NCCL all-reduces per call (buffers
  free before they are written, all partial rows written before they are read); no kernel ever
  waits on another GPU. With
  ``balanced_ranges`` each rank holds ONE contiguous key range of equal causal work, so a
  rank makes one launch and each row has one partial per rank.

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


def balanced_ranges(Lk, world, rank, causal=True, Lq=None):
    """One contiguous key range [k0, k1) for ``rank`` such that every rank's keys are attended
    by the same number of (query, key) pairs. Non-causal: equal key counts. Causal with
    bottom-right alignment: key j is seen by Lq - max(0, j - (Lk - Lq)) rows, so the early keys
    weigh more and rank 0's range is the shortest (for Lq = Lk, boundary r sits near
    Lk * (1 - sqrt(1 - r / world)))."""
    Lq = Lk if Lq is None else Lq
    if not causal:
        return [((Lk * rank) // world, (Lk * (rank + 1)) // world)]
    j = torch.arange(Lk, dtype=torch.float64)
    seen = (Lq - (j - (Lk - Lq)).clamp_min(0)).clamp_min(0)
    cum = torch.cumsum(seen, 0)
    total = float(cum[-1]) if Lk > 0 else 0.0

    def bound(r):
        if r <= 0:
            return 0
        if r >= world:
            return Lk
        return int(torch.searchsorted(cum, total * r / world).item())

    return [(bound(rank), bound(rank + 1))]


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


class _PeerBuffers:
    """Receive buffers of one split-KV shape on every rank of a group, mapped on all of them.
    One device allocation per rank (fp32 partial rows [slots][rows_per][BH][D] followed by the
    row log-sum-exp [slots][BH][rows_per]), allocated by libmfa (cudaMalloc, so it can carry a
    CUDA IPC handle), its handle all-gathered once and opened by every other rank."""

    _cache = {}

    def __init__(self, group, slots, rows_per, BH, D, device):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.o_bytes = slots * rows_per * BH * D * 4
        self.o_bytes += (-self.o_bytes) % 256
        nbytes = self.o_bytes + slots * BH * rows_per * 4
        with torch.cuda.device(device):
            ptr, handle = _lib.peer_alloc(nbytes)
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
            self.base = [ptr if g == rank else _lib.peer_open(handles[g]) for g in range(world)]
        self.rank, self.world, self.device = rank, world, device
        self.sync = torch.zeros(1, device=device)

    @classmethod
    def get(cls, group, slots, rows_per, BH, D, device, kind="push"):
        key = (kind, id(group), dist.get_world_size(group), slots, rows_per, BH, D, str(device))
        buf = cls._cache.get(key)
        if buf is None:
            buf = cls._cache[key] = cls(group, slots, rows_per, BH, D, device)
        return buf

    def scatter_table(self, rows_per, slot):
        sc = _lib.MfaPeerScatter()
        sc.n_peers, sc.rows_per_peer, sc.slot = self.world, rows_per, slot
        for g in range(self.world):
            sc.o_recv[g] = self.base[g]
            sc.lse_recv[g] = self.base[g] + self.o_bytes
        return sc


class _DeviceArray:
    """A device pointer presented as an array (``__cuda_array_interface__``), so torch can view
    memory libmfa allocated without copying it."""

    def __init__(self, ptr, shape, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2}


def _view(ptr, shape, device):
    return torch.as_tensor(_DeviceArray(ptr, shape), device=device)


def _order(buf, group):
    """Every rank's GPU work queued so far precedes what any rank queues next (a one-element
    NCCL all-reduce on the current stream)."""
    dist.all_reduce(buf.sync, group=group)


def _split_kv_peer(q, k_parts, v_parts, key_ranges, lk_total, scale, causal, bias, group,
                   out_dtype, events):
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Lq, Hq, D = q.shape
    nch = len(k_parts)
    rows_per = -(-Lq // world)
    buf = _PeerBuffers.get(group, world * nch, rows_per, B * Hq, D, q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _order(buf, group)  # the previous call's merges have read their receive buffers
    kernel = _kernel._tier_mode(q.dtype)
    for c, (kp, vp, (a, _)) in enumerate(zip(k_parts, v_parts, key_ranges)):
        kp, vp = _kernel._last_dim_contig(kp), _kernel._last_dim_contig(vp)
        p = _kernel._packed(q, kp, vp, q, B, Hq, kp.shape[2], Lq, kp.shape[1], D, q.stride()[:3],
                            kp.stride()[:3], vp.stride()[:3], q.stride()[:3], scale, causal, bias,
                            kernel, None, (0, 0), None, None, 0, 0, a, lk_total)
        rc = _lib.fwd_scatter(p, buf.scatter_table(rows_per, rank * nch + c), stream)
        if rc != _lib.OK:
            _kernel._raise_status(rc, "mfa_fwd_scatter")
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events["forward_done"] = ev
    _order(buf, group)  # every rank's partial rows have landed in the owners' buffers
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events["exchange_done"] = ev
    out = torch.empty(rows_per, B, Hq, D, device=q.device, dtype=out_dtype)
    rc = _lib.lse_merge(buf.base[rank], buf.base[rank] + buf.o_bytes, world * nch, rows_per,
                        B * Hq, D, out.data_ptr(), _kernel._DTYPES[out_dtype], None, stream)
    if rc != _lib.OK:
        _kernel._raise_status(rc, "mfa_lse_merge")
    r0, r1 = row_shard(Lq, world, rank)
    return out[: r1 - r0].transpose(0, 1), (r0, r1)


def _split_kv_pull(q, k_parts, v_parts, key_ranges, lk_total, scale, causal, bias, group,
                   out_dtype, events):
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Lq, Hq, D = q.shape
    nch = len(k_parts)
    BH = B * Hq
    buf = _PeerBuffers.get(group, nch, Lq, BH, D, q.device, kind="pull")
    slot_o = Lq * BH * D * 4
    slot_lse = BH * Lq * 4
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _order(buf, group)  # every rank has finished reading this rank's buffer in the last call
    own = buf.base[rank]
    for c, (kp, vp, (a, _)) in enumerate(zip(k_parts, v_parts, key_ranges)):
        # this rank's partial rows, row-major [Lq][B][Hq][D] fp32, and their log-sum-exp
        o = _view(own + c * slot_o, (Lq, B, Hq, D), q.device)
        lse = _view(own + buf.o_bytes + c * slot_lse, (B, Hq, Lq), q.device)
        _kernel.forward_bshd(q, kp, vp, o.transpose(0, 1), scale, causal, bias, lse=lse,
                             k_pos_offset=a, lk_total=lk_total)
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events["forward_done"] = ev
    _order(buf, group)  # every rank's partials are complete
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events["exchange_done"] = ev
    r0, r1 = row_shard(Lq, world, rank)
    out = torch.empty(max(r1 - r0, 0), B, Hq, D, device=q.device, dtype=out_dtype)
    o_ptrs = [buf.base[g] + c * slot_o for g in range(world) for c in range(nch)]
    lse_ptrs = [buf.base[g] + buf.o_bytes + c * slot_lse for g in range(world) for c in range(nch)]
    rc = _lib.lse_merge_rows(o_ptrs, lse_ptrs, Lq, r0, r1 - r0, BH, D, out.data_ptr(),
                             _kernel._DTYPES[out_dtype], None, stream)
    if rc != _lib.OK:
        _kernel._raise_status(rc, "mfa_lse_merge_rows")
    return out.transpose(0, 1), (r0, r1)


def flash_attn_split_kv(q, k_parts, v_parts, key_ranges, lk_total, softmax_scale=None,
                        causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                        group=None, out_dtype=None, gather=False, events=None, merge="auto"):
    """Attention of the full query set against keys spread over ranks.

    q: [B, Lq, Hq, D] (every rank); k_parts/v_parts: this rank's key chunks, each
    [B, n_i, Hkv, D], holding global key positions key_ranges[i] = (start, end) of lk_total.
    Returns (o_rows [B, r1 - r0, Hq, D] in out_dtype (default q.dtype), (r0, r1)): this rank's
    query rows of the merged output. With ``gather=True`` the rows of every rank are
    all-gathered and the full [B, Lq, Hq, D] output is returned on every rank instead.

    ``merge``: "pull" (each rank's forward writes its partials to its own buffer; each rank
    then merges its rows reading every rank's buffer through peer memory), "peer" (the forward
    scatters partial rows to their owners through peer memory, then a local merge), "nccl"
    (all-gather of the row log-sum-exp, rescale, reduce-scatter), or "auto": "pull" when the
    tensor-core kernel takes the inputs and the group has at most 8 ranks, else "nccl". With
    "pull" and "peer" every rank must pass the same number of key chunks."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    B, Lq, Hq, D = q.shape
    alibi = (_kernel._broadcast_alibi_slopes(alibi_slopes, B, Hq, q.device)
             if alibi_slopes is not None else None)
    bias = _kernel._BiasParams(softcap, window_size[0], window_size[1], alibi)
    world = dist.get_world_size(group)
    if merge == "auto":
        peer_ok = (q.is_cuda and world <= _lib.MAX_PEERS and q.shape[-1] % 8 == 0
                   and q.dtype in (torch.float16, torch.bfloat16))
        merge = "pull" if peer_ok else "nccl"
    if merge == "pull":
        out, rows = _split_kv_pull(q, k_parts, v_parts, key_ranges, lk_total, scale, causal,
                                   bias, group, out_dtype or q.dtype, events)
        return _gather_rows(out, rows, Lq, group) if gather else (out, rows)
    if merge == "peer":
        out, rows = _split_kv_peer(q, k_parts, v_parts, key_ranges, lk_total, scale, causal,
                                   bias, group, out_dtype or q.dtype, events)
        return _gather_rows(out, rows, Lq, group) if gather else (out, rows)
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
    return _gather_rows(out, (r0, r1), Lq, group) if gather else (out, (r0, r1))


def _gather_rows(out, rows, Lq, group):
    """All ranks' row blocks [B, r1 - r0, H, D] -> the full [B, Lq, H, D] on every rank."""
    r0, r1 = rows
    world = dist.get_world_size(group)
    per = -(-Lq // world)
    B, _, H, D = out.shape
    full = torch.zeros(world * per, B, H, D, device=out.device, dtype=out.dtype)
    mine = torch.zeros(per, B, H, D, device=out.device, dtype=out.dtype)
    mine[: r1 - r0] = out.transpose(0, 1)
    dist.all_gather_into_tensor(full, mine, group=group)
    return full[:Lq].transpose(0, 1).contiguous()
