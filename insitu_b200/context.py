"""One sequence's decode-step scan across shards that each hold a causal range
of its cached tokens (the context split of benchmark config 5).

The reference scans a sequence in one process (``attend_online``,
ops/attention.py:451-513). Here shard r holds tokens [T_r, T_{r+1}) in its own
cache. The online recurrence crosses shards through one number per (item,
query head) -- the running maximum entering the shard -- and one composite
per item going the other way:

1. every shard scores its rows and reports its maximum (``scan_maxima``);
2. shard r's incoming maximum is the maximum over shards before it
   (``exclusive_prefix_max``);
3. every shard folds its rows into a composite given that maximum
   (``scan_part``);
4. the composites, in causal order, fold into the outputs (``merge_parts``):
   bit-exact with the single-process scan whenever the 32-bit accumulator
   clamp provably never fires (else the cache latches INS_ERANGE).

``context_split_scan`` runs steps 1-4 over a ``torch.distributed`` process
group (NCCL across GPUs: two all-gathers of a few KB per item);
``local_split_scan`` runs them for shards that are sequences of one cache, in
causal order, with no communication.
"""

from __future__ import annotations

import torch

S_LO = -(1 << 47)   # the running maximum before any token (48-bit scores)


def exclusive_prefix_max(maxima_by_shard, shard: int) -> torch.Tensor:
    """The running maximum entering ``shard``: the element-wise maximum of the
    maxima of shards 0 .. shard-1, or S_LO for the first shard."""
    ref = maxima_by_shard[0]
    m = torch.full_like(ref, S_LO)
    for r in range(shard):
        m = torch.maximum(m, maxima_by_shard[r].to(m.device))
    return m


PHASES = ("scores", "gather_maxima", "values", "gather_parts", "merge")


def context_split_scan(pc, seq_ids, q_rot, *, lengths=None, group=None, stats: bool = True,
                       events=None):
    """Steps 1-4 on every rank of ``group``; rank order is causal order. Every
    rank returns the merged (out, stats) for its ``seq_ids``. ``events``, a
    list of len(PHASES) + 1 CUDA events, is recorded between the phases
    (scores, all-gather of the maxima, values, all-gather of the composites,
    merge) on the current stream."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mark = (lambda i: events[i].record()) if events is not None else (lambda i: None)
    mark(0)
    maxima = pc.scan_maxima(seq_ids, q_rot, lengths=lengths)
    mark(1)
    gathered = torch.empty((world * maxima.shape[0], *maxima.shape[1:]), dtype=maxima.dtype,
                           device=maxima.device)
    dist.all_gather_into_tensor(gathered, maxima, group=group)
    gathered = gathered.view(world, *maxima.shape)
    mark(2)
    part = pc.scan_part(seq_ids, exclusive_prefix_max(gathered, rank), lengths=lengths)
    mark(3)
    parts = torch.empty((world * part.numel(),), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(parts, part, group=group)
    parts = parts.view(world, part.numel())
    mark(4)
    res = pc.merge_parts(parts, maxima.shape[0], stats=stats)
    mark(5)
    return res


def local_split_scan(pc, shard_seq_ids, q_rot, *, stats: bool = True):
    """Steps 1-4 for shards held as sequences of one cache: ``shard_seq_ids``
    lists, in causal order, one array of B sequence ids per shard (the b-th
    entries of all shards are the ranges of one sequence)."""
    maxima, parts = [], []
    for r, ids in enumerate(shard_seq_ids):
        maxima.append(pc.scan_maxima(ids, q_rot))
        parts.append(pc.scan_part(ids, exclusive_prefix_max(maxima, r)))
    return pc.merge_parts(torch.stack(parts), maxima[0].shape[0], stats=stats)
