"""The context split's orchestration over a process group, on CPU (gloo,
world size 2): each rank reports its maxima, receives the exclusive prefix
maximum of the ranks before it, and every rank merges the parts in rank
order. The device work is replaced by a recording fake; the arithmetic of the
split itself is tested on the GPU in test_context_split.py.
"""

from __future__ import annotations

import os

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist                                   # noqa: E402
import torch.multiprocessing as mp                                 # noqa: E402


class FakeShard:
    """Stands in for PagedCache: maxima depend on the rank, parts record the
    m_in they were given, merge returns the parts it received."""

    def __init__(self, rank):
        self.rank = rank

    def scan_maxima(self, seq_ids, q_rot, *, lengths=None):
        # (B=1, n_kv=2, groups=2); rank 0 has the larger maximum on head 0,
        # rank 1 on head 3
        m = torch.tensor([[[100, 5], [7, 1]]], dtype=torch.int64)
        if self.rank == 1:
            m = torch.tensor([[[50, 9], [3, 200]]], dtype=torch.int64)
        return m

    def scan_part(self, seq_ids, m_in, *, lengths=None):
        self.m_in = m_in.clone()
        return torch.tensor([self.rank, *m_in.flatten().tolist()], dtype=torch.int64)

    def merge_parts(self, parts, B, *, stats=True):
        return parts, None


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from insitu_b200.context import S_LO, context_split_scan
        shard = FakeShard(rank)
        parts, _ = context_split_scan(shard, [0], None)
        q.put((rank, shard.m_in.tolist(), parts.tolist(), S_LO))
    finally:
        dist.destroy_process_group()


def test_context_split_over_gloo_two_ranks():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, m_in, parts, s_lo = q.get(timeout=120)
        res[rank] = (m_in, parts, s_lo)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    s_lo = res[0][2]
    # rank 0 starts from nothing; rank 1 from rank 0's maxima
    assert res[0][0] == [[[s_lo, s_lo], [s_lo, s_lo]]]
    assert res[1][0] == [[[100, 5], [7, 1]]]
    # both ranks merge the same parts, in rank order
    want = [[0, s_lo, s_lo, s_lo, s_lo], [1, 100, 5, 7, 1]]
    assert res[0][1] == want and res[1][1] == want


def test_exclusive_prefix_max():
    from insitu_b200.context import S_LO, exclusive_prefix_max
    ms = [torch.tensor([3, -5]), torch.tensor([1, 9]), torch.tensor([4, 0])]
    assert exclusive_prefix_max(ms, 0).tolist() == [S_LO, S_LO]
    assert exclusive_prefix_max(ms, 1).tolist() == [3, -5]
    assert exclusive_prefix_max(ms, 2).tolist() == [3, 9]
