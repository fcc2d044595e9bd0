"""``DecodeAttention``: the below-the-seam half of a decode step, batched.

For each sequence in a batch: rotate q, k, v; quantise and append k, v; scan
the whole compressed cache for every KV head and every query head of its
group; return Q(acc_frac) outputs in merge_heads order. This is
kernel.py:253-355 (the part the FPGA runs) for B sequences at once, as one
ingress launch and one scan launch.
"""

from __future__ import annotations

import numpy as np
import torch

from .config import FixedFormat, Geometry, QuantConfig
from .engine import PagedCache


class DecodeAttention:
    def __init__(self, quant: QuantConfig, fmt: FixedFormat | None = None,
                 geo: Geometry | None = None, *, max_seqs: int = 1, capacity: int = 4096,
                 page_tokens: int = 256, device=None):
        self.pc = PagedCache(quant, fmt, geo, max_seqs=max_seqs, capacity=capacity,
                             page_tokens=page_tokens, device=device)
        self.geo = self.pc.geo

    @property
    def row_bytes(self) -> int:
        return self.pc.row_bytes

    def prefill(self, seq: int, k, v, chunk: int = 1 << 18) -> None:
        """Append n tokens of one sequence without attending (fills a cache)."""
        n = k.shape[0]
        for lo in range(0, n, chunk):
            hi = min(n, lo + chunk)
            self.pc.ingress(np.full(hi - lo, seq, np.int32), k[lo:hi], v[lo:hi])

    def step(self, q, k, v, seq_ids=None, *, mode: str = "online", out=None, stats_out=None):
        """One decode token per sequence: q (B, Hq, d), k/v (B, n_kv, d) int32.

        Returns (out (B, Hq, d) int64, stats (B, n_kv, 6) int64), both on the
        device. The new token is appended before the scan, so it attends to
        itself (the causality note of hw/vectors.py:22-30).
        """
        B = q.shape[0]
        ids = list(range(B)) if seq_ids is None else seq_ids
        if out is None and stats_out is None:
            return self.pc.step(ids, q, k, v, mode=mode)
        q_rot = self.pc.ingress(ids, k, v, q)
        return self.pc.scan(ids, q_rot, mode=mode, out=out, stats_out=stats_out)

    def prefill_attend(self, seq: int, q, k, v, *, mode: str = "online"):
        """A prefill chunk of one sequence: append its n tokens (one ingress
        launch), then every token attends the cache up to and including
        itself (one scan launch, the sequence entered n times with causal
        lengths) -- the attend_online_batch / attend_causal_batch of
        ops/attention.py:517-871 for all KV heads. q (n, Hq, d), k/v (n, n_kv,
        d) int32. Returns out (n, Hq, d) and stats (n, n_kv, 6)."""
        n = k.shape[0]
        base = self.pc.length(seq)
        q_rot = self.pc.ingress([seq] * n, k, v, q)
        return self.pc.scan([seq] * n, q_rot, lengths=base + 1 + np.arange(n), mode=mode)

    @staticmethod
    def merge_heads(out: torch.Tensor) -> torch.Tensor:
        """(B, heads, d) -> (B, heads*d), ops/project.py:67-74."""
        return out.reshape(out.shape[0], -1)

    def close(self) -> None:
        self.pc.close()
