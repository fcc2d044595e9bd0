"""``CompressedAttention``: scores, online and two-pass softmax on the codes
(ops/attention.py:257-513), on the GPU.

``kv`` may be a ``DeviceKV`` from this package's ``CompressedCache`` (scanned
in place) or a host ``CompressedKV`` (uploaded into a scratch cache first, so
the reference's own arrays can be fed to the GPU kernels unchanged).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .cache import DeviceKV
from .config import FixedFormat, Geometry, QuantConfig
from .quantize import CompressedKV, KVQuantizer


@dataclass
class AttentionStats:
    """What the step did (ops/attention.py:257-274)."""

    n_tokens: int = 0
    rescale_events: int = 0
    score_overflows: int = 0
    acc_overflows: int = 0
    max_abs_score: int = 0
    max_abs_acc: int = 0

    def merge(self, other: "AttentionStats") -> None:
        self.n_tokens = max(self.n_tokens, other.n_tokens)
        self.rescale_events += other.rescale_events
        self.score_overflows += other.score_overflows
        self.acc_overflows += other.acc_overflows
        self.max_abs_score = max(self.max_abs_score, other.max_abs_score)
        self.max_abs_acc = max(self.max_abs_acc, other.max_abs_acc)

    @staticmethod
    def from_row(row) -> "AttentionStats":
        return AttentionStats(*(int(x) for x in row))


class CompressedAttention:
    """Scores and accumulates directly on codes, for one KV head's cache."""

    def __init__(self, quantizer: KVQuantizer, fmt: FixedFormat | None = None,
                 quant: QuantConfig | None = None) -> None:
        self.z = quantizer
        self.fmt = fmt or quantizer.fmt
        self.quant = quant or quantizer.quant
        self.score_shift = self.fmt.score_shift_for(self.quant)
        self.acc_shift = self.fmt.acc_shift_for(self.quant)
        self.score_mode = "fused"
        self._scratch = {}

    # -- where the rows come from ------------------------------------------------
    def _resident(self, kv, heads: int):
        """(PagedCache, kv_head, length) holding kv's rows for a group of `heads`."""
        if isinstance(kv, DeviceKV):
            pc = kv.cache.pc
            if pc.geo.kv_groups != heads:
                raise ValueError(f"this cache scores {pc.geo.kv_groups} query heads per KV "
                                 f"head; got {heads}")
            return pc, kv.kv_head, kv.length
        if not isinstance(kv, CompressedKV):
            raise TypeError("kv must be a DeviceKV or a CompressedKV")
        rows = self.z.pack(kv).reshape(-1, 1, self.z.bytes_per_token)
        T = rows.shape[0]
        from .engine import PagedCache
        key = (heads, T)
        pc = self._scratch.get(key)
        if pc is None:
            cap = max(256, 1 << max(0, T - 1).bit_length())
            pc = PagedCache(self.quant, self.fmt, Geometry(1, heads, self.z.d), max_seqs=1,
                            capacity=cap, device=self.z.device)
            self._scratch = {key: pc}
        pc.reset(0)
        pc.import_rows(0, rows)
        return pc, 0, T

    @staticmethod
    def _heads(q_rot):
        q = np.asarray(q_rot if not isinstance(q_rot, torch.Tensor) else q_rot.cpu())
        return np.atleast_2d(q).astype(np.int64)

    # -- scoring -------------------------------------------------------------
    def scores(self, q_rot, kv, trace=None):
        """All scores for the query heads against T cached tokens, Q(acc_frac)."""
        q = self._heads(q_rot)
        pc, head, T = self._resident(kv, q.shape[0])
        s, ovf = pc.scores(0, head, torch.from_numpy(q.astype(np.int32)), 0, T)
        pc.status()
        out = s.cpu().numpy()
        return out.reshape(np.shape(q_rot)[:-1] + (T,)), int(ovf.item())

    # -- the two softmaxes -------------------------------------------------------
    def _attend(self, q_rot, kv, mode):
        q = self._heads(q_rot)
        pc, head, T = self._resident(kv, q.shape[0])
        g = pc.geo
        # One KV head of one sequence: place the group's query at its KV head.
        full = torch.zeros((1, g.num_heads, g.head_dim), dtype=torch.int32)
        full[0, head * g.kv_groups:(head + 1) * g.kv_groups] = torch.from_numpy(
            q.astype(np.int32))
        out, st = pc.scan([0], full, lengths=[T], mode=mode)
        pc.status()
        y = out[0, head * g.kv_groups:(head + 1) * g.kv_groups].cpu().numpy()
        stats = AttentionStats.from_row(st[0, head].cpu().numpy())
        return y.reshape(np.shape(q_rot)), stats

    def _attend_batch(self, q_rot, kv, base, mode):
        """Query i of a prefill against cached tokens [0, base + i]: one scan
        launch, the sequence entered once per query with its causal length."""
        q = np.asarray(q_rot if not isinstance(q_rot, torch.Tensor) else q_rot.cpu()).astype(np.int64)
        if q.ndim == 2:
            q = q[:, None, :]
        n, heads = q.shape[0], q.shape[1]
        pc, head, T = self._resident(kv, heads)
        lengths = base + 1 + np.arange(n, dtype=np.int64)
        if n and lengths[-1] > T:
            raise ValueError(f"query {n - 1} attends token {lengths[-1] - 1}; the cache holds {T}")
        g = pc.geo
        full = torch.zeros((n, g.num_heads, g.head_dim), dtype=torch.int32)
        full[:, head * g.kv_groups:(head + 1) * g.kv_groups] = torch.from_numpy(q.astype(np.int32))
        out, st = pc.scan([0] * n, full, lengths=lengths, mode=mode)
        pc.status()
        y = out[:, head * g.kv_groups:(head + 1) * g.kv_groups].cpu().numpy()
        rows = st[:, head].cpu().numpy()
        stats = AttentionStats.from_row(rows[0]) if n else AttentionStats()
        for r in rows[1:]:
            stats.merge(AttentionStats.from_row(r))
        return y.reshape(np.shape(q_rot)), stats

    def attend_online_batch(self, q_rot, kv, base: int = 0, trace=None):
        """attend_online for every query token of a prefill (ops/attention.py:
        794-871): query i attends cached tokens [0, base + i]. Outputs are the
        per-token loop's, as the reference pins its batch form to; the
        statistics are the per-token ones merged (AttentionStats.merge)."""
        if self.score_mode != "fused":
            raise ValueError("attend_online_batch runs the fused (architecture B) path only")
        return self._attend_batch(q_rot, kv, base, "online")

    def attend_causal_batch(self, q_rot, kv, base: int = 0, tile: int = 256, trace=None):
        """attend_two_pass for every query token of a prefill
        (ops/attention.py:517-670), causal as attend_online_batch."""
        return self._attend_batch(q_rot, kv, base, "two_pass")

    def attend_online(self, q_rot, kv, trace=None):
        """One streaming pass with a running maximum (ops/attention.py:451-513)."""
        if self.score_mode != "fused":
            raise ValueError("attend_online runs the fused (architecture B) path only")
        return self._attend(q_rot, kv, "online")

    def attend_two_pass(self, q_rot, kv, trace=None):
        """Global maximum, then one accumulation (ops/attention.py:429-449)."""
        return self._attend(q_rot, kv, "two_pass")
