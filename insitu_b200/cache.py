"""The cache interface (cache/base.py) and its GPU implementation
(cache/compressed.py).

``CompressedCache`` has the reference's constructor, ``append_rotated``,
``view``, ``view_from_buffer``, ``reset``, ``bytes_per_token`` and ``stats``,
so ``kernel.py`` can construct it in place of the numpy one. The packed codes
live in a paged HBM pool; there is no decoded host shadow. ``view`` returns a
``DeviceKV`` -- a handle to one KV head's causal prefix on the device -- which
``CompressedAttention`` scans in place and which materialises a host
``CompressedKV`` only when asked for its arrays.
"""

from __future__ import annotations

import abc

import numpy as np

from .config import FixedFormat, Geometry, QuantConfig
from .quantize import CompressedKV, KVQuantizer


class KVCache(abc.ABC):
    """Per-layer, per-KV-head storage for one sequence (cache/base.py:29-81)."""

    def __init__(self, n_kv_heads: int, head_dim: int, capacity: int) -> None:
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.capacity = capacity
        self.length = 0

    @property
    @abc.abstractmethod
    def bytes_per_token(self) -> int:
        """One token, all KV heads."""

    @abc.abstractmethod
    def append(self, k, v, positions, trace=None) -> None:
        """Store (tokens, n_kv_heads, head_dim) of post-RoPE K and V."""

    @abc.abstractmethod
    def view(self, kv_head: int, trace=None):
        """Everything stored for one KV head, in causal order."""

    def reset(self) -> None:
        self.length = 0

    def _check_room(self, n: int) -> None:
        if self.length + n > self.capacity:
            raise ValueError(
                f"cache holds {self.length} of {self.capacity} tokens; cannot append {n}. "
                f"Grow `capacity` at construction -- growing here would hide a reallocation "
                f"inside a decode step.")

    def stats(self) -> dict:
        return {"tokens": self.length, "capacity": self.capacity,
                "bytes_per_token": self.bytes_per_token,
                "bytes_resident": self.length * self.bytes_per_token}


class DeviceKV:
    """One KV head's first ``length`` cached tokens, resident on the GPU.

    Behaves like ``CompressedKV`` where the reference's code reads it
    (``select``, ``n_tokens``, the four arrays), but the arrays are copied off
    the device only on first access -- the scan never needs them.
    """

    def __init__(self, cache: "CompressedCache", kv_head: int, length: int):
        self.cache, self.kv_head, self.length = cache, kv_head, length
        self._host = None

    @property
    def n_tokens(self) -> int:
        return self.length

    def select(self, sl):
        if isinstance(sl, slice) and sl.step in (None, 1) and (sl.start in (None, 0)):
            stop = self.length if sl.stop is None else sl.stop
            stop = max(0, min(self.length, stop if stop >= 0 else self.length + stop))
            return DeviceKV(self.cache, self.kv_head, stop)
        return self.host().select(sl)

    def host(self) -> CompressedKV:
        if self._host is None:
            rows = self.cache.pc.export(0, self.kv_head, 0, self.length)
            self._host = self.cache.quantizer.unpack(rows)
        return self._host

    @property
    def k_idx(self):
        return self.host().k_idx

    @property
    def k_norm(self):
        return self.host().k_norm

    @property
    def v_idx(self):
        return self.host().v_idx

    @property
    def v_norm(self):
        return self.host().v_norm


class CompressedCache(KVCache):
    """Codes and norms in the rotated space, in a paged HBM pool (one sequence)."""

    def __init__(self, n_kv_heads: int, head_dim: int, capacity: int, quant: QuantConfig,
                 fmt: FixedFormat | None = None, qk_frac: int | None = None, *,
                 kv_groups: int = 4, page_tokens: int = 256, device=None) -> None:
        super().__init__(n_kv_heads, head_dim, capacity)
        from .engine import PagedCache
        fmt = fmt or FixedFormat()
        self.fmt = fmt
        self.quantizer = KVQuantizer(head_dim, quant, fmt, device=device)
        self._row = self.quantizer.bytes_per_token
        self.pc = PagedCache(quant, fmt, Geometry(n_kv_heads, kv_groups, head_dim),
                             max_seqs=1, capacity=capacity, page_tokens=page_tokens,
                             device=device)

    @property
    def bytes_per_token(self) -> int:
        return self._row * self.n_kv_heads

    def append_rotated(self, k_rot, v_rot, trace=None) -> None:
        """Store K and V that are already rotated and in Q(qk_frac)."""
        k = np.asarray(k_rot) if not hasattr(k_rot, "device") else k_rot
        n = k.shape[0]
        self._check_room(n)
        self.pc.ingress(np.zeros(n, np.int32), k_rot, v_rot, prerotated=True)
        self.pc.status()
        self.length += n

    def append_wire(self, k, v, q=None):
        """The fused ingress: rotate and append wire-format k/v; rotate q too.

        The GPU fusion of kernel.py:271-284. Returns the rotated q or None.
        """
        n = k.shape[0]
        self._check_room(n)
        q_rot = self.pc.ingress(np.zeros(n, np.int32), k, v, q)
        self.length += n
        return q_rot

    def append(self, k, v, positions, trace=None) -> None:
        raise NotImplementedError(
            "CompressedCache stores rotated tokens; call append_rotated (or append_wire).")

    def view(self, kv_head: int, trace=None, n_reads: int = 1) -> DeviceKV:
        return DeviceKV(self, kv_head, self.length)

    def view_from_buffer(self, kv_head: int) -> CompressedKV:
        """The same view decoded from the packed bytes the device holds."""
        return self.quantizer.unpack(self.pc.export(0, kv_head, 0, self.length))

    @property
    def buf(self) -> np.ndarray:
        """The packed rows, (length, n_kv_heads, row_bytes), copied from the device."""
        rows = [self.pc.export(0, h, 0, self.length) for h in range(self.n_kv_heads)]
        return np.stack(rows, axis=1) if rows else np.zeros((0, 0, self._row), np.uint8)

    def reset(self) -> None:
        super().reset()
        self.pc.reset(0)
