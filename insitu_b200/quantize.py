"""The quantiser's interface: ``CompressedKV``, ``KVQuantizer`` (ops/quantize.py).

``encode`` runs on the GPU (the ingress kernel's norm, threshold encode and
bit-pack, reached through a small utility cache). ``pack`` / ``unpack`` are
the row codec of the reference's wire format (ops/quantize.py:237-296), kept on
the host because they convert between the device cache and host bytes; they
compute nothing the scan needs.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass

import numpy as np

from .config import FixedFormat, Geometry, QuantConfig
from .rotate import Rotation
from .tables import codebook


@dataclass(frozen=True)
class CompressedKV:
    """One KV head's compressed tokens (ops/quantize.py:99-118)."""

    k_idx: np.ndarray     # (..., d) uint8 codes
    k_norm: np.ndarray    # (...,) int64, Q(norm_frac)
    v_idx: np.ndarray
    v_norm: np.ndarray

    @property
    def n_tokens(self) -> int:
        return int(np.prod(self.k_idx.shape[:-1])) if self.k_idx.ndim > 1 else 1

    def select(self, sl) -> "CompressedKV":
        return CompressedKV(self.k_idx[sl], self.k_norm[sl], self.v_idx[sl], self.v_norm[sl])


@dataclass(frozen=True)
class Plane:
    """One quantised field (ops/quantize.py:63-96)."""

    name: str
    bits: int
    centroids: np.ndarray
    boundaries: np.ndarray
    d: int
    qk_frac: int
    norm_frac: int
    centroid_frac: int

    @property
    def threshold_frac(self) -> int:
        return self.centroid_frac + self.norm_frac

    @property
    def code_bytes(self) -> int:
        total = self.d * self.bits
        if total % 8:
            raise ValueError(f"plane {self.name}: {self.d}*{self.bits} bits is not whole bytes")
        return total // 8


# The row format (ops/quantize.py:237-264): a field of d codes of `bits` bits
# is the little-endian integer sum(code_j << (bits * j)) in d * bits / 8
# bytes, and a norm is a little-endian two's-complement integer of norm_bits.
# Eight consecutive codes fill exactly `bits` bytes, so each group of eight is
# assembled as one 64-bit word (the ingress kernel packs 32-bit words the same
# way) and its low `bits` bytes are kept.

def _pack_codes(idx: np.ndarray, bits: int) -> np.ndarray:
    idx = np.asarray(idx)
    d = idx.shape[-1]
    groups = idx.astype(np.uint64).reshape(*idx.shape[:-1], d // 8, 8)
    words = (groups << (np.uint64(bits) * np.arange(8, dtype=np.uint64))).sum(axis=-1, dtype=np.uint64)
    raw = words.astype("<u8").view(np.uint8).reshape(*words.shape, 8)
    return np.ascontiguousarray(raw[..., :bits]).reshape(*idx.shape[:-1], d // 8 * bits)


def _unpack_codes(buf: np.ndarray, bits: int, d: int) -> np.ndarray:
    buf = np.asarray(buf, dtype=np.uint8)
    lead = buf.shape[:-1]
    raw = np.zeros((*lead, d // 8, 8), dtype=np.uint8)
    raw[..., :bits] = buf.reshape(*lead, d // 8, bits)
    words = raw.view("<u8")                     # (..., d // 8, 1)
    codes = (words >> (np.uint64(bits) * np.arange(8, dtype=np.uint64))) & np.uint64((1 << bits) - 1)
    return codes.astype(np.uint8).reshape(*lead, d)


def _pack_word(x: np.ndarray, bits: int) -> np.ndarray:
    nb = bits // 8
    raw = np.asarray(x, dtype=np.int64).astype("<i8").view(np.uint8)
    return np.ascontiguousarray(raw.reshape(*np.shape(x), 8)[..., :nb])


def _unpack_word(buf: np.ndarray, bits: int) -> np.ndarray:
    buf = np.asarray(buf, dtype=np.uint8)
    raw = np.zeros((*buf.shape[:-1], 8), dtype=np.uint8)
    raw[..., :bits // 8] = buf
    v = raw.view("<i8")[..., 0]
    # two's complement of `bits` bits: the top bit of the field carries -2^(bits-1)
    return v - (((v >> (bits - 1)) & 1) << bits)


class KVQuantizer:
    """A rotation, two codebooks and the wire format (ops/quantize.py:121-264)."""

    def __init__(self, d: int, quant: QuantConfig, fmt: FixedFormat | None = None,
                 device=None) -> None:
        fmt = fmt or FixedFormat()
        self.d, self.quant, self.fmt, self.device = d, quant, fmt, device
        self.rotation = Rotation.for_quant(quant, d, device=device)
        kc, kb = codebook(quant.codebook, quant.key_bits, fmt.centroid_frac, quant.symmetric)
        vc, vb = codebook(quant.codebook, quant.value_bits, fmt.centroid_frac, quant.symmetric)
        self.key = Plane("key", quant.key_bits, kc, kb, d, fmt.qk_frac, quant.norm_frac,
                         fmt.centroid_frac)
        self.value = Plane("value", quant.value_bits, vc, vb, d, fmt.qk_frac, quant.norm_frac,
                           fmt.centroid_frac)
        if self.key.threshold_frac < fmt.qk_frac:
            raise ValueError(
                f"centroid_frac + norm_frac = {self.key.threshold_frac} is below qk_frac = "
                f"{fmt.qk_frac}; the threshold comparison would have to truncate x")

    @property
    def bytes_per_token(self) -> int:
        return self.key.code_bytes + self.value.code_bytes + 2 * (self.quant.norm_bits // 8)

    def encode(self, k_rot, v_rot, trace=None) -> CompressedKV:
        """Already-rotated K and V -> codes and norms, on the GPU."""
        k = np.asarray(k_rot, dtype=np.int64)
        v = np.asarray(v_rot, dtype=np.int64)
        if k.shape != v.shape or k.shape[-1] != self.d:
            raise ValueError(f"k_rot {k.shape} and v_rot {v.shape} must match (..., {self.d})")
        lead = k.shape[:-1]
        n = int(np.prod(lead)) if lead else 1
        rows = _encode_rows(self.quant, self.fmt, self.d, k.reshape(n, self.d),
                            v.reshape(n, self.d), self.device)
        kv = self.unpack(rows)
        return CompressedKV(kv.k_idx.reshape(*lead, self.d), kv.k_norm.reshape(lead),
                            kv.v_idx.reshape(*lead, self.d), kv.v_norm.reshape(lead))

    def pack(self, kv: CompressedKV) -> np.ndarray:
        parts = [_pack_codes(kv.k_idx, self.key.bits), _pack_codes(kv.v_idx, self.value.bits),
                 _pack_word(kv.k_norm, self.quant.norm_bits),
                 _pack_word(kv.v_norm, self.quant.norm_bits)]
        return np.concatenate(parts, axis=-1)

    def unpack(self, buf: np.ndarray) -> CompressedKV:
        buf = np.asarray(buf, dtype=np.uint8)
        nb = self.quant.norm_bits // 8
        kb, vb = self.key.code_bytes, self.value.code_bytes
        if buf.shape[-1] != self.bytes_per_token:
            raise ValueError(f"expected {self.bytes_per_token} B per token, got {buf.shape[-1]}")
        o = 0
        k_idx = _unpack_codes(buf[..., o:o + kb], self.key.bits, self.d); o += kb
        v_idx = _unpack_codes(buf[..., o:o + vb], self.value.bits, self.d); o += vb
        k_norm = _unpack_word(buf[..., o:o + nb], self.quant.norm_bits); o += nb
        v_norm = _unpack_word(buf[..., o:o + nb], self.quant.norm_bits)
        return CompressedKV(k_idx, k_norm, v_idx, v_norm)


@functools.lru_cache(maxsize=16)
def utility_cache(quant: QuantConfig, fmt: FixedFormat, device_index: int, capacity: int):
    """A one-sequence, one-KV-head cache the utility entry points run through."""
    from .engine import PagedCache
    return PagedCache(quant, fmt, Geometry(n_kv_heads=1, kv_groups=1, head_dim=64),
                      max_seqs=1, capacity=capacity, device=device_index)


def _device_index(device) -> int:
    import torch
    if device is None:
        return torch.cuda.current_device()
    return torch.device("cuda", device).index if not isinstance(device, torch.device) \
        else device.index


def _encode_rows(quant, fmt, d, k, v, device) -> np.ndarray:
    """Rotated k/v (n, d) -> packed rows (n, row_bytes) through the ingress kernel."""
    chunk = 1 << 16
    pc = utility_cache(quant, fmt, _device_index(device), chunk)
    out = []
    for lo in range(0, k.shape[0], chunk):
        hi = min(lo + chunk, k.shape[0])
        pc.reset(0)
        pc.ingress(np.zeros(hi - lo, np.int32), k[lo:hi, None, :], v[lo:hi, None, :],
                   prerotated=True)
        pc.status()
        out.append(pc.export(0, 0))
    pc.reset(0)
    return np.concatenate(out) if out else np.zeros((0, quant.bytes_per_token(d)), np.uint8)
