"""The fixed-point contract and the cache geometry.

Mirrors the reference's ``QuantConfig`` and ``FixedFormat`` (INSITU
``config.py:132-254``): same field names, same defaults, same derived shifts,
so a caller holding the reference's config objects can build this one from
them field by field (``from_reference``). Only the fields the hot path reads
are kept; the hardware-cycle model (``HardwareConfig``) has no role on a GPU.
"""

from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class QuantConfig:
    """Rotate-then-quantize parameters for one KV head (config.py:132-207)."""

    key_bits: int = 3
    value_bits: int = 2
    norm_bits: int = 16
    norm_frac: int = 9
    seed: int = 0
    symmetric: bool = True
    rot_rounds: int = 1
    codebook: str = "gaussian"

    def __post_init__(self) -> None:
        for name, b in (("key_bits", self.key_bits), ("value_bits", self.value_bits)):
            if not 1 <= b <= 8:
                raise ValueError(f"{name}={b} outside the supported range 1..8")
        if self.rot_rounds < 0:
            raise ValueError(f"rot_rounds={self.rot_rounds} must not be negative")
        if self.codebook not in ("gaussian", "uniform"):
            raise ValueError(f"codebook={self.codebook!r}; expected gaussian or uniform")
        if self.norm_frac >= self.norm_bits:
            raise ValueError(f"norm_frac={self.norm_frac} leaves no integer bits in "
                             f"norm_bits={self.norm_bits}")
        if self.norm_bits % 8:
            raise ValueError(f"norm_bits={self.norm_bits} is not whole bytes")

    def bytes_per_token(self, head_dim: int) -> int:
        """Compressed bytes per (token, KV head) (config.py:192-207)."""
        code_bits = head_dim * (self.key_bits + self.value_bits)
        if code_bits % 8:
            raise ValueError(
                f"head_dim*(key_bits+value_bits) = {code_bits} is not a whole number of "
                f"bytes; choose widths summing to a multiple of {8 // math.gcd(8, head_dim)}")
        return code_bits // 8 + 2 * (self.norm_bits // 8)


@dataclass(frozen=True)
class FixedFormat:
    """Q-format widths downstream of the float->fixed cast (config.py:214-254)."""

    qk_frac: int = 16
    qk_width: int = 24
    centroid_frac: int = 15
    acc_frac: int = 16
    acc_width: int = 32
    score_width: int = 48
    prob_frac: int = 15
    prob_width: int = 16
    exp_lut_bits: int = 8
    saturate: bool = True
    recip_norm_bits: int = 32

    def score_shift_for(self, quant: QuantConfig) -> int:
        return self.qk_frac + self.centroid_frac + quant.norm_frac - self.acc_frac

    def acc_shift_for(self, quant: QuantConfig) -> int:
        return self.centroid_frac + quant.norm_frac + self.prob_frac - self.acc_frac


@dataclass(frozen=True)
class Geometry:
    """Attention shape below the seam: KV heads, the GQA group, head_dim.

    The reference derives these from ``ModelConfig`` (config.py:33-125); the
    hot path needs only the three numbers. Llama-3.2-1B is 8 KV heads, 4 query
    heads per group, d = 64.
    """

    n_kv_heads: int = 8
    kv_groups: int = 4
    head_dim: int = 64

    def __post_init__(self) -> None:
        d = self.head_dim
        if d & (d - 1) or d < 2:
            raise ValueError(f"head_dim={d} must be a power of two (Walsh-Hadamard butterfly)")
        if d > 256:
            raise ValueError(f"head_dim={d} above the 256 this build supports")
        if self.n_kv_heads < 1 or self.kv_groups < 1:
            raise ValueError("need at least one KV head and one query head per group")

    @property
    def num_heads(self) -> int:
        return self.n_kv_heads * self.kv_groups


def from_reference(quant, fmt=None) -> tuple[QuantConfig, FixedFormat]:
    """Copy the reference's QuantConfig / FixedFormat objects field by field."""
    q = QuantConfig(**{f: getattr(quant, f) for f in QuantConfig.__dataclass_fields__})
    if fmt is None:
        return q, FixedFormat()
    return q, FixedFormat(**{f: getattr(fmt, f) for f in FixedFormat.__dataclass_fields__
                             if hasattr(fmt, f)})
