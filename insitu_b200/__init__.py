"""insitu_b200: INSITU's compressed-KV decode attention, B200-native.

The hot path -- ingress (rotate, norm, codebook-quantise, bit-pack, paged
write) and the code-domain scan (scores on codes, fixed-point online softmax,
V accumulation, normalised reciprocal) -- is hand-written CUDA for sm_100a
behind the C ABI in ``include/insitu_b200.h``. This package mirrors the
reference's operator interfaces above it:

    Rotation            ops/rotate.py
    KVQuantizer         ops/quantize.py
    CompressedCache     cache/compressed.py   (KVCache, cache/base.py)
    CompressedAttention ops/attention.py
    DecodeAttention     the batched decode step below the seam (kernel.py:253-355)
    PagedCache          the C-ABI handle itself
"""

from .config import FixedFormat, Geometry, QuantConfig

__all__ = ["FixedFormat", "Geometry", "QuantConfig", "Rotation", "KVQuantizer", "CompressedKV",
           "KVCache", "CompressedCache", "CompressedAttention", "AttentionStats",
           "DecodeAttention", "PagedCache", "AttentionLayer"]


def __getattr__(name):
    # Lazy: importing the package must not require torch or a GPU (the CPU
    # tests and the build check import it on machines without either).
    if name == "Rotation":
        from .rotate import Rotation
        return Rotation
    if name in ("KVQuantizer", "CompressedKV"):
        from . import quantize
        return getattr(quantize, name)
    if name in ("KVCache", "CompressedCache"):
        from . import cache
        return getattr(cache, name)
    if name in ("CompressedAttention", "AttentionStats"):
        from . import attention
        return getattr(attention, name)
    if name == "AttentionLayer":
        from .layer import AttentionLayer
        return AttentionLayer
    if name == "DecodeAttention":
        from .decode import DecodeAttention
        return DecodeAttention
    if name == "PagedCache":
        from .engine import PagedCache
        return PagedCache
    raise AttributeError(name)
