"""Host codecs of the board's byte formats around the cache (no device work).

* The 24-bit lane stream: signed integers packed LSB first, ``bits`` each
  (``pack_lanes`` / ``unpack_lanes``, hw/vectors.py:72-104), and the ingress
  stream of a decode token built from them: per KV head h the vectors k_h,
  v_h, q_{h*groups} .. q_{h*groups+groups-1} (``VectorSet.ingress_groups``,
  hw/vectors.py:178-196). ``PagedCache.ingress_lanes`` takes this stream on
  the device.
* The DDR image of a cache (``DdrLayout``, hw/ddr_layout.py): how many bytes
  ``PagedCache.ddr_image`` writes, and ``row_at`` to read a row back out of an
  image on the host.
"""

from __future__ import annotations

import numpy as np

BEAT_BYTES = 16
PAGE = 4096


def pack_lanes(values, bits: int = 24) -> bytes:
    """Signed integers -> LSB-first packed bytes; the last byte zero-padded."""
    v = np.asarray(values, dtype=np.int64).reshape(-1)
    if bits <= 0:
        raise ValueError(f"bits={bits} must be positive")
    mask = (1 << bits) - 1
    acc = 0
    for i, x in enumerate(v):
        acc |= (int(x) & mask) << (i * bits)
    return acc.to_bytes((v.size * bits + 7) // 8, "little")


def unpack_lanes(buf: bytes, bits: int, count: int) -> np.ndarray:
    """The inverse of pack_lanes, sign-extended."""
    acc = int.from_bytes(bytes(buf), "little")
    mask, sign = (1 << bits) - 1, 1 << (bits - 1)
    return np.array([(((acc >> (i * bits)) & mask) ^ sign) - sign for i in range(count)],
                    dtype=np.int64)


def ingress_stream(q, k, v, bits: int = 24) -> np.ndarray:
    """The board's ingress stream of n tokens: q (n, n_kv*groups, d), k and v
    (n, n_kv, d) -> uint8 bytes, token after token."""
    q, k, v = (np.asarray(x, dtype=np.int64) for x in (q, k, v))
    n, n_kv = k.shape[0], k.shape[1]
    groups = q.shape[1] // n_kv
    out = []
    for t in range(n):
        for h in range(n_kv):
            grp = np.concatenate([k[t, h][None], v[t, h][None], q[t, h * groups:(h + 1) * groups]])
            out.append(pack_lanes(grp, bits))
    return np.frombuffer(b"".join(out), dtype=np.uint8).copy()


def ddr_planes(row_fields):
    """(lo, width) of every plane: the fields split into 16-byte beats."""
    planes = []
    for lo, hi in row_fields:
        a = lo
        while a < hi:
            b = min(a + BEAT_BYTES, hi)
            if (b - a) > BEAT_BYTES or BEAT_BYTES % (b - a):
                raise ValueError("a plane is neither a beat nor a whole fraction of one")
            planes.append((a, b - a))
            a = b
    return planes


def ddr_span(planes, capacity: int) -> int:
    raw = capacity * max(w for _, w in planes)
    return (raw + PAGE - 1) // PAGE * PAGE


def row_at(img, planes, capacity: int, head: int, token: int) -> np.ndarray:
    """One packed row reassembled from a DDR image."""
    img = np.asarray(img, dtype=np.uint8)
    span = ddr_span(planes, capacity)
    parts = []
    for p, (_, w) in enumerate(planes):
        a = (head * len(planes) + p) * span + token * w
        parts.append(img[a:a + w])
    return np.concatenate(parts)
