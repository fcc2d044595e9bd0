"""The host half of a decode step on the GPU (kernel.py:197-249), up to the
wire: projections, QK-norm, the attention scale, RoPE and the Q8.16 cast.

* The projections are plain GEMMs and run as library GEMMs: fp16-rounded
  weights and activations, fp32 products and fp32 accumulation
  (numerics/fp.py:25-46, ``matvec``). Their accumulation order is the
  library's, so they match the reference within float32 rounding, not bit for
  bit -- as the reference's own note on ``matvec`` expects of any order.
* Everything after them is ``ins_seam`` (one kernel), bit-exact with the
  reference given the same projection outputs: rms_norm in float32 with
  numpy's summation order, the scale in float64, RoPE in float64 or in fixed
  point, round-half-even saturating cast.

The RoPE tables are built here on the host, by the reference's own recipe
(ops/rope.py:131-148, llama3 scaling ops/rope.py:98-109): the integers are
the format, like the codebooks.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .engine import PagedCache, _ptr, _stream


@dataclass(frozen=True)
class RopeScaling:
    """Llama 3's rescaling of the RoPE frequencies (ops/rope.py:48-109)."""
    factor: float
    low_freq_factor: float
    high_freq_factor: float
    original_max_position: int

    def apply(self, inv_freq: np.ndarray) -> np.ndarray:
        # Frequencies whose wavelength exceeds original_max_position /
        # low_freq_factor are divided by `factor`; those below
        # original_max_position / high_freq_factor are kept; in between they
        # blend linearly in original_max_position / wavelength. The float64
        # operations are those of the reference, in its order, because the
        # RoPE tables built from them are integers of the wire format.
        freq = np.asarray(inv_freq, dtype=np.float64)
        span = float(self.original_max_position)
        period = 2.0 * np.pi / freq
        long_edge, short_edge = span / self.low_freq_factor, span / self.high_freq_factor
        base = np.where(period > long_edge, freq / self.factor, freq)
        t = (span / period - self.low_freq_factor) / (self.high_freq_factor - self.low_freq_factor)
        blend = (1.0 - t) * base / self.factor + t * base
        mid = (period <= long_edge) & (period >= short_edge)
        return np.where(mid, blend, base)


def rope_tables(d: int, max_position: int, theta: float = 10000.0, frac: int = 15,
                scaling: RopeScaling | None = None):
    """(cos, sin): int64 [max_position, d/2] in Q(32, frac), round half even."""
    if d % 2:
        raise ValueError(f"head_dim={d} must be even")
    half = d // 2
    inv = 1.0 / (theta ** (np.arange(0, half, dtype=np.float64) * 2.0 / d))
    if scaling is not None:
        inv = scaling.apply(inv)
    ang = np.arange(max_position, dtype=np.float64)[:, None] * inv[None, :]
    lim = (1 << 31) - 1
    q = lambda x: np.clip(np.rint(x * (1 << frac)).astype(np.int64), -lim - 1, lim)
    return q(np.cos(ang)), q(np.sin(ang))


def project(w: torch.Tensor, x: torch.Tensor, bias: torch.Tensor | None = None, *,
            rounded: bool = False) -> torch.Tensor:
    """``matvec`` (numerics/fp.py:25-46) on the GPU through this library's
    projection kernel (ins_project): fp16-rounded operands, exact fp32
    products, fp32 sums. w (out, in): float16, or float32 to be rounded to
    fp16 (``rounded``: already fp16-exact, converted without change);
    x (n, in) -> (n, out) fp32."""
    from . import _lib
    w16 = w if w.dtype == torch.float16 else w.to(torch.float16)
    x32 = x.to(torch.float32).contiguous()
    b = None if bias is None else bias.to(device=x32.device, dtype=torch.float32).contiguous()
    return _lib.ops().project(w16.contiguous(), x32, b)


class Seam:
    """The seam of one layer on the cache's GPU."""

    def __init__(self, pc: PagedCache, *, max_position: int = 4096, theta: float = 10000.0,
                 scaling: RopeScaling | None = None, rope_frac: int = 15, q_norm=None, k_norm=None,
                 norm_eps: float = 1e-6, cast_after_rope: bool = True):
        self.pc = pc
        d = pc.geo.head_dim
        cos, sin = rope_tables(d, max_position, theta, rope_frac, scaling)
        dev = pc.device
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        g = lambda w: None if w is None else torch.as_tensor(np.asarray(w, np.float32)).to(dev)
        self.q_norm, self.k_norm = g(q_norm), g(k_norm)
        self.cfg = _lib.SeamCfg(_ptr(self.q_norm), _ptr(self.k_norm), float(norm_eps),
                                int(bool(cast_after_rope)), float(1.0 / np.sqrt(d)), _ptr(self.cos),
                                _ptr(self.sin), rope_frac, max_position)

    def __call__(self, q, k, v, positions, *, host_stats: bool = True):
        """Projection outputs (float32: q (n, Hq, d), k and v (n, n_kv, d)) ->
        the wire q, k, v (device int32) and the conversion statistics
        {n_values, n_saturated, max_abs_float}; with ``host_stats=False`` the
        statistics stay on the device as ins_seam wrote them (no sync)."""
        pc = self.pc
        t = lambda x: torch.as_tensor(x).to(pc.device, torch.float32).contiguous()
        q, k, v = t(q), t(k), t(v)
        n = q.shape[0]
        on_device = torch.is_tensor(positions) and positions.device.type == "cuda"
        if on_device:       # e.g. position_ids: checked by the kernel, no host read
            pos = positions.to(pc.device, torch.int64).reshape(-1).expand(n).contiguous() \
                if positions.numel() == 1 else positions.to(pc.device, torch.int64).reshape(-1).contiguous()
            if pos.numel() != n:
                raise ValueError(f"{pos.numel()} positions for {n} tokens")
        else:
            pos = np.ascontiguousarray(np.broadcast_to(np.asarray(positions, np.int64), (n,)))
        wq = torch.empty(q.shape, dtype=torch.int32, device=pc.device)
        wk = torch.empty(k.shape, dtype=torch.int32, device=pc.device)
        wv = torch.empty(v.shape, dtype=torch.int32, device=pc.device)
        conv = torch.zeros(3, dtype=torch.int64, device=pc.device)
        fn = pc._L.ins_seam_device_positions if on_device else pc._L.ins_seam
        _lib.check(fn(pc._h, n, _ptr(q), _ptr(k), _ptr(v), pos.data_ptr() if on_device else pos.ctypes.data,
                      C.byref(self.cfg), _ptr(wq), _ptr(wk), _ptr(wv), _ptr(conv), _stream(pc.device)))
        return wq, wk, wv, (conv_stats(conv) if host_stats else conv)


def conv_stats(conv: torch.Tensor) -> dict:
    """ins_seam's statistics triple (int64: values, saturated, the bits of the
    largest |float| as a float64) as a host dict."""
    c = conv.cpu().numpy()
    return {"n_values": int(c[0]), "n_saturated": int(c[1]),
            "max_abs_float": float(np.frombuffer(c[2:3].tobytes(), np.float64)[0])}
