"""A whole attention layer's decode step on the GPU (kernel.py:178-357):
projections, the seam, the compressed cache and its scan, and the output
projection with the inverse rotation folded into W_o (ops/output.py:49-84,
weights.py:70-109).

Integer stages are bit-exact with the reference; the four projections are
library GEMMs over fp16-rounded operands with fp32 products and sums, so y
matches the reference's ``AttentionKernel.forward`` within float32 rounding
of those sums -- and, where a float lands within that rounding of a Q8.16
half-way point, within one wire LSB.
"""

from __future__ import annotations

import numpy as np
import torch

from .config import FixedFormat, Geometry, QuantConfig
from .decode import DecodeAttention
from .rotate import Rotation
from .seam import RopeScaling, Seam, conv_stats, project


def fold_o_proj(o_proj, rotation: Rotation, num_heads: int, head_dim: int) -> np.ndarray:
    """W_o' = W_o @ blockdiag_h(R^T), once at weight-load time, in float64,
    returned in the input's dtype (ops/output.py:49-80). o_proj is
    (hidden, num_heads * head_dim), head-major like merge_heads."""
    w = np.asarray(o_proj)
    if w.shape[1] != num_heads * head_dim:
        raise ValueError(f"o_proj takes {w.shape[1]} inputs; the block gives {num_heads} x {head_dim}")
    r = rotation.matrix().T
    block = np.zeros((num_heads * head_dim,) * 2, dtype=np.float64)
    for h in range(num_heads):
        block[h * head_dim:(h + 1) * head_dim, h * head_dim:(h + 1) * head_dim] = r
    return (w.astype(np.float64) @ block).astype(w.dtype)


class AttentionLayer:
    """One layer: x (tokens, hidden) fp32 in, y (tokens, hidden) fp32 out,
    its compressed cache on the GPU. ``w_o`` is the checkpoint's W_o; pass
    ``o_folded=True`` when it already carries the fold."""

    def __init__(self, w_q, w_k, w_v, w_o, *, hidden: int, num_heads: int, num_kv_heads: int,
                 head_dim: int = 64, quant: QuantConfig | None = None, fmt: FixedFormat | None = None,
                 rope_theta: float = 10000.0, max_position: int = 4096,
                 rope_scaling: RopeScaling | None = None, q_norm=None, k_norm=None,
                 norm_eps: float = 1e-6, biases=(None, None, None, None), o_folded: bool = False,
                 cast_after_rope: bool = True, softmax: str = "two_pass", capacity: int = 4096,
                 device=None, decoder: DecodeAttention | None = None, seq: int = 0):
        # "two_pass" is AttentionKernel's default (kernel.py:117-124); the
        # board runs "online"
        self.softmax = softmax
        self.quant = quant or QuantConfig(key_bits=4, value_bits=2)
        self.fmt = fmt or FixedFormat()
        self.hidden, self.hq, self.hk, self.d = hidden, num_heads, num_kv_heads, head_dim
        geo = Geometry(num_kv_heads, num_heads // num_kv_heads, head_dim)
        # a shared decoder holds several layers' caches as its sequences (one
        # page pool, layer = sequence slot); this layer then does not own it
        self._owns_dec = decoder is None
        if decoder is None:
            decoder = DecodeAttention(self.quant, self.fmt, geo, max_seqs=1, capacity=capacity,
                                      device=device)
        elif decoder.geo != geo or decoder.pc.quant != self.quant or decoder.pc.fmt != self.fmt:
            raise ValueError("the shared decoder was built for another geometry or format")
        if not 0 <= seq < decoder.pc.max_seqs:
            raise ValueError(f"sequence slot {seq} outside the decoder's {decoder.pc.max_seqs}")
        self.dec, self.seq = decoder, seq
        dev = self.dec.pc.device
        if not o_folded:
            w_o = fold_o_proj(np.asarray(w_o, np.float64), Rotation.for_quant(self.quant, head_dim),
                              num_heads, head_dim)
        # the weights rounded to fp16 once and held as fp16 for the projection
        # kernel (ins_project); q, k and v are one projection over their
        # stacked rows (each output is the same fp32 dot product of
        # fp16-rounded operands)
        f16 = lambda w: torch.as_tensor(np.asarray(w, dtype=np.float16)).to(dev)
        self.w_qkv = torch.cat([f16(w_q), f16(w_k), f16(w_v)]).contiguous()
        self.w_o = f16(w_o)
        nq, nk = num_heads * head_dim, num_kv_heads * head_dim
        bq, bk, bv, bo = biases
        self.b_qkv = None
        if bq is not None or bk is not None or bv is not None:
            z = lambda x, m: np.zeros(m, np.float32) if x is None else np.asarray(x, np.float32)
            self.b_qkv = torch.as_tensor(np.concatenate([z(bq, nq), z(bk, nk), z(bv, nk)])).to(dev)
        self.b_o = None if bo is None else torch.as_tensor(np.asarray(bo, np.float32)).to(dev)
        self._split = (nq, nk, nk)
        self.seam = Seam(self.dec.pc, max_position=max_position, theta=rope_theta, scaling=rope_scaling,
                         rope_frac=self.fmt.centroid_frac, q_norm=q_norm, k_norm=k_norm,
                         norm_eps=norm_eps, cast_after_rope=cast_after_rope)
        # ConversionStats kept on the device (values and saturations summed,
        # the largest |float| as a float64), read when asked for
        self._conv_n = torch.zeros(2, dtype=torch.int64, device=dev)
        self._conv_max = torch.zeros(1, dtype=torch.float64, device=dev)
        self._last_conv = None

    def forward(self, x, positions=None):
        """Rows of x are decode tokens, in order (a prefill when there are
        several). Returns y (tokens, hidden) fp32 on the device and the
        attention output (tokens, num_heads * head_dim) int64 Q(acc_frac)."""
        pc = self.dec.pc
        x = torch.as_tensor(x).to(pc.device, torch.float32)
        if x.ndim == 1:
            x = x[None]
        n = x.shape[0]
        T = pc.length(self.seq)
        if positions is None:
            pos = np.arange(T, T + n)
        elif torch.is_tensor(positions) and positions.device.type == "cuda":
            pos = positions            # stays on the device; the seam kernel checks it
        else:
            pos = np.asarray(positions, np.int64)
        q, k, v = project(self.w_qkv, x, self.b_qkv, rounded=True).split(self._split, dim=1)
        q = q.reshape(n, self.hq, self.d)
        k = k.reshape(n, self.hk, self.d)
        v = v.reshape(n, self.hk, self.d)
        wq, wk, wv, conv = self.seam(q, k, v, pos, host_stats=False)
        self.last_wire = (wq, wk, wv)
        self._last_conv = conv
        self._conv_n += conv[:2]
        torch.maximum(self._conv_max, conv[2:].view(torch.float64), out=self._conv_max)
        out, self.last_stats = self.dec.prefill_attend(self.seq, wq, wk, wv, mode=self.softmax)
        merged = out.reshape(n, self.hq * self.d)
        acc = merged.to(torch.float64) / float(1 << self.fmt.qk_frac)      # Q.to_float
        y = project(self.w_o, acc, self.b_o, rounded=True)
        return y, merged

    @property
    def conversion(self) -> dict:
        """All calls' ConversionStats so far (reads the device: a sync)."""
        n = self._conv_n.cpu().numpy()
        return {"n_values": int(n[0]), "n_saturated": int(n[1]),
                "max_abs_float": float(self._conv_max.item())}

    @property
    def last_conversion(self) -> dict | None:
        """The last call's ConversionStats (a sync)."""
        return None if self._last_conv is None else conv_stats(self._last_conv)

    def close(self) -> None:
        if self._owns_dec:
            self.dec.close()
