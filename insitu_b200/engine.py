"""``PagedCache``: one C-ABI cache handle, driven with torch device tensors.

torch is the plumbing here -- device memory, the current stream -- and nothing
else. Every byte of compute runs in the CUDA kernels behind the C ABI.

A ``PagedCache`` holds up to ``max_seqs`` sequences of one attention layer in
a paged pool on one GPU. It is what the reference-shaped classes
(``CompressedCache``, ``CompressedAttention``) and the batched decode step
(``DecodeAttention``) are built on.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import _lib
from .config import FixedFormat, Geometry, QuantConfig
from .tables import Tables


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


if hasattr(torch._C, "_cuda_getCurrentRawStream"):
    def _stream(device: torch.device):
        return torch._C._cuda_getCurrentRawStream(device.index)
else:                                                # pragma: no cover
    def _stream(device: torch.device):
        return torch.cuda.current_stream(device).cuda_stream


def _host_array(x, n: int, ctype, np_dtype):
    """``x`` (a scalar, a sequence or an array) broadcast to ``n`` entries of
    ``ctype`` in host memory; returns (keep-alive object, address). Plain
    Python lists take the short path: one ctypes array, no numpy."""
    if isinstance(x, (list, tuple)) and len(x) == n:
        arr = (ctype * n)(*x)
        return arr, C.addressof(arr)
    if isinstance(x, (int, np.integer)):
        arr = (ctype * n)(*([int(x)] * n))
        return arr, C.addressof(arr)
    arr = np.ascontiguousarray(np.broadcast_to(np.asarray(x, dtype=np_dtype), (n,)))
    return arr, arr.ctypes.data


def _ids(x, n: int) -> list:
    """``x`` (a scalar, a sequence or an array) as a list of ``n`` Python ints,
    the form the torch operators take."""
    if isinstance(x, list) and len(x) == n:
        return x
    if isinstance(x, (int, np.integer)):
        return [int(x)] * n
    return np.broadcast_to(np.asarray(x, dtype=np.int64), (n,)).tolist()


def _raise_mapped(err: Exception):
    """Re-raise an operator's error as the C ABI's exception class for its
    status (the message starts with "[status N]"), e.g. CapacityError."""
    msg = str(err)
    i = msg.find("[status ")
    if i >= 0:
        code = int(msg[i + 8:msg.index("]", i)])
        raise _lib._ERRORS.get(code, _lib.InsituError)(code, msg[msg.index("]", i) + 2:].split("\n")[0]) from None
    raise err


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("insitu_b200 needs a CUDA device (sm_100a); there is no CPU path")


class PagedCache:
    """Paged compressed KV cache for ``max_seqs`` sequences, plus its kernels."""

    def __init__(self, quant: QuantConfig, fmt: FixedFormat | None = None,
                 geo: Geometry | None = None, *, max_seqs: int = 1, capacity: int = 4096,
                 page_tokens: int = 256, n_pages: int | None = None,
                 device: int | torch.device | None = None):
        _require_cuda()
        self.quant = quant
        self.fmt = fmt or FixedFormat()
        self.geo = geo or Geometry()
        if self.geo.head_dim != 64:
            raise ValueError("this build supports head_dim 64")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device("cuda", device).index
                                   if not isinstance(device, torch.device) else device.index)
        self.tables = Tables.build(quant, self.fmt, self.geo.head_dim)
        pages_per_seq = max(1, math.ceil(capacity / page_tokens))
        if n_pages is None:
            n_pages = max_seqs * pages_per_seq
        t = self.tables
        f = self.fmt
        self.cfg = _lib.Config(
            self.geo.head_dim, self.geo.n_kv_heads, self.geo.kv_groups, quant.key_bits,
            quant.value_bits, quant.norm_bits, quant.norm_frac, f.qk_frac, f.centroid_frac,
            f.acc_frac, f.acc_width, f.score_width, f.prob_frac, f.exp_lut_bits, int(f.saturate),
            quant.rot_rounds, t.rot_shift, t.rot_inv_sqrt_q15, page_tokens, max_seqs,
            pages_per_seq, 0, n_pages)
        self._keep = [np.ascontiguousarray(a, dtype=np.int64) for a in (
            t.signs.reshape(-1) if t.signs.size else np.zeros(1, np.int64), t.k_centroids,
            t.k_bounds if t.k_bounds.size else np.zeros(1, np.int64), t.v_centroids,
            t.v_bounds if t.v_bounds.size else np.zeros(1, np.int64), t.exp_table)]
        p = lambda a: a.ctypes.data_as(C.POINTER(C.c_int64))
        tb = _lib.Tables(*(p(a) for a in self._keep), t.log2e, t.delta_max)
        self._L = _lib.lib()
        self._ops = _lib.ops()                 # the torch operators of the per-step calls
        h = C.c_void_p()
        _lib.check(self._L.ins_cache_create(C.byref(self.cfg), C.byref(tb), self.device.index,
                                            C.byref(h)))
        self._h = h
        self.max_seqs = max_seqs
        self.page_tokens = page_tokens
        self.row_bytes = self._L.ins_bytes_per_token(C.byref(self.cfg))
        self.capacity = int(self._L.ins_cache_capacity(self._h))

    # -- lifecycle -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            torch.cuda.synchronize(self.device)
            self._L.ins_cache_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def length(self, seq: int = 0) -> int:
        return int(self._L.ins_cache_length(self._h, seq))

    def launches(self) -> int:
        """Kernels launched so far by this cache's ingress, seam and scan calls."""
        return int(self._L.ins_cache_launches(self._h))

    def reset(self, seq: int | None = None) -> None:
        _lib.check(self._L.ins_cache_reset(self._h, -1 if seq is None else seq))

    def status(self) -> None:
        """Raise if a kernel latched an error (range, bounded-wait timeout)."""
        _lib.check(self._L.ins_cache_status(self._h, _stream(self.device)))

    def set_tiles(self, mode: str = "auto") -> None:
        """Tile size of the online scan (ins_cache_set_tiles): "auto", "large"
        or "small". A tuning knob; every mode gives the same results."""
        _lib.check(self._L.ins_cache_set_tiles(self._h, _lib.INS_TILES[mode]))

    def set_scan_kernel(self, mode: str = "split") -> None:
        """Kernels of the online scan (ins_cache_set_scan_kernel): "split"
        (separate launches, the default) or "fused" (one persistent launch).
        Same results."""
        _lib.check(self._L.ins_cache_set_scan_kernel(self._h, _lib.INS_SCAN[mode]))

    def set_wait_test(self, poll_limit: int = 1 << 22, item: int = -1, chunk: int = 0,
                      head: int = 0) -> None:
        """Test hook of the online scan's bounded waits (ins_cache_set_wait_test):
        the look-back of the fused kernel, the staged rows of the value pass."""
        _lib.check(self._L.ins_cache_set_wait_test(self._h, poll_limit, item, chunk, head))

    def recomputed(self) -> int:
        """Items of the last online scan that the exact sequential kernel redid
        (ins_scan_recomputed); 0 when the context-parallel scan proved them all."""
        k = self._L.ins_scan_recomputed(self._h, _stream(self.device))
        if k < 0:
            _lib.check(_lib.INS_ECUDA)
        return int(k)

    def recomputed_total(self) -> int:
        """Items the exact sequential kernel redid over every online scan of
        this cache so far (ins_scan_recomputed_total)."""
        k = self._L.ins_scan_recomputed_total(self._h, _stream(self.device))
        if k < 0:
            _lib.check(_lib.INS_ECUDA)
        return int(k)

    # -- tensors -------------------------------------------------------------
    def _dev_i32(self, x, shape_tail) -> torch.Tensor:
        if (isinstance(x, torch.Tensor) and x.dtype == torch.int32 and x.device == self.device
                and x.is_contiguous() and tuple(x.shape[1:]) == tuple(shape_tail)):
            return x
        t = torch.as_tensor(x)
        if t.dtype != torch.int32:
            if t.dtype.is_floating_point:
                raise TypeError("fixed-point input must be integer; convert with Q.from_float")
            if t.numel() and (int(t.max()) >= 2 ** 31 or int(t.min()) < -2 ** 31):
                raise _lib.RangeError(_lib.INS_ERANGE, "value does not fit int32")
            t = t.to(torch.int32)
        t = t.to(self.device).contiguous()
        if tuple(t.shape[1:]) != tuple(shape_tail):
            raise ValueError(f"expected (..., {shape_tail}), got {tuple(t.shape)}")
        return t

    # -- kernels -------------------------------------------------------------
    def ingress(self, seq_ids, k, v, q=None, *, prerotated: bool = False):
        """Rotate, quantise, pack and append one token per row (see ins_ingress).

        ``k``, ``v``: (n, n_kv, d); ``q``: (n, n_kv*groups, d) or None.
        Returns the rotated q (device int32) or None.
        """
        g = self.geo
        k = self._dev_i32(k, (g.n_kv_heads, g.head_dim))
        v = self._dev_i32(v, (g.n_kv_heads, g.head_dim))
        n = k.shape[0]
        if v.shape[0] != n:
            raise ValueError("k and v carry different token counts")
        if q is not None:
            q = self._dev_i32(q, (g.num_heads, g.head_dim))
            if q.shape[0] != n:
                raise ValueError("q carries a different token count")
        try:
            return self._ops.ingress(self._h.value, _ids(seq_ids, n), k, v, q, g.n_kv_heads, g.num_heads,
                                     prerotated)
        except (RuntimeError, ValueError) as e:
            _raise_mapped(e)

    def ingress_lanes(self, seq_ids, lanes) -> torch.Tensor:
        """ins_ingress from the board's ingress stream: ``lanes`` holds n tokens
        of ``lanes_bytes_per_token`` bytes (see insitu_b200.wire). Returns the
        rotated q (device int32, (n, n_kv*groups, d))."""
        g = self.geo
        per = int(self._L.ins_lanes_bytes_per_token(self._h))
        t = torch.as_tensor(lanes)
        if t.dtype != torch.uint8 or t.numel() % per:
            raise ValueError(f"lanes must be uint8, a whole number of {per}-byte tokens")
        t = t.reshape(-1).to(self.device).contiguous()
        n = t.numel() // per
        ids, ids_p = _host_array(seq_ids, n, C.c_int32, np.int32)
        q_rot = torch.empty((n, g.num_heads, g.head_dim), dtype=torch.int32, device=self.device)
        _lib.check(self._L.ins_ingress_lanes(self._h, n, ids_p, _ptr(t), _ptr(q_rot),
                                             _stream(self.device)))
        return q_rot

    @property
    def lanes_bytes_per_token(self) -> int:
        return int(self._L.ins_lanes_bytes_per_token(self._h))

    def ddr_image(self, seq: int, capacity: int) -> torch.Tensor:
        """The board's DDR image of one sequence (ins_cache_ddr_image): a
        device uint8 tensor of ins_ddr_image_bytes(capacity) bytes."""
        nb = int(self._L.ins_ddr_image_bytes(self._h, capacity))
        if nb < 0:
            _lib.check(_lib.INS_EINVAL)
        img = torch.empty(nb, dtype=torch.uint8, device=self.device)
        _lib.check(self._L.ins_cache_ddr_image(self._h, seq, capacity, _ptr(img), _stream(self.device)))
        return img

    def rotate(self, x) -> torch.Tensor:
        """Rotation.apply on the device: (..., d) int32 in, int32 out."""
        t = torch.as_tensor(x)
        shape = t.shape
        t = self._dev_i32(t.reshape(-1, self.geo.head_dim), (self.geo.head_dim,))
        y = torch.empty_like(t)
        _lib.check(self._L.ins_rotate(self._h, t.shape[0], _ptr(t), _ptr(y),
                                      _stream(self.device)))
        return y.reshape(shape)

    def scores(self, seq: int, kv_head: int, q_rot, t0: int = 0, n: int | None = None):
        """(s, overflows) for rows [t0, t0+n) of one sequence and KV head."""
        g = self.geo
        q = self._dev_i32(torch.as_tensor(q_rot).reshape(g.kv_groups, g.head_dim),
                          (g.head_dim,))
        if n is None:
            n = self.length(seq) - t0
        s = torch.empty((g.kv_groups, max(n, 0)), dtype=torch.int64, device=self.device)
        ovf = torch.zeros(1, dtype=torch.int64, device=self.device)
        _lib.check(self._L.ins_scores(self._h, seq, kv_head, t0, n, _ptr(q), _ptr(s), _ptr(ovf),
                                      _stream(self.device)))
        return s, ovf

    def finalize(self, acc, l):
        """_finalize (ops/attention.py:873-880) on the device for n (acc, l)
        pairs: acc (n, d) and l (n,) int64 -> (out (n, d), reciprocal (n,),
        total shift (n,)), by the scan epilogue's own device function."""
        a = torch.as_tensor(acc, dtype=torch.int64).to(self.device).contiguous()
        lv = torch.as_tensor(l, dtype=torch.int64).to(self.device).contiguous()
        n = lv.numel()
        if a.shape != (n, self.geo.head_dim):
            raise ValueError(f"acc must be (n, {self.geo.head_dim}) for n = {n} values of l")
        out = torch.empty_like(a)
        r = torch.empty(n, dtype=torch.int64, device=self.device)
        sh = torch.empty(n, dtype=torch.int64, device=self.device)
        _lib.check(self._L.ins_finalize(self._h, n, _ptr(a), _ptr(lv), _ptr(out), _ptr(r), _ptr(sh),
                                        _stream(self.device)))
        return out, r, sh

    def exp_lut(self, delta) -> torch.Tensor:
        """ExpLut.__call__ (ops/attention.py:153-159) on the device through the
        scan kernels' three forms of the lookup: (3, n) int32."""
        d = torch.as_tensor(delta, dtype=torch.int64).to(self.device).contiguous().reshape(-1)
        p = torch.empty((3, d.numel()), dtype=torch.int32, device=self.device)
        _lib.check(self._L.ins_exp_lut(self._h, d.numel(), _ptr(d), _ptr(p), _stream(self.device)))
        return p

    def scan(self, seq_ids, q_rot, *, lengths=None, mode: str = "online", stats: bool = True,
             out: torch.Tensor | None = None, stats_out: torch.Tensor | None = None):
        """One decode step for B sequences: (out (B, Hq, d) int64, stats (B, n_kv, 6))."""
        g = self.geo
        q = self._dev_i32(q_rot, (g.num_heads, g.head_dim))
        B = q.shape[0]
        lens = None if lengths is None else _ids(lengths, B)
        m = {"online": _lib.INS_SOFTMAX_ONLINE, "two_pass": _lib.INS_SOFTMAX_TWO_PASS}[mode]
        try:
            res, st = self._ops.scan(self._h.value, _ids(seq_ids, B), lens, q, g.n_kv_heads, m,
                                     bool(stats or stats_out is not None))
        except (RuntimeError, ValueError) as e:
            _raise_mapped(e)
        if out is not None:
            out.copy_(res)
            res = out
        if stats_out is not None:
            stats_out.copy_(st)
            st = stats_out
        return res, (st if stats else None)

    def step(self, seq_ids, q, k, v, *, mode: str = "online", stats: bool = True):
        """One decode token per sequence in one call (the ``insitu::step``
        operator): the ingress of q, k, v (B rows, one per sequence), then the
        scan of every sequence with the new token. Returns (out, stats)."""
        g = self.geo
        k = self._dev_i32(k, (g.n_kv_heads, g.head_dim))
        v = self._dev_i32(v, (g.n_kv_heads, g.head_dim))
        q = self._dev_i32(q, (g.num_heads, g.head_dim))
        m = {"online": _lib.INS_SOFTMAX_ONLINE, "two_pass": _lib.INS_SOFTMAX_TWO_PASS}[mode]
        try:
            return self._ops.step(self._h.value, _ids(seq_ids, q.shape[0]), q, k, v, g.n_kv_heads, m, stats)
        except (RuntimeError, ValueError) as e:
            _raise_mapped(e)

    # -- context split (one sequence across shards) -------------------------------
    S_LO = -(1 << 47)   # the running maximum before any token (score_width 48)

    def _split_args(self, seq_ids, q_rot, lengths):
        g = self.geo
        q = self._dev_i32(q_rot, (g.num_heads, g.head_dim))
        B = q.shape[0]
        ids = np.ascontiguousarray(np.broadcast_to(np.asarray(seq_ids, dtype=np.int32), (B,)))
        lens = None
        if lengths is not None:
            lens = np.ascontiguousarray(np.broadcast_to(np.asarray(lengths, dtype=np.int64), (B,)))
        return q, B, ids, lens

    def scan_maxima(self, seq_ids, q_rot, *, lengths=None) -> torch.Tensor:
        """Phase 1 of a context split (ins_scan_maxima): this shard's maximum
        score per (sequence, KV head, query head), (B, n_kv, groups) int64."""
        q, B, ids, lens = self._split_args(seq_ids, q_rot, lengths)
        mx = torch.empty((B, self.geo.n_kv_heads, self.geo.kv_groups), dtype=torch.int64,
                         device=self.device)
        _lib.check(self._L.ins_scan_maxima(self._h, B, ids.ctypes.data_as(C.c_void_p),
                                           None if lens is None else lens.ctypes.data_as(C.c_void_p),
                                           _ptr(q), _ptr(mx), _stream(self.device)))
        self._split_q = q          # the same q_rot buffer must reach phase 2
        return mx

    def scan_part(self, seq_ids, m_in, *, lengths=None) -> torch.Tensor:
        """Phase 2 (ins_scan_part): this shard's composites given the running
        maximum entering it (``m_in`` shaped like scan_maxima's result); one
        uint8 buffer of part_bytes(B) bytes."""
        q = getattr(self, "_split_q", None)
        if q is None:
            raise RuntimeError("scan_part needs scan_maxima first")
        _, B, ids, lens = self._split_args(seq_ids, q, lengths)
        m = torch.as_tensor(m_in, dtype=torch.int64).to(self.device).contiguous()
        if m.numel() != B * self.geo.n_kv_heads * self.geo.kv_groups:
            raise ValueError("m_in must hold one value per (sequence, KV head, query head)")
        part = torch.empty(self.part_bytes(B), dtype=torch.uint8, device=self.device)
        _lib.check(self._L.ins_scan_part(self._h, B, ids.ctypes.data_as(C.c_void_p),
                                         None if lens is None else lens.ctypes.data_as(C.c_void_p),
                                         _ptr(q), _ptr(m), _ptr(part), _stream(self.device)))
        self._split_q = None
        return part

    def part_bytes(self, B: int) -> int:
        n = self._L.ins_part_bytes(self._h, int(B))
        if n < 0:
            _lib.check(_lib.INS_EINVAL)
        return int(n)

    def merge_parts(self, parts: torch.Tensor, B: int, *, stats: bool = True):
        """Fold the shards' composites (``parts``: (n_parts, part_bytes(B)) uint8
        on this device, in causal order) into outputs and stats, as
        ``scan`` returns them for the whole sequences."""
        g = self.geo
        p = torch.as_tensor(parts).to(self.device).contiguous()
        n_parts = p.shape[0]
        if p.dtype != torch.uint8 or p.numel() != n_parts * self.part_bytes(B):
            raise ValueError("parts must be (n_parts, part_bytes(B)) uint8")
        out = torch.empty((B, g.num_heads, g.head_dim), dtype=torch.int64, device=self.device)
        st = torch.empty((B, g.n_kv_heads, len(_lib.STATS_FIELDS)), dtype=torch.int64,
                         device=self.device) if stats else None
        _lib.check(self._L.ins_merge_parts(self._h, B, n_parts, _ptr(p), _ptr(out), _ptr(st),
                                           _stream(self.device)))
        return out, st

    # -- format conversion (blocking) --------------------------------------------
    def export(self, seq: int, kv_head: int, t0: int = 0, n: int | None = None) -> np.ndarray:
        """Rows [t0, t0+n) in the reference's packed format: (n, row_bytes) uint8."""
        if n is None:
            n = self.length(seq) - t0
        rows = np.empty((max(n, 0), self.row_bytes), dtype=np.uint8)
        torch.cuda.synchronize(self.device)
        _lib.check(self._L.ins_cache_export(self._h, seq, kv_head, t0, n,
                                            rows.ctypes.data_as(C.c_void_p)))
        return rows

    def import_rows(self, seq: int, rows) -> None:
        """Append packed rows shaped (n, n_kv, row_bytes) -- a cache image."""
        rows = np.ascontiguousarray(rows, dtype=np.uint8)
        if rows.ndim != 3 or rows.shape[1:] != (self.geo.n_kv_heads, self.row_bytes):
            raise ValueError(f"expected (n, {self.geo.n_kv_heads}, {self.row_bytes}) rows, "
                             f"got {rows.shape}")
        torch.cuda.synchronize(self.device)
        _lib.check(self._L.ins_cache_import(self._h, seq, rows.shape[0],
                                            rows.ctypes.data_as(C.c_void_p)))
