"""ctypes wrapper over the CPU oracle (``oracle.c``).

TEST INFRASTRUCTURE. The parity tests, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this module to check or time the
CUDA path; the product package ``insitu_b200`` never imports it.

Each method names the reference function it restates (path:line inside the
INSITU repository). Arrays cross as int64 / uint8 numpy arrays.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "d", "key_bits", "value_bits", "norm_bits", "norm_frac", "qk_frac", "centroid_frac",
        "acc_frac", "acc_width", "score_width", "prob_frac", "exp_lut_bits", "saturate",
        "rounds", "rot_shift", "rot_inv_sqrt_q15")] + [
        (n, C.POINTER(C.c_int64)) for n in (
            "signs", "k_centroids", "k_bounds", "v_centroids", "v_bounds", "exp_table")] + [
        ("log2e", C.c_int64)]


class Stats(C.Structure):
    """AttentionStats (ops/attention.py:257-274)."""
    _fields_ = [(n, C.c_int64) for n in (
        "n_tokens", "rescale_events", "score_overflows", "acc_overflows",
        "max_abs_score", "max_abs_acc")]

    def as_tuple(self):
        return tuple(int(getattr(self, n)) for n, _ in self._fields_)


class _Trace(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_int64)) for n in ("s", "m", "p", "l", "grew", "factor", "acc")]


def build(force: bool = False) -> str:
    """Compile ``liboracle.so`` next to its source with the committed Makefile."""
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        cfgp = C.POINTER(_Cfg)
        L.or_rotate.argtypes = [cfgp, _i64p, _i64p, C.c_int64]
        L.or_isqrt.argtypes = [C.c_int64]
        L.or_isqrt.restype = C.c_int64
        L.or_norm_wire.argtypes = [cfgp, _i64p, _i64p, C.c_int64]
        L.or_encode_plane.argtypes = [cfgp, _i64p, _i64p, C.c_int32, _u8p, C.c_int64]
        L.or_bytes_per_token.argtypes = [cfgp]
        L.or_pack.argtypes = [cfgp, _u8p, _i64p, _u8p, _i64p, _u8p, C.c_int64]
        L.or_unpack.argtypes = [cfgp, _u8p, _u8p, _i64p, _u8p, _i64p, C.c_int64]
        L.or_exp.argtypes = [cfgp, C.c_int64]
        L.or_exp.restype = C.c_int64
        L.or_exp_two_step.argtypes = [cfgp, C.c_int64]
        L.or_exp_two_step.restype = C.c_int64
        L.or_exp_delta_max.argtypes = [cfgp]
        L.or_exp_delta_max.restype = C.c_int64
        L.or_reciprocal.argtypes = [cfgp, C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]
        L.or_finalize.argtypes = [cfgp, _i64p, C.c_int64, _i64p]
        L.or_scores.argtypes = [cfgp, _i64p, C.c_int32, _u8p, _i64p, C.c_int64, _i64p]
        L.or_scores.restype = C.c_int64
        L.or_attend_online.argtypes = [cfgp, _i64p, C.c_int32, _u8p, _i64p, _u8p, _i64p,
                                       C.c_int64, _i64p, C.POINTER(Stats), C.POINTER(_Trace)]
        L.or_attend_two_pass.argtypes = [cfgp, _i64p, C.c_int32, _u8p, _i64p, _u8p, _i64p,
                                         C.c_int64, _i64p, C.POINTER(Stats)]
        L.or_attend_online_rows.argtypes = [cfgp, _i64p, C.c_int32, _u8p, C.c_int64, C.c_int64,
                                            _i64p, C.POINTER(Stats)]
        L.or_decode_layer.argtypes = [cfgp, C.c_int32, C.c_int32, C.c_int32,
                                      C.POINTER(C.c_void_p), _i64p, _i64p, _i64p,
                                      C.POINTER(Stats), C.c_int32]
        L.or_ingress_rows.argtypes = [cfgp, _i64p, _i64p, _u8p, C.c_int64, C.c_int32]
        _lib = L
    return _lib


def _i64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _u8(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint8))


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} failed with status {rc}")


class Oracle:
    """One quantiser + attention configuration, with its integer tables.

    ``signs`` is the (rounds, d) +-1 sign diagonal; the codebooks and the exp
    table are the integers the reference builds (Codebook.gaussian,
    ops/codebook.py:67-120; ExpLut, ops/attention.py:104-151).
    """

    def __init__(self, *, d=64, key_bits=4, value_bits=2, k_centroids, k_bounds,
                 v_centroids, v_bounds, signs, exp_table, log2e=94548, norm_bits=16,
                 norm_frac=9, qk_frac=16, centroid_frac=15, acc_frac=16, acc_width=32,
                 score_width=48, prob_frac=15, exp_lut_bits=8, saturate=True):
        self.d, self.key_bits, self.value_bits = d, key_bits, value_bits
        e = d.bit_length() - 1
        rot_shift = e // 2 if e % 2 == 0 else -1
        inv = int(round((1 << 15) / np.sqrt(d)))
        self._keep = [_i64(np.asarray(signs).reshape(-1)), _i64(k_centroids), _i64(k_bounds),
                      _i64(v_centroids), _i64(v_bounds), _i64(exp_table)]
        ptr = lambda a: a.ctypes.data_as(C.POINTER(C.c_int64))
        signs_a = self._keep[0]
        self.rounds = signs_a.size // d
        self.cfg = _Cfg(d, key_bits, value_bits, norm_bits, norm_frac, qk_frac, centroid_frac,
                        acc_frac, acc_width, score_width, prob_frac, exp_lut_bits, int(saturate),
                        self.rounds, rot_shift, inv, *(ptr(a) for a in self._keep), log2e)
        self.L = lib()

    @property
    def bytes_per_token(self) -> int:
        return self.L.or_bytes_per_token(C.byref(self.cfg))

    # -- ingress ---------------------------------------------------------
    def rotate(self, x):                       # Rotation.apply, ops/rotate.py:170
        x = _i64(x)
        y = np.empty_like(x)
        _check(self.L.or_rotate(C.byref(self.cfg), x.reshape(-1), y.reshape(-1),
                                x.size // self.d), "rotate")
        return y

    def isqrt(self, a):                        # ops/quantize.py:42
        return self.L.or_isqrt(int(a))

    def norm_wire(self, x_rot):                # ops/quantize.py:164
        x = _i64(x_rot)
        n = np.empty(x.shape[:-1], dtype=np.int64)
        _check(self.L.or_norm_wire(C.byref(self.cfg), x.reshape(-1), n.reshape(-1),
                                   x.size // self.d), "norm")
        return n

    def encode_plane(self, x_rot, norm, plane):  # ops/quantize.py:183
        x = _i64(x_rot)
        idx = np.empty(x.shape, dtype=np.uint8)
        _check(self.L.or_encode_plane(C.byref(self.cfg), x.reshape(-1), _i64(norm).reshape(-1),
                                      plane, idx.reshape(-1), x.size // self.d), "encode")
        return idx

    def encode(self, k_rot, v_rot):            # ops/quantize.py:198
        kn, vn = self.norm_wire(k_rot), self.norm_wire(v_rot)
        return self.encode_plane(k_rot, kn, 0), kn, self.encode_plane(v_rot, vn, 1), vn

    def pack(self, k_idx, k_norm, v_idx, v_norm):  # ops/quantize.py:237
        k_idx = _u8(k_idx)
        n = k_idx.size // self.d
        rows = np.empty((n, self.bytes_per_token), dtype=np.uint8)
        _check(self.L.or_pack(C.byref(self.cfg), k_idx.reshape(-1), _i64(k_norm).reshape(-1),
                              _u8(v_idx).reshape(-1), _i64(v_norm).reshape(-1),
                              rows.reshape(-1), n), "pack")
        return rows.reshape(*k_idx.shape[:-1], self.bytes_per_token)

    def unpack(self, rows):                    # ops/quantize.py:254
        rows = _u8(rows)
        n = rows.size // self.bytes_per_token
        lead = rows.shape[:-1]
        ki = np.empty((n, self.d), np.uint8)
        vi = np.empty((n, self.d), np.uint8)
        kn = np.empty(n, np.int64)
        vn = np.empty(n, np.int64)
        _check(self.L.or_unpack(C.byref(self.cfg), rows.reshape(-1), ki.reshape(-1), kn, vi.reshape(-1),
                                vn, n), "unpack")
        return (ki.reshape(*lead, self.d), kn.reshape(lead), vi.reshape(*lead, self.d),
                vn.reshape(lead))

    def ingress_rows(self, k, v, threads=1):   # rotate + encode + pack
        k, v = _i64(k), _i64(v)
        n = k.size // self.d
        rows = np.empty((n, self.bytes_per_token), np.uint8)
        _check(self.L.or_ingress_rows(C.byref(self.cfg), k.reshape(-1), v.reshape(-1),
                                      rows.reshape(-1), n, threads), "ingress")
        return rows.reshape(*k.shape[:-1], self.bytes_per_token)

    # -- softmax pieces -------------------------------------------------------
    def exp(self, delta):                      # ops/attention.py:153
        return np.array([self.L.or_exp(C.byref(self.cfg), int(x)) for x in np.ravel(delta)],
                        dtype=np.int64).reshape(np.shape(delta))

    def exp_two_step(self, delta):             # ops/attention.py:161
        return np.array([self.L.or_exp_two_step(C.byref(self.cfg), int(x))
                         for x in np.ravel(delta)], dtype=np.int64).reshape(np.shape(delta))

    def exp_delta_max(self):
        return self.L.or_exp_delta_max(C.byref(self.cfg))

    def reciprocal(self, l):                   # ops/attention.py:197
        r, s = C.c_int64(), C.c_int64()
        rr, ss = [], []
        for x in np.ravel(l):
            self.L.or_reciprocal(C.byref(self.cfg), int(x), C.byref(r), C.byref(s))
            rr.append(r.value)
            ss.append(s.value)
        return np.array(rr, np.int64), np.array(ss, np.int64)

    def finalize(self, acc, l):                # ops/attention.py:873
        acc = _i64(acc).reshape(-1, self.d)
        out = np.empty_like(acc)
        for i, li in enumerate(np.ravel(l)):
            self.L.or_finalize(C.byref(self.cfg), acc[i], int(li), out[i])
        return out

    # -- attention ------------------------------------------------------------
    def scores(self, q_rot, k_idx, k_norm):    # ops/attention.py:333
        q = _i64(q_rot).reshape(-1, self.d)
        T = np.asarray(k_norm).size
        s = np.empty((q.shape[0], T), np.int64)
        ovf = self.L.or_scores(C.byref(self.cfg), q.reshape(-1), q.shape[0],
                               _u8(k_idx).reshape(-1), _i64(k_norm), T, s.reshape(-1))
        return s, int(ovf)

    def attend_online(self, q_rot, k_idx, k_norm, v_idx, v_norm, trace=False):
        """attend_online (ops/attention.py:451-513) -> (out, stats[, trace])."""
        q = _i64(q_rot).reshape(-1, self.d)
        H, T = q.shape[0], np.asarray(k_norm).size
        out = np.empty((H, self.d), np.int64)
        st = Stats()
        tr = None
        bufs = {}
        if trace:
            for n in ("s", "m", "p", "l", "grew", "factor"):
                bufs[n] = np.zeros((T, H), np.int64)
            bufs["acc"] = np.zeros((T, H, self.d), np.int64)
            tr = _Trace(**{n: a.ctypes.data_as(C.POINTER(C.c_int64)) for n, a in bufs.items()})
        _check(self.L.or_attend_online(C.byref(self.cfg), q.reshape(-1), H,
                                       _u8(k_idx).reshape(-1), _i64(k_norm),
                                       _u8(v_idx).reshape(-1), _i64(v_norm), T, out.reshape(-1),
                                       C.byref(st), C.byref(tr) if tr is not None else None),
               "attend_online")
        return (out, st.as_tuple(), bufs) if trace else (out, st.as_tuple())

    def attend_two_pass(self, q_rot, k_idx, k_norm, v_idx, v_norm):
        """attend_two_pass (ops/attention.py:429-449) -> (out, stats)."""
        q = _i64(q_rot).reshape(-1, self.d)
        H, T = q.shape[0], np.asarray(k_norm).size
        out = np.empty((H, self.d), np.int64)
        st = Stats()
        _check(self.L.or_attend_two_pass(C.byref(self.cfg), q.reshape(-1), H,
                                         _u8(k_idx).reshape(-1), _i64(k_norm),
                                         _u8(v_idx).reshape(-1), _i64(v_norm), T,
                                         out.reshape(-1), C.byref(st)), "attend_two_pass")
        return out, st.as_tuple()

    def attend_online_rows(self, q_rot, rows):
        """attend_online over packed rows (T, row_bytes) of one KV head."""
        q = _i64(q_rot).reshape(-1, self.d)
        rows = _u8(rows)
        out = np.empty((q.shape[0], self.d), np.int64)
        st = Stats()
        _check(self.L.or_attend_online_rows(C.byref(self.cfg), q.reshape(-1), q.shape[0],
                                            rows.reshape(-1), rows.shape[-1], rows.shape[0],
                                            out.reshape(-1), C.byref(st)), "attend_online_rows")
        return out, st.as_tuple()

    def decode_layer(self, q_rot, caches, threads=1):
        """One decode step of a layer (kernel.py:338-345).

        ``q_rot`` (B, n_kv*H, d); ``caches`` a list of B uint8 arrays shaped
        (T_b, n_kv, row_bytes). Returns out (B, n_kv*H, d) and stats (B, n_kv, 6).
        """
        q = _i64(q_rot)
        B = q.shape[0]
        n_kv = caches[0].shape[1]
        H = q.shape[1] // n_kv
        caches = [_u8(c) for c in caches]
        ptrs = (C.c_void_p * B)(*[c.ctypes.data for c in caches])
        T = np.array([c.shape[0] for c in caches], np.int64)
        out = np.empty_like(q)
        st = (Stats * (B * n_kv))()
        _check(self.L.or_decode_layer(C.byref(self.cfg), B, n_kv, H, ptrs, T, q.reshape(-1),
                                      out.reshape(-1), st, threads), "decode_layer")
        stats = np.array([s.as_tuple() for s in st], np.int64).reshape(B, n_kv, 6)
        return out, stats


# --------------------------------------------------------------------------
# The board's byte formats around the cache, restated in numpy (small inputs)
# --------------------------------------------------------------------------

def unpack_lanes(buf, bits: int, count: int) -> np.ndarray:
    """unpack_lanes (hw/vectors.py:95-104): LSB-first fields, sign-extended."""
    acc = int.from_bytes(bytes(np.asarray(buf, dtype=np.uint8)), "little")
    out = np.empty(count, dtype=np.int64)
    for i in range(count):
        f = (acc >> (i * bits)) & ((1 << bits) - 1)
        out[i] = f - (1 << bits) if f >> (bits - 1) else f
    return out


def ingress_from_stream(stream, n_kv: int, groups: int, d: int = 64, bits: int = 24):
    """The q, k, v of one token from its ingress stream: per KV head h the
    vectors [k_h, v_h, q_{h*groups} ..] (VectorSet.ingress_groups,
    hw/vectors.py:178-196). Returns q (n_kv*groups, d), k, v (n_kv, d)."""
    vec = d * bits // 8
    stream = np.asarray(stream, dtype=np.uint8)
    q = np.empty((n_kv * groups, d), np.int64)
    k = np.empty((n_kv, d), np.int64)
    v = np.empty((n_kv, d), np.int64)
    for h in range(n_kv):
        base = h * (2 + groups) * vec
        get = lambda j: unpack_lanes(stream[base + j * vec: base + (j + 1) * vec], bits, d)
        k[h], v[h] = get(0), get(1)
        for j in range(groups):
            q[h * groups + j] = get(2 + j)
    return q, k, v


def ddr_image(rows, kbytes: int, vbytes: int, capacity: int) -> np.ndarray:
    """DdrLayout.image (hw/ddr_layout.py:96-245) of rows (n, n_kv, row_bytes):
    planes = the fields (K codes, V codes, norms) cut into 16-byte beats; each
    plane spans capacity x the widest plane, rounded up to 4 KB; head-major."""
    rows = np.asarray(rows, dtype=np.uint8)
    n, heads, rb = rows.shape
    planes = []
    for lo, hi in ((0, kbytes), (kbytes, kbytes + vbytes), (kbytes + vbytes, rb)):
        a = lo
        while a < hi:
            b = min(a + 16, hi)
            planes.append((a, b))
            a = b
    span = -(-capacity * max(b - a for a, b in planes) // 4096) * 4096
    img = np.zeros(heads * len(planes) * span, dtype=np.uint8)
    for h in range(heads):
        for p, (a, b) in enumerate(planes):
            start = (h * len(planes) + p) * span
            chunk = rows[:, h, a:b].reshape(-1)
            img[start:start + chunk.size] = chunk
    return img
