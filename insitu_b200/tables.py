"""The integer tables the kernels consume, built on the host once per config.

Three tables define the compressed format, and the device never derives any
of them itself:

* the sign diagonal of the randomized Hadamard rotation, drawn from numpy's
  PCG64 stream for ``seed`` (the format definition in INSITU
  ``ops/rotate.py:144-155``: ``integers(0, 2, size=(rounds, d)) * 2 - 1``);
* the Lloyd-Max codebooks for the rotated (standard-normal) channels, as
  Q(centroid_frac) integers with floor-midpoint decision boundaries
  (``ops/codebook.py:67-120``), or the MSE-optimal uniform control
  (``ops/codebook.py:123-154``);
* the 2^-x table of the fixed-point exponential and its two constants
  (``ops/attention.py:104-151``).

The solver below is this package's own statement of Lloyd's algorithm. Its
numerical recipe (a 65,536-point grid over +-8 sigma, equal-mass starting
quantiles, a 1e-12 stopping tolerance, forced symmetry, round-half-even to
Q1.15, floor midpoints) has to match the reference's choices step for step,
because the integers it produces are part of the on-HBM format: a codebook that
differed in one LSB would decode every cache written under the other. The
parity tests pin every width 1..8 of both kinds against the reference's own
integers.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass

import numpy as np

from .config import FixedFormat, QuantConfig


# --------------------------------------------------------------------------
# codebooks
# --------------------------------------------------------------------------

def _ascending(a: np.ndarray) -> np.ndarray:
    """Nudge ties that rounding to Q(frac) created, so levels stay strictly increasing."""
    a = a.astype(np.int64).copy()
    for i in range(1, a.size):
        if a[i] <= a[i - 1]:
            a[i] = a[i - 1] + 1
    return a


def _to_q(x: np.ndarray, frac: int) -> np.ndarray:
    """Round half to even into Q(frac), saturating to 32 bits."""
    r = np.rint(np.asarray(x, dtype=np.float64) * (1 << frac)).astype(np.int64)
    return np.clip(r, -(1 << 31), (1 << 31) - 1)


def _normal_grid(points: int = 1 << 16, span: float = 8.0):
    x = np.linspace(-span, span, points)
    w = np.exp(-0.5 * x * x)
    return x, w / w.sum()


@functools.lru_cache(maxsize=64)
def lloyd_max(bits: int, frac: int = 15, symmetric: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """(centroids, boundaries) of the N(0,1) Lloyd-Max quantizer, in Q(frac)."""
    if bits < 1:
        raise ValueError(f"bits={bits} must be at least 1")
    n = 1 << bits
    x, w = _normal_grid()
    levels = np.interp((np.arange(n) + 0.5) / n, np.cumsum(w), x)
    for _ in range(200):
        cells = np.searchsorted(0.5 * (levels[:-1] + levels[1:]), x)
        mass = np.bincount(cells, weights=w, minlength=n)
        moment = np.bincount(cells, weights=w * x, minlength=n)
        updated = np.where(mass > 0, moment / np.maximum(mass, 1e-300), levels)
        converged = np.allclose(updated, levels, atol=1e-12)
        levels = updated
        if converged:
            break
    if symmetric:
        levels = 0.5 * (levels - levels[::-1])
    cent = _ascending(_to_q(levels, frac))
    bounds = _ascending((cent[:-1] + cent[1:]) >> 1)
    return cent, bounds


@functools.lru_cache(maxsize=64)
def uniform_levels(bits: int, frac: int = 15) -> tuple[np.ndarray, np.ndarray]:
    """MSE-optimal equally spaced quantizer for N(0,1): scan the clipping range."""
    n = 1 << bits
    x, w = _normal_grid()
    best, best_err = None, np.inf
    for clip in np.linspace(0.5, 6.0, 400):
        lv = np.linspace(-clip, clip, n) if n > 1 else np.array([0.0])
        err = float((w * (lv[np.searchsorted(0.5 * (lv[:-1] + lv[1:]), x)] - x) ** 2).sum())
        if err < best_err:
            best, best_err = lv, err
    cent = _ascending(_to_q(best, frac))
    return cent, _ascending((cent[:-1] + cent[1:]) >> 1)


def codebook(kind: str, bits: int, frac: int = 15, symmetric: bool = True):
    if kind == "gaussian":
        return lloyd_max(bits, frac, symmetric)
    if kind == "uniform":
        return uniform_levels(bits, frac)
    raise ValueError(f"unknown codebook {kind!r}")


# --------------------------------------------------------------------------
# rotation signs and the exponential
# --------------------------------------------------------------------------

def sign_diagonal(d: int, seed: int, rounds: int = 1) -> np.ndarray:
    """(rounds, d) int64 of +-1: numpy PCG64(seed), one stream for all rounds."""
    if d & (d - 1):
        raise ValueError(f"d={d} must be a power of two for a Hadamard butterfly")
    if rounds < 0:
        raise ValueError(f"rounds={rounds} must not be negative")
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, 2, size=(rounds, d)).astype(np.int64) * 2 - 1


def rotation_scale(d: int) -> tuple[int, int]:
    """(shift, inv_sqrt_q15): 1/sqrt(d) as an exact shift when log2(d) is even
    (shift >= 0), else shift = -1 and a round(2^15/sqrt(d)) multiply."""
    e = d.bit_length() - 1
    if e % 2 == 0:
        return e // 2, int(round((1 << 15) / np.sqrt(d)))
    return -1, int(round((1 << 15) / np.sqrt(d)))


def exp_table(fmt: FixedFormat) -> tuple[np.ndarray, int, int]:
    """(table, log2e, delta_max) of exp(-x) = 2^-i * 2^-f.

    table[k] = rint(2^(-k/n) * 2^prob_frac) for n = 2^exp_lut_bits entries;
    log2e = round(log2(e) * 2^acc_frac); delta_max is the smallest distance
    whose result is zero for certain, at and above which the input is clamped.
    """
    n = 1 << fmt.exp_lut_bits
    table = np.rint(2.0 ** (-(np.arange(n, dtype=np.float64) / n)) * (1 << fmt.prob_frac))
    table = table.astype(np.int64)
    log2e = int(round(np.log2(np.e) * (1 << fmt.acc_frac)))
    span = (fmt.prob_frac + 2) << fmt.exp_lut_bits
    num = (span << (fmt.acc_frac - fmt.exp_lut_bits)) << fmt.acc_frac
    delta_max = -(-num // log2e)
    return table, log2e, delta_max


@dataclass(frozen=True)
class Tables:
    """Everything the device needs for one (QuantConfig, FixedFormat, d)."""

    d: int
    signs: np.ndarray            # (rounds, d) int64 +-1
    rot_shift: int
    rot_inv_sqrt_q15: int
    k_centroids: np.ndarray
    k_bounds: np.ndarray
    v_centroids: np.ndarray
    v_bounds: np.ndarray
    exp_table: np.ndarray
    log2e: int
    delta_max: int

    @staticmethod
    def build(quant: QuantConfig, fmt: FixedFormat, d: int) -> "Tables":
        kc, kb = codebook(quant.codebook, quant.key_bits, fmt.centroid_frac, quant.symmetric)
        vc, vb = codebook(quant.codebook, quant.value_bits, fmt.centroid_frac, quant.symmetric)
        shift, inv = rotation_scale(d)
        table, log2e, dmax = exp_table(fmt)
        return Tables(d=d, signs=sign_diagonal(d, quant.seed, quant.rot_rounds),
                      rot_shift=shift, rot_inv_sqrt_q15=inv, k_centroids=kc, k_bounds=kb,
                      v_centroids=vc, v_bounds=vb, exp_table=table, log2e=log2e,
                      delta_max=dmax)
