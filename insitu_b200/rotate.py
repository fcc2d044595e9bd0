"""``Rotation``: the randomized Hadamard transform (ops/rotate.py:107-251).

``apply`` runs the rotation kernel on the GPU. The sign diagonal comes from
numpy's PCG64 stream, because that stream is the format's definition of it.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .tables import rotation_scale, sign_diagonal


@dataclass(frozen=True)
class Rotation:
    d: int
    signs: np.ndarray          # (rounds, d) int64 +-1
    seed: int
    device: object = None

    @property
    def rounds(self) -> int:
        return self.signs.shape[0]

    @staticmethod
    def for_quant(quant, d: int, device=None) -> "Rotation":
        """The one constructor every call site uses (ops/rotate.py:124-142)."""
        return Rotation.from_seed(d, quant.seed, quant.rot_rounds, device=device)

    @staticmethod
    def from_seed(d: int, seed: int, rounds: int = 1, device=None) -> "Rotation":
        return Rotation(d=d, signs=sign_diagonal(d, seed, rounds), seed=seed, device=device)

    @property
    def shift(self) -> int | None:
        s, _ = rotation_scale(self.d)
        return s if s >= 0 else None

    @property
    def inv_sqrt_q15(self) -> int:
        return rotation_scale(self.d)[1]

    def apply(self, x, trace=None, unit: str = ""):
        """Rotate along the last axis on the GPU. Fixed-point in, same Q out.

        numpy in -> int64 numpy out (the reference's types); a CUDA tensor in
        -> an int32 CUDA tensor out, with no host round trip.
        """
        import torch
        from .config import QuantConfig
        from .quantize import _device_index, utility_cache
        is_tensor = isinstance(x, torch.Tensor)
        a = x if is_tensor else np.asarray(x)
        if a.shape[-1] != self.d:
            raise ValueError(f"rotate expects last axis {self.d}, got {a.shape[-1]}")
        if not is_tensor and a.dtype.kind not in "iu":
            raise TypeError(f"fixed-point op on dtype {a.dtype}; convert with Q.from_float first")
        quant = QuantConfig(key_bits=1, value_bits=1, seed=self.seed, rot_rounds=self.rounds)
        from .config import FixedFormat
        pc = utility_cache(quant, FixedFormat(), _device_index(self.device), 16)
        if not np.array_equal(pc.tables.signs, self.signs):
            raise ValueError("signs do not come from this rotation's seed")
        y = pc.rotate(a if is_tensor else torch.from_numpy(np.ascontiguousarray(a)))
        pc.status()
        return y if is_tensor else y.cpu().numpy().astype(np.int64)

    def matrix(self) -> np.ndarray:
        """The dense d x d form R_last ... R_0, for the offline W_o fold (host)."""
        h = np.array([[1.0]])
        while h.shape[0] < self.d:
            h = np.block([[h, h], [h, -h]])
        m = np.eye(self.d)
        for r in range(self.rounds):
            m = ((h * self.signs[r]) / np.sqrt(self.d)) @ m
        return m
