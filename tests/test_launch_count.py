"""The library's own count of the kernels it launched (ins_cache_launches),
which bench.py reports as gpu_launches: per step the upload of the ingress's
slots and the ingress (2), then the online scan -- the upload of its tile
plan and 3 launches with the single-launch kernel (the scan, the fold and the
exact re-run of unproven items), or 4 with the separate launches (scores,
values, fold, exact re-run), whether or not an item's tiles fit one fold
block. The small uploads are kernels whose parameter carries the bytes."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


@pytest.mark.parametrize("T,kernel,per_step", [(4096, "fused", 6), (48 * 1024, "fused", 6),
                                               (4096, "split", 7), (48 * 1024, "split", 7)])
def test_launches_per_decode_step(T, kernel, per_step):
    pytest.importorskip("torch")
    from insitu_b200 import DecodeAttention, FixedFormat, Geometry, QuantConfig
    rng = np.random.default_rng(T)
    dec = DecodeAttention(QuantConfig(key_bits=4, value_bits=2), FixedFormat(), Geometry(8, 4, 64),
                          max_seqs=1, capacity=T + 8)
    dec.pc.set_scan_kernel(kernel)
    dec.prefill(0, _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64)))
    before = dec.pc.launches()
    for _ in range(3):
        dec.step(_wire(rng, (1, 32, 64), 1 / 8), _wire(rng, (1, 8, 64)), _wire(rng, (1, 8, 64)))
    dec.pc.status()
    assert dec.pc.launches() - before == 3 * per_step
    dec.close()
