"""Benchmark configs 3 and 4 at test size: the CUDA path against the oracle.

Config 4 is batched decode over a paged cache whose sequences have lengths
drawn uniformly (seeded), for the 4b/2b and 3b/3b codebooks: here 12
sequences of 1K-6K tokens (the benchmark runs 256 of 1K-64K). Config 3 is a
stack of independent layer caches, each fed its own tokens, decoded layer by
layer: here 16 layers of 512 tokens and two decode steps (the benchmark runs
16 x 8K). Every output, statistic and cached byte must equal the oracle's.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


def _decoder(kb, vb, max_seqs, capacity):
    from insitu_b200 import DecodeAttention, FixedFormat, Geometry, QuantConfig
    return DecodeAttention(QuantConfig(key_bits=kb, value_bits=vb), FixedFormat(), Geometry(8, 4, 64),
                           max_seqs=max_seqs, capacity=capacity)


@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3)])
def test_config4_batched_uniform_lengths(kb, vb):
    rng = np.random.default_rng(40 + kb)
    lens = rng.integers(1024, 6 * 1024 + 1, size=12)
    B = len(lens)
    dec = _decoder(kb, vb, B, int(lens.max()) + 4)
    orc = make_oracle(key_bits=kb, value_bits=vb)
    caches = []
    for b, T in enumerate(lens):
        k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
        dec.prefill(b, k, v)
        caches.append((k, v))
    # one decode token per sequence (batched ingress + batched scan), twice
    for step in range(2):
        q = _wire(rng, (B, 32, 64), 1.0 / 8.0)
        k1, v1 = _wire(rng, (B, 8, 64)), _wire(rng, (B, 8, 64))
        out, st = dec.step(q, k1, v1)
        caches = [(np.concatenate([k, k1[b:b + 1]]), np.concatenate([v, v1[b:b + 1]]))
                  for b, (k, v) in enumerate(caches)]
        rows = [orc.ingress_rows(k, v, threads=8) for k, v in caches]
        want, wst = orc.decode_layer(orc.rotate(q), rows, threads=8)
        np.testing.assert_array_equal(out.cpu().numpy(), want, err_msg=f"step {step}")
        np.testing.assert_array_equal(st.cpu().numpy(), wst, err_msg=f"step {step}")
    dec.pc.status()
    for b in (0, B - 1):
        for h in (0, 7):
            np.testing.assert_array_equal(dec.pc.export(b, h), rows[b][:, h])
    assert dec.pc.recomputed() == 0
    dec.close()


def test_config3_layer_stack():
    rng = np.random.default_rng(3)
    L, T = 16, 512
    orc = make_oracle()
    layers = []
    for _ in range(L):
        dec = _decoder(4, 2, 1, T + 4)
        k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
        dec.prefill(0, k, v)
        layers.append([dec, k, v])
    for step in range(2):
        for li, (dec, k, v) in enumerate(layers):
            q = _wire(rng, (1, 32, 64), 1.0 / 8.0)
            k1, v1 = _wire(rng, (1, 8, 64)), _wire(rng, (1, 8, 64))
            out, st = dec.step(q, k1, v1)
            k, v = np.concatenate([k, k1]), np.concatenate([v, v1])
            layers[li][1:] = [k, v]
            rows = orc.ingress_rows(k, v, threads=8)
            want, wst = orc.decode_layer(orc.rotate(q), [rows], threads=8)
            np.testing.assert_array_equal(out.cpu().numpy(), want, err_msg=f"layer {li} step {step}")
            np.testing.assert_array_equal(st.cpu().numpy(), wst, err_msg=f"layer {li} step {step}")
            if step == 1:
                got = np.stack([dec.pc.export(0, h) for h in range(8)], axis=1)
                np.testing.assert_array_equal(got, rows, err_msg=f"layer {li} cache bytes")
    for dec, _, _ in layers:
        dec.pc.status()
        dec.close()
