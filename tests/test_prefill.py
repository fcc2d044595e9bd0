"""Prefill through the same cache: every token of a chunk
attends the cache up to and including itself, as attend_online_batch /
attend_causal_batch do (ops/attention.py:517-871) -- which the reference pins
bit-identical to the per-token loop, the loop the oracle restates."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


@pytest.mark.parametrize("mode", ["online", "two_pass"])
def test_prefill_chunk_equals_the_per_token_loop(mode):
    from insitu_b200 import DecodeAttention, FixedFormat, Geometry, QuantConfig
    rng = np.random.default_rng(61)
    T0, n = 500, 300
    dec = DecodeAttention(QuantConfig(key_bits=4, value_bits=2), FixedFormat(), Geometry(8, 4, 64),
                          max_seqs=2, capacity=1024)
    k0, v0 = _wire(rng, (T0, 8, 64)), _wire(rng, (T0, 8, 64))
    dec.prefill(1, k0, v0)
    q, k, v = _wire(rng, (n, 32, 64), 1 / 8), _wire(rng, (n, 8, 64)), _wire(rng, (n, 8, 64))
    out, st = dec.prefill_attend(1, q, k, v, mode=mode)
    dec.pc.status()
    orc = make_oracle()
    rows = orc.ingress_rows(np.concatenate([k0, k]), np.concatenate([v0, v]), threads=8)
    q_rot = orc.rotate(q)
    if mode == "online":
        want, wst = orc.decode_layer(q_rot, [rows[:T0 + i + 1] for i in range(n)], threads=8)
        np.testing.assert_array_equal(st.cpu().numpy(), wst)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    else:
        for i in (0, 1, 150, n - 1):
            for h in (0, 7):
                w, _ = orc.attend_two_pass(q_rot[i, 4 * h:4 * h + 4], *_unpack(rows[:T0 + i + 1, h]))
                np.testing.assert_array_equal(out[i, 4 * h:4 * h + 4].cpu().numpy(), w)
    assert dec.pc.length(1) == T0 + n and dec.pc.length(0) == 0
    dec.close()


def _unpack(rows):
    from insitu_b200 import KVQuantizer, QuantConfig
    kv = KVQuantizer(64, QuantConfig(key_bits=4, value_bits=2)).unpack(rows)
    return kv.k_idx, kv.k_norm, kv.v_idx, kv.v_norm


def test_mirror_batch_forms_equal_single_queries(widths):
    from insitu_b200 import CompressedAttention, CompressedCache, QuantConfig
    g = lambda s: widths[f"k4v2_{s}"]
    cache = CompressedCache(1, 64, 128, QuantConfig(key_bits=4, value_bits=2))
    cache.append_rotated(g("k_rot")[:, None, :].astype(np.int32), g("v_rot")[:, None, :].astype(np.int32))
    T = cache.length
    attn = CompressedAttention(cache.quantizer)
    kv = cache.view(0)
    rng = np.random.default_rng(3)
    base = T - 12
    qs = np.stack([g("q_rot")] * 12) + rng.integers(-3000, 3000, size=(12,) + g("q_rot").shape)
    ob, sb = attn.attend_online_batch(qs, kv, base=base)
    tb, _ = attn.attend_causal_batch(qs, kv, base=base)
    for i in range(12):
        one, _ = attn.attend_online(qs[i], kv.select(slice(0, base + i + 1)))
        two, _ = attn.attend_two_pass(qs[i], kv.select(slice(0, base + i + 1)))
        np.testing.assert_array_equal(ob[i], one)
        np.testing.assert_array_equal(tb[i], two)
    assert sb.n_tokens == T
    with pytest.raises(ValueError):
        attn.attend_online_batch(qs, kv, base=T - 5)
