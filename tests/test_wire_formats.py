"""The board's byte formats on the GPU: the 24-bit lane ingress stream and the
DDR image of a cache, bit for bit against the
reference's own golden files and the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _pc(kb=4, vb=2, max_seqs=1, capacity=4096):
    from insitu_b200 import FixedFormat, Geometry, PagedCache, QuantConfig
    return PagedCache(QuantConfig(key_bits=kb, value_bits=vb), FixedFormat(), Geometry(8, 4, 64),
                      max_seqs=max_seqs, capacity=capacity)


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


def test_lane_stream_ingress_matches_golden(tbvec):
    pc = _pc()
    assert pc.lanes_bytes_per_token == 9216
    q_rot = pc.ingress_lanes([0], tbvec["ingress_stream"])
    pc.status()
    np.testing.assert_array_equal(q_rot.cpu().numpy()[0], tbvec["rot_q"])
    rows = np.stack([pc.export(0, h) for h in range(8)], axis=1)[0]
    np.testing.assert_array_equal(rows, tbvec["kv_rows"])


@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3)])
def test_lane_stream_equals_int32_ingress(kb, vb):
    from insitu_b200 import wire
    rng = np.random.default_rng(kb * 10 + vb)
    lens = [150, 1, 97]
    ids = np.concatenate([np.full(n, b, np.int32) for b, n in enumerate(lens)])
    rng.shuffle(ids)
    n = ids.size
    q, k, v = _wire(rng, (n, 32, 64), 1 / 8), _wire(rng, (n, 8, 64)), _wire(rng, (n, 8, 64))
    a, b = _pc(kb, vb, 3, 256), _pc(kb, vb, 3, 256)
    qa = a.ingress(ids, k, v, q)
    qb = b.ingress_lanes(ids, wire.ingress_stream(q, k, v))
    a.status()
    b.status()
    assert torch.equal(qa, qb)
    for s in range(3):
        for h in (0, 5):
            np.testing.assert_array_equal(a.export(s, h), b.export(s, h))
    oa, sa = a.scan(np.arange(3), qa[:3])
    ob, sb = b.scan(np.arange(3), qb[:3])
    assert torch.equal(oa, ob) and torch.equal(sa, sb)


def test_ddr_image_matches_golden_and_oracle(tbvec):
    import oracle
    from insitu_b200._lib import CapacityError
    cap = int(tbvec["ddr_map"][0])
    pc = _pc(capacity=cap)
    pc.import_rows(0, tbvec["cache_rows"])
    img = pc.ddr_image(0, cap)
    np.testing.assert_array_equal(img.cpu().numpy(), tbvec["ddr_image"])
    # a larger, ragged pair of sequences against the oracle, twice (the
    # padding must come out zero whatever the buffer held)
    rng = np.random.default_rng(9)
    pc2 = _pc(3, 3, max_seqs=2, capacity=1536)
    for s, n in enumerate((1300, 257)):
        pc2.ingress(np.full(n, s, np.int32), _wire(rng, (n, 8, 64)), _wire(rng, (n, 8, 64)))
    for s in (0, 1):
        rows = np.stack([pc2.export(s, h) for h in range(8)], axis=1)
        want = oracle.ddr_image(rows, 24, 24, 1400)
        for _ in range(2):
            np.testing.assert_array_equal(pc2.ddr_image(s, 1400).cpu().numpy(), want)
    with pytest.raises(CapacityError):
        pc2.ddr_image(0, 1000)
