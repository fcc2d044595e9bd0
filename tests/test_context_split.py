"""The context split: one sequence's cached tokens held by several shards.

On one GPU the shards are sequences of one cache holding consecutive ranges;
the merged result must equal the single-sequence scan and the oracle bit for
bit (values, statistics), for even and ragged splits, with rescale points on
both sides of shard boundaries. The orchestration over a process group is
covered on CPU in test_context_split_host.py.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _pc(max_seqs, capacity, kb=4, vb=2, groups=4):
    from insitu_b200 import FixedFormat, Geometry, PagedCache, QuantConfig
    return PagedCache(QuantConfig(key_bits=kb, value_bits=vb), FixedFormat(), Geometry(8, groups, 64),
                      max_seqs=max_seqs, capacity=capacity)


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


def _split_cache(T, cuts, rng, kb=4, vb=2, groups=4, k=None):
    """Sequence 0 holds all T tokens; sequences 1.. hold the shards [cuts]."""
    bounds = [0, *cuts, T]
    pc = _pc(max_seqs=len(bounds), capacity=T, kb=kb, vb=vb, groups=groups)
    k = _wire(rng, (T, 8, 64)) if k is None else k
    v = _wire(rng, (T, 8, 64))
    pc.ingress(np.zeros(T, np.int32), k, v)
    for r in range(len(bounds) - 1):
        lo, hi = bounds[r], bounds[r + 1]
        if hi > lo:
            pc.ingress(np.full(hi - lo, r + 1, np.int32), k[lo:hi], v[lo:hi])
    return pc, k, v, len(bounds) - 1


@pytest.mark.parametrize("T,cuts", [(20000, [10000]), (30001, [1, 7777, 20000, 29999]),
                                    (9000, [3000, 6000])])
def test_split_equals_whole_sequence_and_oracle(T, cuts):
    from insitu_b200.context import local_split_scan
    rng = np.random.default_rng(T + len(cuts))
    pc, k, v, n = _split_cache(T, cuts, rng)
    orc = make_oracle()
    qr = orc.rotate(_wire(rng, (1, 32, 64), 1.0 / 8.0))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    want_out, want_st = pc.scan([0], q_rot)
    out, st = local_split_scan(pc, [[r + 1] for r in range(n)], q_rot)
    pc.status()
    assert torch.equal(out, want_out)
    assert torch.equal(st, want_st)
    rows = orc.ingress_rows(k, v, threads=8)
    want, wst = orc.decode_layer(qr, [rows], threads=8)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    np.testing.assert_array_equal(st.cpu().numpy(), wst)


def _rising(T, step, rng):
    base = _wire(rng, (64,), 0.5).astype(np.int64)
    scale = 1.0 + (np.arange(T) // step) * 0.01
    kk = np.clip(np.rint(base[None, :] * scale[:, None] / 8) + rng.integers(-40, 40, size=(T, 64)),
                 -(1 << 23), (1 << 23) - 1).astype(np.int32)
    return np.stack([kk] * 8, axis=1), base


@pytest.mark.parametrize("tiles", ["large", "small"])
def test_split_under_both_tile_sizes(tiles):
    from insitu_b200.context import local_split_scan
    rng = np.random.default_rng(31)
    T = 9000
    pc, k, v, n = _split_cache(T, [2500, 6100], rng)
    pc.set_tiles(tiles)
    orc = make_oracle()
    qr = orc.rotate(_wire(rng, (1, 32, 64), 1.0 / 8.0))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    out, st = local_split_scan(pc, [[r + 1] for r in range(n)], q_rot)
    pc.status()
    rows = orc.ingress_rows(k, v, threads=8)
    want, wst = orc.decode_layer(qr, [rows], threads=8)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    np.testing.assert_array_equal(st.cpu().numpy(), wst)


def test_split_with_rescales_in_every_shard():
    """Rising keys: the running maximum moves in every shard, so the composites
    carry rescale entries and the merge applies them across boundaries."""
    from insitu_b200.context import local_split_scan
    rng = np.random.default_rng(5)
    T = 12000
    base = _wire(rng, (64,), 0.5).astype(np.int64)
    scale = 1.0 + (np.arange(T) // 400) * 0.01
    kk = np.clip(np.rint(base[None, :] * scale[:, None] / 8) + rng.integers(-40, 40, size=(T, 64)),
                 -(1 << 23), (1 << 23) - 1).astype(np.int32)
    k = np.stack([kk] * 8, axis=1)
    pc, k, v, n = _split_cache(T, [4000, 8000], rng, k=k)
    orc = make_oracle()
    qr = orc.rotate(np.tile(base[None, None, :] // 4, (1, 32, 1)))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    want_out, want_st = pc.scan([0], q_rot)
    assert want_st[0, :, 1].sum() > 30            # many rescale events overall
    out, st = local_split_scan(pc, [[1], [2], [3]], q_rot)
    pc.status()
    assert torch.equal(out, want_out)
    assert torch.equal(st, want_st)


def test_split_batched_3b3b_and_errors():
    from insitu_b200.context import local_split_scan
    from insitu_b200._lib import ArgumentError
    rng = np.random.default_rng(8)
    # two sequences, each split in two shards: ids (1, 2) and (3, 4)
    T = [6000, 2500]
    pc = _pc(max_seqs=5, capacity=6000, kb=3, vb=3)
    data = []
    for b, t in enumerate(T):
        k, v = _wire(rng, (t, 8, 64)), _wire(rng, (t, 8, 64))
        data.append((k, v))
        cut = t // 3
        pc.ingress(np.full(cut, 1 + 2 * b, np.int32), k[:cut], v[:cut])
        pc.ingress(np.full(t - cut, 2 + 2 * b, np.int32), k[cut:], v[cut:])
    orc = make_oracle(key_bits=3, value_bits=3)
    qr = orc.rotate(_wire(rng, (2, 32, 64), 1.0 / 8.0))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    out, st = local_split_scan(pc, [[1, 3], [2, 4]], q_rot)
    pc.status()
    rows = [orc.ingress_rows(k, v, threads=8) for k, v in data]
    want, wst = orc.decode_layer(qr, rows, threads=8)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    np.testing.assert_array_equal(st.cpu().numpy(), wst)
    # phase 2 without phase 1, or after another scan, is refused
    pc.scan([1, 3], q_rot)
    with pytest.raises(ArgumentError):
        pc._split_q = pc._dev_i32(q_rot, (32, 64))
        pc.scan_part([1, 3], torch.zeros((2, 8, 4), dtype=torch.int64))


def test_split_that_cannot_prove_exactness_is_reported():
    """Keys rising every few tokens put hundreds of rescales in each shard, more
    than a composite carries: the merge must refuse (INS_ERANGE from status)
    instead of returning a result it cannot prove."""
    from insitu_b200.context import local_split_scan
    from insitu_b200._lib import RangeError
    rng = np.random.default_rng(6)
    T = 8000
    k, base = _rising(T, 3, rng)
    pc, k, v, n = _split_cache(T, [4000], rng, k=k)
    orc = make_oracle()
    q_rot = torch.from_numpy(orc.rotate(np.tile(base[None, None, :] // 4, (1, 32, 1))).astype(np.int32))
    local_split_scan(pc, [[1], [2]], q_rot)
    with pytest.raises(RangeError, match="context-split"):
        pc.status()
    # the cache stays usable: the whole-sequence scan still runs
    out, st = pc.scan([0], q_rot)
    pc.status()
    assert out.shape == (1, 32, 64)
