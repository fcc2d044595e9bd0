"""CUDA path vs the oracle and the reference's golden vectors, bit for bit.

Every test here calls the hand-written sm_100a kernels through the C ABI
(``insitu_b200.PagedCache`` -> ``libinsitu_b200.so``). Integer, byte and index
results must be identical; there is no tolerance anywhere in this file.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _pc(kb=4, vb=2, n_kv=8, groups=4, max_seqs=1, capacity=4096, page_tokens=256, seed=0):
    from insitu_b200 import FixedFormat, Geometry, PagedCache, QuantConfig
    return PagedCache(QuantConfig(key_bits=kb, value_bits=vb, seed=seed), FixedFormat(),
                      Geometry(n_kv, groups, 64), max_seqs=max_seqs, capacity=capacity,
                      page_tokens=page_tokens)


def _np(t):
    return t.cpu().numpy()


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0).astype(np.int64)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


# -- ingress -----------------------------------------------------------------

def test_rotation_kernel_matches_rot_vectors(tbvec):
    pc = _pc(n_kv=1, groups=1)
    for s in ("q", "k", "v"):
        got = _np(pc.rotate(torch.from_numpy(tbvec[f"wire_{s}"].astype(np.int32))))
        np.testing.assert_array_equal(got, tbvec[f"rot_{s}"])
    got = _np(pc.rotate(torch.from_numpy(tbvec["rot_random_in"].astype(np.int32))))
    np.testing.assert_array_equal(got, tbvec["rot_random_out"])
    pc.status()


def test_fused_ingress_matches_kv_rows_and_rot_q(tbvec):
    pc = _pc()
    q_rot = pc.ingress([0], tbvec["wire_k"][None], tbvec["wire_v"][None],
                       tbvec["wire_q"][None])
    pc.status()
    np.testing.assert_array_equal(_np(q_rot)[0], tbvec["rot_q"])
    rows = np.stack([pc.export(0, h) for h in range(8)], axis=1)[0]
    np.testing.assert_array_equal(rows, tbvec["kv_rows"])


def test_encoder_matches_enc_vectors_incl_boundary_ties(tbvec):
    x = tbvec["enc_in"].astype(np.int32)                       # already rotated
    n = x.shape[0]
    pc = _pc(n_kv=1, groups=1, capacity=1024)
    pc.ingress(np.zeros(n, np.int32), x[:, None, :], x[:, None, :], prerotated=True)
    pc.status()
    from insitu_b200 import KVQuantizer, QuantConfig
    kv = KVQuantizer(64, QuantConfig(key_bits=4, value_bits=2)).unpack(pc.export(0, 0))
    np.testing.assert_array_equal(kv.k_norm, tbvec["enc_norm"])
    np.testing.assert_array_equal(kv.v_norm, tbvec["enc_norm"])
    np.testing.assert_array_equal(kv.k_idx, tbvec["enc_idx_key"])
    np.testing.assert_array_equal(kv.v_idx, tbvec["enc_idx_value"])


# -- the scan's scalar stages, driven directly ---------------------------------------

def test_finalize_edges_through_the_device_reciprocal(tbvec):
    """The 49 finalize rows of tb/vectors (17 of them constructed l edges:
    l = 0, 1, powers of two, the 32-bit window boundaries, the 48-bit cap),
    which tests/test_vectors.py:557-634 treats as finalize.sv's contract, run
    through the device reciprocal and epilogue every scan uses."""
    pc = _pc(n_kv=1, groups=1)
    out, r, sh = pc.finalize(torch.from_numpy(tbvec["fin_acc"]), torch.from_numpy(tbvec["fin_l"]))
    pc.status()
    np.testing.assert_array_equal(_np(r), tbvec["fin_recip"])
    np.testing.assert_array_equal(_np(sh), tbvec["fin_shift"])
    np.testing.assert_array_equal(_np(out), tbvec["fin_out"])
    # and against the oracle on random (acc, l) spanning every lead-one position
    rng = np.random.default_rng(91)
    lead = rng.integers(0, 50, size=512)
    l = (np.int64(1) << lead) + rng.integers(0, 1 << 20, size=512) % np.maximum(1, np.int64(1) << lead)
    l[:3] = (0, 1, 2)
    acc = rng.integers(-(1 << 31), 1 << 31, size=(512, 64))
    out, r, sh = pc.finalize(torch.from_numpy(acc), torch.from_numpy(l))
    orc = make_oracle()
    wr, wsh = orc.reciprocal(l)
    np.testing.assert_array_equal(_np(r), wr)
    np.testing.assert_array_equal(_np(sh), wsh)
    np.testing.assert_array_equal(_np(out), orc.finalize(acc, l))


def test_exp_lut_sweep_in_every_device_form(tbvec):
    """The 13,565-point exp sweep of tb/vectors (every table step, the clamp at
    delta_max, the zero tail) through the three device forms of the lookup."""
    pc = _pc(n_kv=1, groups=1)
    p = _np(pc.exp_lut(torch.from_numpy(tbvec["exp_in"])))
    pc.status()
    for row in range(3):
        np.testing.assert_array_equal(p[row], tbvec["exp_out"], err_msg=f"form {row}")
    # a negative distance is refused, as the reference's ValueError
    pc.exp_lut(torch.tensor([5, -1]))
    from insitu_b200._lib import RangeError
    with pytest.raises(RangeError):
        pc.status()


# -- scan over the reference's own cache image ----------------------------------

@pytest.fixture(scope="module")
def tb_cache(tbvec):
    pc = _pc()
    pc.import_rows(0, tbvec["cache_rows"])
    return pc


def test_imported_image_exports_byte_identical(tb_cache, tbvec):
    for h in range(8):
        np.testing.assert_array_equal(tb_cache.export(0, h), tbvec["cache_rows"][:, h])


def test_scores_kernel_matches_scores_hex(tb_cache, tbvec):
    q = tbvec["rot_q"].astype(np.int32)
    got = []
    for h in range(8):
        s, ovf = tb_cache.scores(0, h, torch.from_numpy(q[4 * h:4 * h + 4]))
        got.append(_np(s))
        assert int(ovf.item()) == 0
    np.testing.assert_array_equal(np.concatenate(got), tbvec["scores"])


def test_scores_signed_norm_edge_rows(tbvec):
    pc = _pc(n_kv=1, groups=1)
    rows = tbvec["score_edge_rows"][:, None, :]
    pc.import_rows(0, rows)
    s, _ = pc.scores(0, 0, torch.from_numpy(tbvec["rot_q"][:1].astype(np.int32)))
    np.testing.assert_array_equal(_np(s)[0], tbvec["score_edge_gold"])


def test_online_scan_matches_out_online(tb_cache, tbvec):
    out, st = tb_cache.scan([0], torch.from_numpy(tbvec["rot_q"][None].astype(np.int32)))
    tb_cache.status()
    np.testing.assert_array_equal(_np(out).reshape(1, -1), tbvec["out_online"])
    orc = make_oracle()
    _, ost = orc.decode_layer(tbvec["rot_q"][None], [tbvec["cache_rows"]])
    np.testing.assert_array_equal(_np(st), ost)


def test_two_pass_scan_matches_out_hex(tb_cache, tbvec):
    out, _ = tb_cache.scan([0], torch.from_numpy(tbvec["rot_q"][None].astype(np.int32)),
                           mode="two_pass")
    np.testing.assert_array_equal(_np(out).reshape(1, -1), tbvec["out_two_pass"])


def test_stress_query_with_many_rescale_factors(tbvec, widths):
    pc = _pc(n_kv=1, groups=4)
    pc.import_rows(0, widths["stress_rows"][:, None, :])
    out, st = pc.scan([0], torch.from_numpy(widths["stress_q_rot"][None].astype(np.int32)))
    np.testing.assert_array_equal(_np(out)[0], widths["stress_online"])
    np.testing.assert_array_equal(_np(st)[0, 0], widths["stress_online_stats"])


def test_saturating_accumulator_clamps_exactly(widths):
    pc = _pc(n_kv=1, groups=4)
    pc.import_rows(0, widths["sat_rows"][:, None, :])
    q = torch.from_numpy(widths["sat_q_rot"][None].astype(np.int32))
    out, st = pc.scan([0], q)
    np.testing.assert_array_equal(_np(out)[0], widths["sat_online"])
    np.testing.assert_array_equal(_np(st)[0, 0], widths["sat_online_stats"])
    assert _np(st)[0, 0, 3] > 0
    out2, st2 = pc.scan([0], q, mode="two_pass")
    np.testing.assert_array_equal(_np(out2)[0], widths["sat_two_pass"])
    np.testing.assert_array_equal(_np(st2)[0, 0], widths["sat_two_pass_stats"])


# -- every width the reference tests --------------------------------------------

@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3), (3, 2), (4, 4), (6, 6), (1, 1)])
def test_widths_end_to_end(widths, kb, vb):
    t = f"k{kb}v{vb}"
    g = lambda n: widths[f"{t}_{n}"]
    pc = _pc(kb, vb, n_kv=1, groups=4)
    T = g("k").shape[0]
    pc.ingress(np.zeros(T, np.int32), g("k")[:, None, :].astype(np.int32),
               g("v")[:, None, :].astype(np.int32))
    pc.status()
    np.testing.assert_array_equal(pc.export(0, 0), g("rows"))
    q_rot = _np(pc.rotate(torch.from_numpy(g("q").astype(np.int32))))
    np.testing.assert_array_equal(q_rot, g("q_rot"))
    s, ovf = pc.scores(0, 0, torch.from_numpy(q_rot))
    np.testing.assert_array_equal(_np(s), g("scores"))
    out, st = pc.scan([0], torch.from_numpy(q_rot[None]))
    np.testing.assert_array_equal(_np(out)[0], g("online"))
    np.testing.assert_array_equal(_np(st)[0, 0], g("online_stats"))
    out2, st2 = pc.scan([0], torch.from_numpy(q_rot[None]), mode="two_pass")
    np.testing.assert_array_equal(_np(out2)[0], g("two_pass"))
    np.testing.assert_array_equal(_np(st2)[0, 0], g("two_pass_stats"))


# -- benchmark config 1: 512 sequential ingress steps, then bit-exact ----------------

def test_config1_sequential_ingress_and_decode(config1):
    pc = _pc(capacity=512)
    wk, wv = config1["wire_k"], config1["wire_v"]
    steps = list(config1["steps"])
    for t in range(wk.shape[0]):
        if t in steps:
            i = steps.index(t)
            q_rot = pc.ingress([0], wk[t:t + 1], wv[t:t + 1], config1["wire_q"][i:i + 1])
            out, _ = pc.scan([0], q_rot)
            np.testing.assert_array_equal(_np(out).reshape(-1), config1["out_online"][i],
                                          err_msg=f"step {t}")
        else:
            pc.ingress([0], wk[t:t + 1], wv[t:t + 1])
    pc.status()
    rows = np.stack([pc.export(0, h) for h in range(8)], axis=1)
    np.testing.assert_array_equal(rows, config1["cache"])


# -- larger, ragged, batched: GPU vs oracle ------------------------------------------

def test_batched_ragged_decode_matches_oracle():
    rng = np.random.default_rng(11)
    lens = [0, 1, 2, 255, 256, 257, 3000, 9001]
    B = len(lens)
    pc = _pc(max_seqs=B, capacity=9216)
    orc = make_oracle()
    caches = []
    for b, T in enumerate(lens):
        k = _wire(rng, (T, 8, 64))
        v = _wire(rng, (T, 8, 64))
        if T:
            pc.ingress(np.full(T, b, np.int32), k, v)
        caches.append(orc.ingress_rows(k, v, threads=8) if T else np.zeros((0, 8, 52), np.uint8))
    pc.status()
    for b, T in enumerate(lens):
        if T:
            for h in (0, 7):
                np.testing.assert_array_equal(pc.export(b, h), caches[b][:, h])
    q = _wire(rng, (B, 32, 64), 1.0 / 8.0)
    q_rot = orc.rotate(q)
    out, st = pc.scan(np.arange(B), torch.from_numpy(q_rot.astype(np.int32)))
    want, wst = orc.decode_layer(q_rot, caches, threads=8)
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
    # a causal prefix of each sequence (kv.select(slice(0, ctx)))
    pre = [max(0, T - 7) for T in lens]
    out, _ = pc.scan(np.arange(B), torch.from_numpy(q_rot.astype(np.int32)), lengths=pre)
    want, _ = orc.decode_layer(q_rot, [c[:p] for c, p in zip(caches, pre)], threads=8)
    np.testing.assert_array_equal(_np(out), want)


def test_long_single_sequence_matches_oracle():
    rng = np.random.default_rng(12)
    T = 40000
    pc = _pc(capacity=T)
    k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
    pc.ingress(np.zeros(T, np.int32), k, v)
    q_rot = make_oracle().rotate(_wire(rng, (1, 32, 64), 1.0 / 8.0))
    out, st = pc.scan([0], torch.from_numpy(q_rot.astype(np.int32)))
    orc = make_oracle()
    rows = orc.ingress_rows(k, v, threads=8)
    want, wst = orc.decode_layer(q_rot, [rows], threads=8)
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
    # typical data stays on the context-parallel path: none of the 8 items was
    # handed to the exact sequential kernel
    assert pc.recomputed() == 0


def test_queries_at_the_edge_of_the_fp64_range():
    """Scores run as exact FP64 dot products while |q| < 2^30 (for the default
    codebooks, whose key centroids stay below 2^17). KV head 0 sits just inside
    that range (FP64); KV heads 1 and 3 reach it and are handed to the int64
    body. Both give the oracle's bits."""
    rng = np.random.default_rng(21)
    T = 3000
    pc = _pc(capacity=T)
    k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
    pc.ingress(np.zeros(T, np.int32), k, v)
    orc = make_oracle()
    rows = orc.ingress_rows(k, v, threads=8)
    q = rng.integers(-(1 << 20), 1 << 20, size=(1, 32, 64)).astype(np.int64)
    q[0, 0:4, 5] = (1 << 30) - 1
    q[0, 0:4, 6] = -((1 << 30) - 1)
    q[0, 4:8, 9] = -(1 << 30)
    q[0, 13, 40] = (1 << 30) + 12345
    out, st = pc.scan([0], torch.from_numpy(q.astype(np.int32)))
    pc.status()
    want, wst = orc.decode_layer(q, [rows], threads=8)
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
    # the two items past the limit went to the int64 body (head 0 may join
    # them for its score spread, which passes 2^32 below the block maxima)
    assert pc.recomputed() >= 2
    # ins_scores on both paths: head 0 in FP64, head 3 in int64
    from insitu_b200 import KVQuantizer, QuantConfig
    kvq = KVQuantizer(64, QuantConfig(key_bits=4, value_bits=2))
    for h in (0, 3):
        kv = kvq.unpack(rows[:, h])
        s, ovf = pc.scores(0, h, torch.from_numpy(q[0, 4 * h:4 * h + 4].astype(np.int32)))
        ws, wovf = orc.scores(q[0, 4 * h:4 * h + 4], kv.k_idx, kv.k_norm)
        np.testing.assert_array_equal(_np(s), ws)
        assert int(_np(ovf)[0]) == wovf


@pytest.mark.parametrize("groups", [1, 2, 4, 8])
@pytest.mark.parametrize("tiles", ["large", "small"])
@pytest.mark.parametrize("kernel", ["fused", "split"])
def test_both_tile_sizes_match_oracle(groups, tiles, kernel):
    """The scan's two tile sizes (4 or 2 rows per thread; "auto" picks by
    context) give the oracle's bits, for a ragged batch with one sequence of
    rising keys whose running maximum moves across tile boundaries."""
    rng = np.random.default_rng(17 + groups)
    lens = [0, 1, 511, 1024, 1025, 3000, 6000]
    B = len(lens)
    pc = _pc(n_kv=8, groups=groups, max_seqs=B, capacity=6144)
    pc.set_tiles(tiles)
    pc.set_scan_kernel(kernel)
    orc = make_oracle()
    caches = []
    for b, T in enumerate(lens):
        if b == B - 1:
            kk, _ = _rising_keys(T, 97, rng)
            k = np.stack([kk] * 8, axis=1)
        else:
            k = _wire(rng, (T, 8, 64))
        v = _wire(rng, (T, 8, 64))
        if T:
            pc.ingress(np.full(T, b, np.int32), k, v)
        caches.append(orc.ingress_rows(k, v, threads=8) if T else np.zeros((0, 8, 52), np.uint8))
    q = _wire(rng, (B, 8 * groups, 64), 1.0 / 8.0)
    q_rot = orc.rotate(q)
    out, st = pc.scan(np.arange(B), torch.from_numpy(q_rot.astype(np.int32)))
    pc.status()
    want, wst = orc.decode_layer(q_rot, caches, threads=8)
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
    assert wst[B - 1, :, 1].sum() > 8                   # rescales in the rising sequence


# -- error behaviour -------------------------------------------------------------

def test_capacity_overflow_raises_and_changes_nothing():
    from insitu_b200._lib import CapacityError
    pc = _pc(capacity=256)
    rng = np.random.default_rng(1)
    pc.ingress(np.zeros(250, np.int32), _wire(rng, (250, 8, 64)), _wire(rng, (250, 8, 64)))
    with pytest.raises(ValueError):
        pc.ingress(np.zeros(10, np.int32), _wire(rng, (10, 8, 64)), _wire(rng, (10, 8, 64)))
    with pytest.raises(CapacityError):
        pc.ingress(np.zeros(7, np.int32), _wire(rng, (7, 8, 64)), _wire(rng, (7, 8, 64)))
    assert pc.length(0) == 250
    pc.ingress(np.zeros(6, np.int32), _wire(rng, (6, 8, 64)), _wire(rng, (6, 8, 64)))
    assert pc.length(0) == 256


def test_wire_value_outside_24_bits_is_reported():
    from insitu_b200._lib import RangeError
    pc = _pc(n_kv=1, groups=1)
    k = np.zeros((1, 1, 64), np.int32)
    k[0, 0, 5] = 1 << 23
    pc.ingress([0], k, np.zeros_like(k))
    with pytest.raises(RangeError):
        pc.status()
    pc.status()                     # cleared after reading


def test_reset_returns_pages_and_empties_the_sequence():
    pc = _pc(capacity=512, max_seqs=2)
    rng = np.random.default_rng(3)
    pc.ingress(np.zeros(300, np.int32), _wire(rng, (300, 8, 64)), _wire(rng, (300, 8, 64)))
    pc.reset(0)
    assert pc.length(0) == 0
    out, st = pc.scan([0], torch.zeros((1, 32, 64), dtype=torch.int32))
    assert not _np(out).any() and (_np(st)[..., 0] == 0).all()


# -- the reference-shaped classes ------------------------------------------------

def test_dropin_cache_and_attention_match_oracle(widths):
    from insitu_b200 import CompressedAttention, CompressedCache, QuantConfig
    g = lambda n: widths[f"k4v2_{n}"]
    cache = CompressedCache(1, 64, 128, QuantConfig(key_bits=4, value_bits=2))
    cache.append_rotated(g("k_rot")[:, None, :].astype(np.int32),
                         g("v_rot")[:, None, :].astype(np.int32))
    assert cache.length == g("k").shape[0]
    np.testing.assert_array_equal(cache.buf[:, 0], g("rows"))
    attn = CompressedAttention(cache.quantizer)
    kv = cache.view(0)
    out, st = attn.attend_online(g("q_rot"), kv)
    np.testing.assert_array_equal(out, g("online"))
    assert [st.n_tokens, st.rescale_events, st.score_overflows, st.acc_overflows,
            st.max_abs_score, st.max_abs_acc] == g("online_stats").tolist()
    out, _ = attn.attend_two_pass(g("q_rot"), kv)
    np.testing.assert_array_equal(out, g("two_pass"))
    s, ovf = attn.scores(g("q_rot"), kv)
    np.testing.assert_array_equal(s, g("scores"))
    # a causal prefix, and the host-array path
    pre = kv.select(slice(0, 40))
    host = cache.view_from_buffer(0).select(slice(0, 40))
    a, _ = attn.attend_online(g("q_rot"), pre)
    b, _ = attn.attend_online(g("q_rot"), host)
    orc = make_oracle()
    want, _ = orc.attend_online(g("q_rot"), g("k_idx")[:40], g("k_norm")[:40],
                                g("v_idx")[:40], g("v_norm")[:40])
    np.testing.assert_array_equal(a, want)
    np.testing.assert_array_equal(b, want)
    # KVQuantizer.encode on the device
    kvq = cache.quantizer.encode(g("k_rot"), g("v_rot"))
    np.testing.assert_array_equal(kvq.k_idx, g("k_idx"))
    np.testing.assert_array_equal(kvq.v_norm, g("v_norm"))


# -- the context-parallel scan's hard cases ------------------------------------------

def _rising_keys(T, step, rng):
    """Keys along one direction with a norm that grows every `step` tokens, so
    the running maximum keeps moving across chunk boundaries."""
    base = _wire(rng, (64,), 0.5).astype(np.int64)
    scale = 1.0 + (np.arange(T) // step) * 0.01
    k = np.clip(np.rint(base[None, :] * scale[:, None] / 8), -(1 << 23), (1 << 23) - 1)
    k = k + rng.integers(-40, 40, size=(T, 64))
    return np.clip(k, -(1 << 23), (1 << 23) - 1).astype(np.int32), base


@pytest.mark.parametrize("T,step", [(5000, 97), (3000, 1), (70000, 211)])
@pytest.mark.parametrize("kernel", ["fused", "split"])
def test_rescales_across_chunks_and_fallback(T, step, kernel):
    rng = np.random.default_rng(T + step)
    kk, base = _rising_keys(T, step, rng)
    k = np.stack([kk] * 8, axis=1)
    v = _wire(rng, (T, 8, 64))
    pc = _pc(capacity=T)
    pc.set_scan_kernel(kernel)
    pc.ingress(np.zeros(T, np.int32), k, v)
    orc = make_oracle()
    qr = orc.rotate(np.tile(base[None, None, :] // 4, (1, 32, 1)))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    out, st = pc.scan([0], q_rot)
    pc.status()
    rows = orc.ingress_rows(k, v, threads=8)
    want, wst = orc.decode_layer(qr, [rows], threads=8)
    assert wst[0, :, 1].sum() > 20                      # many rescale events
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
    # repeatable: a second launch reuses the scratch and gives the same bits
    out2, st2 = pc.scan([0], q_rot)
    np.testing.assert_array_equal(_np(out2), want)
    np.testing.assert_array_equal(_np(st2), wst)


# -- failure detection: a bounded wait that runs out ---------------------------------

def test_a_lookback_wait_that_runs_out_is_reported_and_the_context_survives():
    """The single-launch scan's tiles wait (bounded) for words the tiles
    before them publish. Withholding one word -- a flag nothing sets -- makes
    the waits behind it give up after the lowered poll limit: the launch
    still finishes, ins_cache_status reports INS_ETIMEOUT (DeviceTimeout),
    and the next scan on the same context is exact again. Nothing faults."""
    from insitu_b200._lib import DeviceTimeout
    rng = np.random.default_rng(66)
    T = 40000                              # 40 tiles of 1024 rows per item
    pc = _pc(capacity=T)
    k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
    pc.ingress(np.zeros(T, np.int32), k, v)
    orc = make_oracle()
    qr = orc.rotate(_wire(rng, (1, 32, 64), 1.0 / 8.0))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    want, wst = orc.decode_layer(qr, [orc.ingress_rows(k, v, threads=8)], threads=8)
    pc.set_scan_kernel("fused")            # the single-launch scan is the one that waits
    pc.set_wait_test(poll_limit=64, item=3, chunk=5, head=2)
    pc.scan([0], q_rot)
    with pytest.raises(DeviceTimeout):
        pc.status()
    pc.set_wait_test()                     # the defaults: nothing withheld
    out, st = pc.scan([0], q_rot)
    pc.status()
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)


def test_a_staged_row_wait_that_runs_out_is_reported_and_the_context_survives():
    """With the separate launches (the default), the value pass waits, bounded,
    for the bulk copies of each tile's V rows. Announcing one tile's copies 16
    bytes larger than they are leaves its wait nothing to complete on: it
    gives up after the lowered poll limit, the launch finishes, the status is
    INS_ETIMEOUT (DeviceTimeout), and the next scan is exact again. Every copy
    still lands; nothing faults."""
    from insitu_b200._lib import DeviceTimeout
    rng = np.random.default_rng(67)
    T = 40000
    pc = _pc(capacity=T)
    k, v = _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64))
    pc.ingress(np.zeros(T, np.int32), k, v)
    orc = make_oracle()
    qr = orc.rotate(_wire(rng, (1, 32, 64), 1.0 / 8.0))
    q_rot = torch.from_numpy(qr.astype(np.int32))
    want, wst = orc.decode_layer(qr, [orc.ingress_rows(k, v, threads=8)], threads=8)
    pc.set_scan_kernel("split")
    pc.set_wait_test(poll_limit=64, item=3, chunk=5, head=0)
    pc.scan([0], q_rot)
    with pytest.raises(DeviceTimeout):
        pc.status()
    pc.set_wait_test()
    out, st = pc.scan([0], q_rot)
    pc.status()
    np.testing.assert_array_equal(_np(out), want)
    np.testing.assert_array_equal(_np(st), wst)
