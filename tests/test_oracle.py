"""Pin the CPU oracle to the reference's own answers (no GPU needed).

Everything compared here is either a file the reference ships in
``tb/vectors`` (parsed into ``tbvec_c64_k4v2.npz``) or an output of the
reference's numpy model captured by ``tests/golden/make_golden.py``. Only once
these pass is the oracle trusted as the checker for the CUDA path.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import make_oracle


# -- tables ---------------------------------------------------------------

def test_tables_match_reference(ref_tables):
    from insitu_b200 import tables as T
    from insitu_b200.config import FixedFormat
    for b in range(1, 9):
        for kind in ("gaussian", "uniform"):
            c, bd = T.codebook(kind, b)
            np.testing.assert_array_equal(c, ref_tables[f"{kind}{b}_centroids"])
            np.testing.assert_array_equal(bd, ref_tables[f"{kind}{b}_bounds"])
    tab, log2e, dmax = T.exp_table(FixedFormat())
    np.testing.assert_array_equal(tab, ref_tables["exp_table"])
    assert [log2e, dmax] == ref_tables["exp_consts"][:2].tolist()
    for seed in (0, 1, 7, 12345):
        for r in (1, 2):
            np.testing.assert_array_equal(T.sign_diagonal(64, seed, r),
                                          ref_tables[f"signs_s{seed}_r{r}"])
    np.testing.assert_array_equal(T.sign_diagonal(32, 0, 1), ref_tables["signs_d32_s0_r1"])


def test_sign_word_and_codebooks_match_shipped_vectors(tbvec):
    from insitu_b200 import tables as T
    s = T.sign_diagonal(64, 0, 1)[0]
    word = sum(int(x < 0) << i for i, x in enumerate(s))
    assert word == int(tbvec["rot_signs_word"][0]) == 0x81191FF5899001F8
    kc, kb = T.codebook("gaussian", 4)
    vc, vb = T.codebook("gaussian", 2)
    np.testing.assert_array_equal(kc, tbvec["cb_centroids_key"])
    np.testing.assert_array_equal(kb, tbvec["enc_bounds_key"])
    np.testing.assert_array_equal(vc, tbvec["cb_centroids_value"])
    np.testing.assert_array_equal(vb, tbvec["enc_bounds_value"])


# -- ingress --------------------------------------------------------------

def test_rotation_matches_rot_vectors(orc, tbvec):
    for s in ("q", "k", "v"):
        np.testing.assert_array_equal(orc.rotate(tbvec[f"wire_{s}"]), tbvec[f"rot_{s}"])
    np.testing.assert_array_equal(orc.rotate(tbvec["rot_random_in"]), tbvec["rot_random_out"])


def test_isqrt_exact():
    orc = make_oracle()
    rng = np.random.default_rng(3)
    for a in list(rng.integers(0, 1 << 53, 2000)) + [0, 1, 2, 3, 4, (1 << 52) - 1, (1 << 53) - 1]:
        r = orc.isqrt(int(a))
        assert r * r <= a < (r + 1) * (r + 1)
    assert orc.isqrt(-1) == -1


def test_encoder_matches_enc_vectors(orc, tbvec):
    x = tbvec["enc_in"]
    norms = orc.norm_wire(x)
    np.testing.assert_array_equal(norms, tbvec["enc_norm"])
    np.testing.assert_array_equal(orc.encode_plane(x, norms, 0), tbvec["enc_idx_key"])
    np.testing.assert_array_equal(orc.encode_plane(x, norms, 1), tbvec["enc_idx_value"])


def test_rows_match_kv_rows_and_cache_rows(orc, tbvec):
    ki, kn, vi, vn = orc.encode(tbvec["rot_k"], tbvec["rot_v"])
    np.testing.assert_array_equal(orc.pack(ki, kn, vi, vn), tbvec["kv_rows"])
    cache = tbvec["cache_rows"]                                  # (65, 8, 52)
    assert cache.shape == (65, 8, 52)
    np.testing.assert_array_equal(cache[-1], tbvec["kv_rows"])
    back = orc.pack(*orc.unpack(cache))
    np.testing.assert_array_equal(back, cache)


def test_ingress_rows_matches_row_by_row(orc, tbvec):
    rows = orc.ingress_rows(tbvec["wire_k"], tbvec["wire_v"], threads=4)
    np.testing.assert_array_equal(rows, tbvec["kv_rows"])


# -- scores and the exponential ----------------------------------------------

def test_scores_match_scores_hex(orc, tbvec):
    q = tbvec["rot_q"]                                           # (32, 64)
    cache = tbvec["cache_rows"]
    got = []
    for h in range(8):
        ki, kn, _, _ = orc.unpack(cache[:, h])
        s, _ = orc.scores(q[4 * h:4 * h + 4], ki, kn)
        got.append(s)
    np.testing.assert_array_equal(np.concatenate(got), tbvec["scores"])


def test_score_edge_rows_signed_norms(orc, tbvec):
    ki, kn, _, _ = orc.unpack(tbvec["score_edge_rows"])
    assert kn.tolist() == [0, 1, 32767, -32768, -1]
    s, _ = orc.scores(tbvec["rot_q"][:1], ki, kn)
    np.testing.assert_array_equal(s[0], tbvec["score_edge_gold"])


def test_exp_sweep_matches_exp_vectors(orc, tbvec):
    dv = tbvec["exp_in"]
    np.testing.assert_array_equal(orc.exp(dv), tbvec["exp_out"])
    np.testing.assert_array_equal(orc.exp_two_step(dv), tbvec["exp_out"])
    assert orc.exp_delta_max() == 772248
    assert orc.exp(-1)[()] == -1


def test_finalize_matches_fin_vectors(orc, tbvec):
    r, sh = orc.reciprocal(tbvec["fin_l"])
    np.testing.assert_array_equal(r, tbvec["fin_recip"])
    np.testing.assert_array_equal(sh, tbvec["fin_shift"])
    np.testing.assert_array_equal(orc.finalize(tbvec["fin_acc"], tbvec["fin_l"]),
                                  tbvec["fin_out"])


# -- the online recurrence -------------------------------------------------

@pytest.mark.parametrize("prefix,qkey", [("sm", None), ("sm2", "sm2_q")])
def test_online_recurrence_matches_softmax_vectors(orc, tbvec, prefix, qkey):
    q = tbvec["rot_q"][:4] if qkey is None else tbvec[qkey]
    ki, kn, vi, vn = orc.unpack(tbvec["cache_rows"][:, 0])
    _, _, tr = orc.attend_online(q, ki, kn, vi, vn, trace=True)
    for name in ("s", "m", "p", "l", "grew", "factor"):
        np.testing.assert_array_equal(tr[name], tbvec[f"{prefix}_{name}"], err_msg=name)
    np.testing.assert_array_equal(tr["acc"], tbvec[f"{prefix}_acc"])


def test_decode_step_matches_out_online(orc, tbvec):
    q = tbvec["rot_q"]
    cache = tbvec["cache_rows"]
    out, stats = orc.decode_layer(q[None], [cache], threads=4)
    np.testing.assert_array_equal(out.reshape(1, -1), tbvec["out_online"])
    # the two-pass form differs, and matches forward()'s default output
    tp = []
    for h in range(8):
        ki, kn, vi, vn = orc.unpack(cache[:, h])
        tp.append(orc.attend_two_pass(q[4 * h:4 * h + 4], ki, kn, vi, vn)[0])
    np.testing.assert_array_equal(np.concatenate(tp).reshape(1, -1), tbvec["out_two_pass"])
    assert not np.array_equal(tbvec["out_two_pass"], tbvec["out_online"])


# -- every width, stress and saturation ------------------------------------

WIDTHS = ((4, 2), (3, 3), (3, 2), (4, 4), (6, 6), (1, 1))


@pytest.mark.parametrize("kb,vb", WIDTHS)
def test_widths_match_reference(widths, kb, vb):
    orc = make_oracle(kb, vb)
    t = f"k{kb}v{vb}"
    g = lambda n: widths[f"{t}_{n}"]
    assert orc.bytes_per_token == int(g("bytes_per_token")[0])
    kr, vr, qr = orc.rotate(g("k")), orc.rotate(g("v")), orc.rotate(g("q"))
    np.testing.assert_array_equal(kr, g("k_rot"))
    np.testing.assert_array_equal(vr, g("v_rot"))
    np.testing.assert_array_equal(qr, g("q_rot"))
    ki, kn, vi, vn = orc.encode(kr, vr)
    np.testing.assert_array_equal(ki, g("k_idx"))
    np.testing.assert_array_equal(vi, g("v_idx"))
    np.testing.assert_array_equal(kn, g("k_norm"))
    np.testing.assert_array_equal(vn, g("v_norm"))
    rows = orc.pack(ki, kn, vi, vn)
    np.testing.assert_array_equal(rows, g("rows"))
    np.testing.assert_array_equal(orc.ingress_rows(g("k"), g("v")), g("rows"))
    np.testing.assert_array_equal(orc.scores(qr, ki, kn)[0], g("scores"))
    out, st = orc.attend_online(qr, ki, kn, vi, vn)
    np.testing.assert_array_equal(out, g("online"))
    assert list(st) == g("online_stats").tolist()
    out2, st2 = orc.attend_two_pass(qr, ki, kn, vi, vn)
    np.testing.assert_array_equal(out2, g("two_pass"))
    assert list(st2) == g("two_pass_stats").tolist()
    out3, st3 = orc.attend_online_rows(qr, rows)
    np.testing.assert_array_equal(out3, g("online"))
    assert st3 == st


def test_stress_query_recurrence(orc, widths):
    g = lambda n: widths[f"stress_{n}"]
    qr = orc.rotate(g("q"))
    np.testing.assert_array_equal(qr, g("q_rot"))
    ki, kn, vi, vn = orc.unpack(g("rows"))
    out, st, tr = orc.attend_online(qr, ki, kn, vi, vn, trace=True)
    np.testing.assert_array_equal(out, g("online"))
    assert list(st) == g("online_stats").tolist()
    for n in ("s", "m", "p", "l", "grew", "factor"):
        np.testing.assert_array_equal(tr[n], g(n), err_msg=n)
    np.testing.assert_array_equal(tr["acc"], g("acc"))
    grown = tr["grew"].astype(bool)
    assert len(set(tr["factor"][grown].tolist())) >= 8


def test_saturation_clamps_like_the_reference(orc, widths):
    g = lambda n: widths[f"sat_{n}"]
    ki, kn, vi, vn = orc.unpack(g("rows"))
    assert kn.max() > 0 and vn.max() == 32767
    out, st = orc.attend_online(g("q_rot"), ki, kn, vi, vn)
    np.testing.assert_array_equal(out, g("online"))
    assert list(st) == g("online_stats").tolist()
    assert st[3] > 0                                              # acc_overflows
    out2, st2 = orc.attend_two_pass(g("q_rot"), ki, kn, vi, vn)
    np.testing.assert_array_equal(out2, g("two_pass"))
    assert list(st2) == g("two_pass_stats").tolist()


# -- benchmark config 1 --------------------------------------------------------

def test_config1_cache_and_selected_steps(orc, config1):
    wk, wv = config1["wire_k"].astype(np.int64), config1["wire_v"].astype(np.int64)
    rows = orc.ingress_rows(wk, wv, threads=8)                   # (512, 8, 52)
    np.testing.assert_array_equal(rows, config1["cache"])
    for i, step in enumerate(config1["steps"]):
        q = orc.rotate(config1["wire_q"][i].astype(np.int64))   # (32, 64)
        out, _ = orc.decode_layer(q[None], [rows[:step + 1]], threads=8)
        np.testing.assert_array_equal(out.reshape(-1), config1["out_online"][i],
                                      err_msg=f"step {step}")


# -- the board's byte formats (hw/vectors.py, hw/ddr_layout.py) -------------------

def test_ingress_stream_unpacks_to_the_wire_vectors(tbvec):
    """ingress.hex is the decode token's stream: its lanes are wire_q/k/v."""
    import oracle
    q, k, v = oracle.ingress_from_stream(tbvec["ingress_stream"], n_kv=8, groups=4)
    np.testing.assert_array_equal(q, tbvec["wire_q"])
    np.testing.assert_array_equal(k, tbvec["wire_k"])
    np.testing.assert_array_equal(v, tbvec["wire_v"])


def test_host_stream_codec_matches_the_golden_stream(tbvec):
    from insitu_b200 import wire
    s = wire.ingress_stream(tbvec["wire_q"][None], tbvec["wire_k"][None], tbvec["wire_v"][None])
    np.testing.assert_array_equal(s, tbvec["ingress_stream"])
    np.testing.assert_array_equal(wire.unpack_lanes(wire.pack_lanes(tbvec["wire_k"][3]), 24, 64),
                                  tbvec["wire_k"][3])


def test_ddr_image_of_the_golden_cache(tbvec):
    """ddr_image.hex is DdrLayout.image of the 65-row cache at capacity 65."""
    import oracle
    cap, total, head_stride, ports = (int(x) for x in tbvec["ddr_map"])
    img = oracle.ddr_image(tbvec["cache_rows"], 32, 16, cap)
    assert img.size == total == 8 * head_stride and ports == 4
    np.testing.assert_array_equal(img, tbvec["ddr_image"])
    from insitu_b200 import wire
    planes = wire.ddr_planes(((0, 32), (32, 48), (48, 52)))
    for h, t in ((0, 0), (7, 64), (3, 17)):
        np.testing.assert_array_equal(wire.row_at(img, planes, cap, h, t), tbvec["cache_rows"][t, h])


# -- the long-context pin: 32K tokens, every KV group, against the reference's numpy --

@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3)])
def test_oracle_matches_reference_numpy_at_32k(kb, vb):
    """The reference's own attend_online (ops/attention.py:451-513) over 32,768
    tokens in all 8 KV groups (about 45 rescales each) is the fixture; the C
    oracle must give its outputs and statistics bit for bit, from rows whose
    bytes hash to the reference's packed rows."""
    import hashlib
    from conftest import golden, long_inputs
    g = golden("long32k.npz")
    tag = f"k{kb}v{vb}"
    k, v, q = long_inputs(kb, vb)
    orc = make_oracle(kb, vb)
    rows = orc.ingress_rows(k, v, threads=8)
    assert hashlib.sha256(rows.tobytes()).digest() == g[f"{tag}_rows_sha256"].tobytes()
    qr = orc.rotate(q)
    np.testing.assert_array_equal(qr, g[f"{tag}_q_rot"])
    out, st = orc.decode_layer(qr[None], [rows], threads=8)
    np.testing.assert_array_equal(out[0], g[f"{tag}_online"])
    np.testing.assert_array_equal(st[0], g[f"{tag}_online_stats"])
