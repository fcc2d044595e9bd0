"""The host half after the projections on the GPU (``ins_seam``): QK-norm, the
attention scale, RoPE and the Q8.16 cast, bit for bit against the reference's
own functions (tests/golden/seam.npz, made by importing the reference), in
both orders of RoPE and cast, with and without QK-norm; the projections as
library GEMMs within float32 rounding."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden


@pytest.fixture(scope="module")
def seam():
    return golden("seam.npz")


def _scaling():
    from insitu_b200.seam import RopeScaling
    return RopeScaling(32.0, 1.0, 4.0, 8192)


def test_rope_tables_match_the_reference_rows(seam):
    from insitu_b200.seam import rope_tables
    cos, sin = rope_tables(64, 1 << 17, 500000.0, 15, _scaling())
    np.testing.assert_array_equal(cos[seam["rope_rows"]], seam["rope_cos_rows"])
    np.testing.assert_array_equal(sin[seam["rope_rows"]], seam["rope_sin_rows"])


@pytest.mark.gpu
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("after", [True, False])
def test_seam_kernel_matches_reference(seam, norm, after):
    torch = pytest.importorskip("torch")
    from insitu_b200 import FixedFormat, Geometry, PagedCache, QuantConfig
    from insitu_b200.seam import Seam
    pc = PagedCache(QuantConfig(key_bits=4, value_bits=2), FixedFormat(), Geometry(8, 4, 64),
                    max_seqs=1, capacity=256)
    sm = Seam(pc, max_position=1 << 17, theta=500000.0, scaling=_scaling(),
              q_norm=seam["q_norm"] if norm else None, k_norm=seam["k_norm"] if norm else None,
              norm_eps=float(seam["eps"][0]), cast_after_rope=after)
    tag = f"n{int(norm)}a{int(after)}"
    for _ in range(2):                      # twice: nothing carries over between calls
        wq, wk, wv, st = sm(seam["q"], seam["k"], seam["v"], seam["pos"])
        np.testing.assert_array_equal(wq.cpu().numpy(), seam[f"wq_{tag}"])
        np.testing.assert_array_equal(wk.cpu().numpy(), seam[f"wk_{tag}"])
        np.testing.assert_array_equal(wv.cpu().numpy(), seam[f"wv_{tag}"])
        assert [st["n_values"], st["n_saturated"]] == list(seam[f"conv_{tag}"])
        assert st["max_abs_float"] == float(seam[f"convmax_{tag}"][0])
    # the wire goes straight into the ingress
    q_rot = pc.ingress(np.zeros(1, np.int32), wk[:1], wv[:1], wq[:1])
    pc.status()
    assert q_rot.shape == (1, 32, 64)
    with pytest.raises(ValueError):
        sm(seam["q"][:1], seam["k"][:1], seam["v"][:1], [1 << 17])
    # positions already on the GPU (ins_seam_device_positions): the same wire
    pos_dev = torch.as_tensor(seam["pos"], dtype=torch.int64, device=pc.device)
    wq, wk, wv, st = sm(seam["q"], seam["k"], seam["v"], pos_dev)
    np.testing.assert_array_equal(wq.cpu().numpy(), seam[f"wq_{tag}"])
    np.testing.assert_array_equal(wk.cpu().numpy(), seam[f"wk_{tag}"])
    np.testing.assert_array_equal(wv.cpu().numpy(), seam[f"wv_{tag}"])
    assert [st["n_values"], st["n_saturated"]] == list(seam[f"conv_{tag}"])
    pc.status()
    # a position beyond the table is caught by the kernel's own bounds check:
    # that token's q and k lanes are zero, v is cast as usual, and the next
    # status call raises
    bad = pos_dev.clone()
    bad[1] = 1 << 17
    wq, wk, wv, _ = sm(seam["q"], seam["k"], seam["v"], bad)
    with pytest.raises(ValueError, match="outside the RoPE table"):
        pc.status()
    assert not wq[1].any() and not wk[1].any()
    np.testing.assert_array_equal(wv.cpu().numpy(), seam[f"wv_{tag}"])
    np.testing.assert_array_equal(wq[0].cpu().numpy(), seam[f"wq_{tag}"][0])
    pc.status()                                  # reported once, then clear


@pytest.mark.gpu
@pytest.mark.parametrize("n,out_dim,in_dim,bias", [(4, 512, 2048, False), (1, 3072, 2048, False),
                                                   (13, 2048, 2048, True), (3, 67, 64, True)])
def test_projection_kernel_within_float32_rounding(n, out_dim, in_dim, bias):
    """ins_project, the library's own projection kernel, against matvec
    (numerics/fp.py:25-46): fp16 operands, fp32 products and sums. The float64
    sum of the same fp16-rounded products is the order-free target; the
    kernel's float32 sums, in its own order, stay within the standard bound
    in_dim * eps * sum |products| (plus the bias's one rounding)."""
    torch = pytest.importorskip("torch")
    from insitu_b200.seam import project
    rng = np.random.default_rng(7 + n)
    w = (rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float32)
    x = rng.standard_normal((n, in_dim)).astype(np.float32)
    b = rng.standard_normal(out_dim).astype(np.float32) if bias else None
    w16, x16 = w.astype(np.float16).astype(np.float64), x.astype(np.float16).astype(np.float64)
    want = x16 @ w16.T + (0.0 if b is None else b.astype(np.float64))
    got = project(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(),
                  None if b is None else torch.from_numpy(b).cuda()).cpu().numpy()
    assert got.dtype == np.float32 and got.shape == (n, out_dim)
    err = np.abs(got.astype(np.float64) - want)
    bound = (in_dim + 1) * np.finfo(np.float32).eps * (np.abs(x16) @ np.abs(w16).T + np.abs(want))
    assert np.all(err <= bound)
