"""A whole layer on the GPU: the W_o fold, and
AttentionLayer.forward against the reference's AttentionKernel.forward on a
small Llama-shaped layer (tests/golden/layer.npz, made by importing the
reference). The integer stages are exact; the four projections are library
GEMMs, so the comparison has a stated tolerance."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden


@pytest.fixture(scope="module")
def layer():
    return golden("layer.npz")


def test_w_o_fold_matches_the_reference(layer):
    from insitu_b200 import QuantConfig
    from insitu_b200.layer import fold_o_proj
    from insitu_b200.rotate import Rotation
    got = fold_o_proj(layer["fold_in"].astype(np.float64),
                      Rotation.for_quant(QuantConfig(key_bits=4, value_bits=2, seed=0), 64), 4, 64)
    np.testing.assert_allclose(got, layer["fold_out"], rtol=0, atol=1e-15)
    folded = fold_o_proj(layer["w_o"].astype(np.float64),
                         Rotation.for_quant(QuantConfig(key_bits=4, value_bits=2, seed=0), 64), 4, 64)
    # the reference folded the float32 original; folding its fp16 copy lands
    # within one fp16 rounding of the same matrix
    assert np.abs(folded - layer["w_o_folded"].astype(np.float64)).max() < 2e-3


@pytest.mark.gpu
def test_layer_integer_and_float_halves_match_attention_kernel(layer):
    """From the reference's wire, the cache and scan give its attention output
    exactly; from that output, W_o' gives its y within float32 rounding."""
    torch = pytest.importorskip("torch")
    from insitu_b200 import AttentionLayer
    from insitu_b200.seam import project
    L = AttentionLayer(layer["w_q"], layer["w_k"], layer["w_v"], layer["w_o_folded"], hidden=256,
                       num_heads=4, num_kv_heads=2, rope_theta=500000.0, max_position=4096,
                       o_folded=True, capacity=64)
    n = layer["x"].shape[0]
    for i in range(n):
        out, _ = L.dec.step(layer["wire_q"][i:i + 1].astype(np.int32),
                            layer["wire_k"][i:i + 1].astype(np.int32),
                            layer["wire_v"][i:i + 1].astype(np.int32), mode="two_pass")
        np.testing.assert_array_equal(out.cpu().numpy().reshape(-1), layer["out"][i], err_msg=f"step {i}")
    L.dec.pc.status()
    acc = torch.from_numpy(layer["out"].astype(np.float64) / 65536.0).cuda()
    y = project(L.w_o, acc).cpu().numpy()
    assert np.abs(y - layer["y"]).max() <= 1e-5 * max(1.0, float(np.abs(layer["y"]).max()))
    L.close()


@pytest.mark.gpu
def test_layer_forward_matches_attention_kernel(layer):
    """x to y on the GPU, projections included: the wire within one LSB, y
    within a tolerance for the lanes those LSBs move."""
    pytest.importorskip("torch")
    from insitu_b200 import AttentionLayer
    L = AttentionLayer(layer["w_q"], layer["w_k"], layer["w_v"], layer["w_o_folded"], hidden=256,
                       num_heads=4, num_kv_heads=2, rope_theta=500000.0, max_position=4096,
                       o_folded=True, capacity=64)
    n = layer["x"].shape[0]
    ys, wires = [], []
    for i in range(n):
        y, _ = L.forward(layer["x"][i:i + 1])
        ys.append(y.cpu().numpy()[0])
        wires.append(np.concatenate([w.cpu().numpy().reshape(-1) for w in L.last_wire]))
    L.dec.pc.status()
    want_wire = np.concatenate([layer["wire_q"].reshape(n, -1), layer["wire_k"].reshape(n, -1),
                                layer["wire_v"].reshape(n, -1)], axis=1)
    dw = np.abs(np.stack(wires).astype(np.int64) - want_wire)
    # fp32 GEMMs in another summation order move a wire lane by at most one
    # Q8.16 LSB, and rarely
    assert dw.max() <= 1 and (dw == 0).mean() > 0.97
    y = np.stack(ys)
    err = np.abs(y - layer["y"]).max() / max(1.0, float(np.abs(layer["y"]).max()))
    assert err <= 1e-2, f"relative error {err}"
    L.close()
