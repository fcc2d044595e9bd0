"""The GPU layer grafted into a transformers LlamaForCausalLM:
greedy decoding of a seeded random-init small model with every attention block
replaced, against the same model grafted with the reference's own adapter
(tests/golden/graft.npz, made by importing the reference)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
           num_key_value_heads=2, head_dim=64, vocab_size=512, max_position_embeddings=512,
           rope_parameters={"rope_type": "default", "rope_theta": 500000.0})


def test_grafted_model_decodes_like_the_reference_graft():
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    from insitu_b200 import QuantConfig
    from insitu_b200.graft import graft, ungraft
    g = golden("graft.npz")
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(transformers.LlamaConfig(**CFG)).eval()
    original = graft(model, layers=[0, 1], quant=QuantConfig(key_bits=4, value_bits=2, seed=0),
                     capacity=64)
    cache = transformers.DynamicCache()
    logits, toks = [], []
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(g["prompt"]), past_key_values=cache, use_cache=True)
        for _ in range(len(g["tokens"])):
            lg = out.logits[0, -1]
            logits.append(lg.numpy())
            nxt = int(lg.argmax())
            toks.append(nxt)
            out = model(input_ids=torch.tensor([[nxt]]), past_key_values=cache, use_cache=True)
    assert toks == g["tokens"].tolist()
    # the projections are GEMMs summed in another order (a wire lane may move
    # by one Q8.16 LSB): the logits agree to a stated tolerance
    err = np.abs(np.stack(logits) - g["logits"]).max() / np.abs(g["logits"]).max()
    assert err < 1e-2, f"relative logit error {err}"
    for blk in (0, 1):
        model.model.layers[blk].self_attn.layer.dec.pc.status()
    ungraft(model, original)
    assert isinstance(model.model.layers[0].self_attn, transformers.models.llama.modeling_llama.LlamaAttention)
