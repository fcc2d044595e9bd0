"""The layer router (host/fpga_layers.py:90-284): every layer of a small
transformers Llama routed through one GPU cache pool, the prompt fed one token
at a time, each step checked against the oracle's below-the-seam half on the
step's own wire. A mistake planted in the check must be counted, more than one
token per call must be refused, and the shared pool must give the same logits
as one cache per layer."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, make_oracle

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=3, num_attention_heads=4,
           num_key_value_heads=2, head_dim=64, vocab_size=512, max_position_embeddings=512,
           rope_parameters={"rope_type": "default", "rope_theta": 500000.0})


class OracleCheck:
    """The host half a verify run compares with: rows appended per step, the
    online scan over them (oracle.decode_layer)."""

    def __init__(self, key_bits, value_bits, plant_at=None):
        self.orc = make_oracle(key_bits=key_bits, value_bits=value_bits)
        self.rows = {}
        self.calls = 0
        self.plant_at = plant_at

    def __call__(self, L, wq, wk, wv):
        assert wq.shape[0] == 1
        new = self.orc.ingress_rows(wk, wv)
        self.rows[L] = new if L not in self.rows else np.concatenate([self.rows[L], new])
        want, _ = self.orc.decode_layer(self.orc.rotate(wq), [self.rows[L]])
        self.calls += 1
        if self.calls == self.plant_at:
            want = want.copy()
            want.reshape(-1)[5] += 1
        return want


def _model():
    import torch
    import transformers
    torch.manual_seed(0)
    return transformers.LlamaForCausalLM(transformers.LlamaConfig(**CFG)).eval()


def _run(model, prompt, n_gen, device="cpu"):
    """Prompt one token at a time, then greedy decode; logits of every step."""
    import torch
    import transformers
    cache = transformers.DynamicCache()
    logits = []
    ids = lambda t: torch.tensor([[int(t)]], device=device)
    with torch.no_grad():
        for t in prompt:
            out = model(input_ids=ids(t), past_key_values=cache, use_cache=True)
            logits.append(out.logits[0, -1].cpu().numpy())
        for _ in range(n_gen):
            nxt = int(out.logits[0, -1].argmax())
            out = model(input_ids=ids(nxt), past_key_values=cache, use_cache=True)
            logits.append(out.logits[0, -1].cpu().numpy())
    return np.stack(logits)


@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3)])
def test_router_agrees_with_the_oracle_every_step(kb, vb):
    torch = pytest.importorskip("torch")
    pytest.importorskip("transformers")
    from insitu_b200.router import GpuLayers
    prompt = golden("graft.npz")["prompt"][0]
    model = _model()
    check = OracleCheck(kb, vb)
    route = GpuLayers(model, layers=range(3), capacity=64, verify=check, quiet=True,
                      key_bits=kb, value_bits=vb)
    assert "NEVER ASKED" in route.summary()
    n_gen = 6
    _run(model, prompt, n_gen)
    calls = 3 * (len(prompt) + n_gen)
    assert route.steps == calls == check.calls
    assert (route.agree, route.disagree) == (calls, 0)
    assert route.tokens == calls and route.dev_ms > 0
    for i in range(3):
        assert route.dec.pc.length(i) == len(prompt) + n_gen
    assert f"{calls} exact, 0 different" in route.summary()
    # the pool holds one slot per layer and nothing else
    assert route.dec.pc.max_seqs == 3
    # a prefill chunk is refused, not run: nothing changes
    with pytest.raises(RuntimeError, match="tokens at once"), torch.no_grad():
        model(input_ids=torch.tensor([[1, 2]]))
    assert route.steps == calls
    route.close()
    assert isinstance(model.model.layers[0].self_attn,
                      __import__("transformers").models.llama.modeling_llama.LlamaAttention)


def test_router_counts_a_planted_disagreement():
    pytest.importorskip("transformers")
    from insitu_b200.router import GpuLayers
    prompt = golden("graft.npz")["prompt"][0][:4]
    model = _model()
    route = GpuLayers(model, layers=[0, 2], capacity=32, verify=OracleCheck(4, 2, plant_at=5),
                      quiet=True)
    _run(model, prompt, 0)
    assert route.steps == 2 * len(prompt)
    assert (route.agree, route.disagree) == (route.steps - 1, 1)
    assert "1 different" in route.summary()
    route.close()


def test_shared_pool_equals_one_cache_per_layer():
    """Layers as slots of one pool against the graft's own per-layer caches,
    both with the online softmax, fed the same tokens: identical logits."""
    pytest.importorskip("transformers")
    from insitu_b200 import QuantConfig
    from insitu_b200.graft import graft, ungraft
    from insitu_b200.router import GpuLayers
    prompt = golden("graft.npz")["prompt"][0][:6]
    model = _model()
    route = GpuLayers(model, layers=range(3), capacity=64)
    a = _run(model, prompt, 4)
    assert route._pending, "without verify the calls are read in batches"
    assert "30 (3 layers x 10 calls, 30 tokens)" in route.summary()
    assert route.agree == route.disagree == 0 and route.steps == 30 and not route._pending
    route.close()
    original = graft(model, layers=range(3), quant=QuantConfig(key_bits=4, value_bits=2),
                     capacity=64, softmax="online")
    b = _run(model, prompt, 4)
    ungraft(model, original)
    np.testing.assert_array_equal(a, b)


def test_router_on_a_gpu_resident_model():
    """The model on the GPU: position_ids reach the seam as a device tensor
    (ins_seam_device_positions, no host read). Same tokens as the model on
    the host, logits within float rounding of the GPU's own MLPs."""
    pytest.importorskip("transformers")
    from insitu_b200.router import GpuLayers
    prompt = golden("graft.npz")["prompt"][0][:6]
    host = _model()
    r1 = GpuLayers(host, layers=range(3), capacity=64)
    a = _run(host, prompt, 4)
    r1.close()
    dev = _model().cuda()
    r2 = GpuLayers(dev, layers=range(3), capacity=64, verify=OracleCheck(4, 2), quiet=True)
    b = _run(dev, prompt, 4, device="cuda")
    assert (r2.agree, r2.disagree) == (30, 0)
    r2.close()
    assert (a.argmax(-1) == b.argmax(-1)).all()
    assert np.abs(a - b).max() / np.abs(a).max() < 1e-3
