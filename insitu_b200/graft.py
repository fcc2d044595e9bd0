"""Drop the GPU layer into a Llama-family transformers model in place of its
attention blocks (the contract of adapters/torch_llama.py:61-253).

    from insitu_b200.graft import graft
    original = graft(model, layers=range(model.config.num_hidden_layers))

A grafted block takes what a decoder layer passes -- hidden_states,
position_ids, past_key_values, ... -- and returns (output, None). RoPE runs
inside (from the block's own table), so position_embeddings is ignored; the
KV cache is the block's own compressed cache on the GPU, and the model's
past_key_values is only advanced (with zeros) so that its length bookkeeping,
which places the next token, stays right. attention_mask is not honoured: the
block is causal by construction, and a batch of more than one sequence is
refused rather than silently attended across.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from .config import FixedFormat, QuantConfig
from .layer import AttentionLayer
from .seam import RopeScaling


class GpuKernelAttention(nn.Module):
    """A Llama attention module's shape around an AttentionLayer."""

    def __init__(self, layer: AttentionLayer, layer_idx: int, n_kv: int, head_dim: int):
        super().__init__()
        self.layer = layer
        self.layer_idx = layer_idx
        self.n_kv, self.head_dim = n_kv, head_dim
        # set by a router: refuse more than one token per call, and report
        # each call (layer index, the layer, its attention output, start and
        # end events on the launching stream)
        self.decode_only = False
        self.observer = None

    def forward(self, hidden_states, *args, **kwargs):
        x = hidden_states
        squeeze = x.dim() == 2
        if squeeze:
            x = x.unsqueeze(0)
        if x.shape[0] != 1:
            raise NotImplementedError(f"batch of {x.shape[0]}: one sequence per grafted block "
                                      "(attention_mask is not honoured)")
        if self.decode_only and x.shape[1] != 1:
            raise RuntimeError(f"layer {self.layer_idx} got {x.shape[1]} tokens at once; this "
                               "route is one token at a time")
        positions = kwargs.get("position_ids")
        if positions is None:
            positions = kwargs.get("cache_position")
        # positions on the GPU go to the seam as they are (checked there, no
        # host read); others are read to the host
        if positions is None:
            pos = None
        elif positions.device.type == "cuda":
            pos = positions.detach().reshape(-1)
        else:
            pos = positions.reshape(-1).detach().numpy().astype(np.int64)
        hook = self.observer
        if hook is not None:
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
        y, merged = self.layer.forward(x[0].float(), pos)
        if hook is not None:
            t1.record()
            hook(self.layer_idx, self.layer, merged, t0, t1)
        cache = kwargs.get("past_key_values")
        if cache is not None:
            filler = torch.zeros((1, self.n_kv, x.shape[1], self.head_dim), dtype=x.dtype, device=x.device)
            try:
                cache.update(filler, filler, self.layer_idx)
            except Exception as e:  # the cache API moves between releases; never silently
                raise RuntimeError(f"could not advance past_key_values for layer {self.layer_idx}; "
                                   "positions after the first token would be wrong") from e
        out = y.to(device=x.device, dtype=hidden_states.dtype)     # (tokens, hidden)
        return (out if squeeze else out[None]), None


def _rope(config):
    params = getattr(config, "rope_parameters", None) or getattr(config, "rope_scaling", None) or {}
    theta = params.get("rope_theta", getattr(config, "rope_theta", 10000.0))
    kind = params.get("rope_type") or params.get("type") or "default"
    if kind == "llama3":
        scaling = RopeScaling(float(params["factor"]), float(params["low_freq_factor"]),
                              float(params["high_freq_factor"]),
                              int(params["original_max_position_embeddings"]))
    elif kind == "default":
        scaling = None
    else:
        raise NotImplementedError(f"RoPE scaling {kind!r} is not modelled")
    return float(theta), scaling


def build_from_layer(attn_module, config, *, quant: QuantConfig | None = None,
                     fmt: FixedFormat | None = None, capacity: int = 4096, layer_idx: int = 0,
                     device=None, decoder=None, seq: int = 0,
                     softmax: str = "two_pass") -> GpuKernelAttention:
    """A GpuKernelAttention from an attention module's weights (W_o is folded).
    ``decoder``/``seq`` place its cache in a shared DecodeAttention's slot."""
    w = lambda n: getattr(attn_module, f"{n}_proj").weight.detach().float().cpu().numpy()

    def b(n):
        lin = getattr(attn_module, f"{n}_proj")
        return None if lin.bias is None else lin.bias.detach().float().cpu().numpy()

    def gain(n):
        mod = getattr(attn_module, n, None)
        return None if mod is None else mod.weight.detach().float().cpu().numpy()

    hq, hk = config.num_attention_heads, config.num_key_value_heads
    d = getattr(config, "head_dim", None) or config.hidden_size // hq
    theta, scaling = _rope(config)
    eps = getattr(getattr(attn_module, "q_norm", None), "variance_epsilon",
                  getattr(config, "rms_norm_eps", 1e-6))
    layer = AttentionLayer(w("q"), w("k"), w("v"), w("o"), hidden=config.hidden_size, num_heads=hq,
                           num_kv_heads=hk, head_dim=d, quant=quant, fmt=fmt, rope_theta=theta,
                           max_position=getattr(config, "max_position_embeddings", 4096),
                           rope_scaling=scaling, q_norm=gain("q_norm"), k_norm=gain("k_norm"),
                           norm_eps=eps, biases=(b("q"), b("k"), b("v"), b("o")), capacity=capacity,
                           device=device, decoder=decoder, seq=seq, softmax=softmax)
    return GpuKernelAttention(layer, layer_idx, hk, d)


def graft(model, layers, *, slots: dict | None = None, **kw) -> dict:
    """Replace model.model.layers[i].self_attn for each i; returns the
    replaced modules (for ungraft). ``slots`` maps a layer to its sequence
    slot in a shared ``decoder=`` passed through ``kw``."""
    original = {}
    for i in layers:
        blk = model.model.layers[i]
        original[i] = blk.self_attn
        extra = {} if slots is None else {"seq": slots[i]}
        blk.self_attn = build_from_layer(blk.self_attn, model.config, layer_idx=i, **extra, **kw)
    return original


def ungraft(model, original: dict) -> None:
    for i, module in original.items():
        model.model.layers[i].self_attn = module
