"""Every grafted layer's attention on the GPU, one token at a time, with an
optional per-step agreement check (the contract of host/fpga_layers.py:90-284).

    from insitu_b200.router import GpuLayers
    route = GpuLayers(model, layers=range(16), capacity=4096, verify=check)
    ... feed the prompt one token at a time, then generate ...
    print(route.summary())

One cache pool, one slot per layer: the layers' compressed caches are the
sequences of a single DecodeAttention (layer L is sequence slot
``layers.index(L)``), so sixteen layers cost one page pool and one set of
tables rather than sixteen -- the GPU form of the reference's sixteen
``cache_base`` addresses into one DDR (host/fpga_layers.py:118-124).

The route is decode-only by default, as the reference's is (fpga_layers.py:
191-200): a call with more than one token raises rather than running, so a
prompt has to be fed token by token and every cached row is written by the
same ingress kernel a generated token takes. ``decode_only=False`` lets a
prefill chunk through the same cache instead.

The softmax is the online one, which is what the reference's board runs and
what its check compares against (``out_online``, fpga_layers.py:236-246).

``verify`` is a callable ``check(layer, wq, wk, wv) -> expected`` given the
step's wire (q (n, Hq, d), k and v (n, n_kv, d), int32 Q8.16 on the host) and
returning the attention output a host implementation of the below-the-seam
half computes for it ((n, Hq, d) or (n, Hq*d) integers). With it, every step
is compared channel by channel and counted as agreeing or not; without it
nothing is recomputed on the host, and a call does not wait for the GPU: its
events and statistics are read in batches (``drain()``, which ``summary()``
and ``close()`` call), so the counters are current after a drain. The router itself never computes on the
CPU: the check is whatever the caller supplies (the reference's own numpy
kernel, or a test's oracle).
"""

from __future__ import annotations

import numpy as np
import torch

from .config import FixedFormat, Geometry, QuantConfig
from .decode import DecodeAttention
from .graft import graft, ungraft

# the reference's bitstream is built for 4-bit keys and 2-bit values
# (fpga_layers.py:28-30); the GPU path takes any codebook pair it supports
DEFAULT_KEY_BITS = 4
DEFAULT_VALUE_BITS = 2


class RouteCounters:
    """What a route did, so a run can say what happened rather than that it
    finished (the counters and summary of host/fpga_layers.py:125-134,
    258-284). Host logic only."""

    def __init__(self, n_layers: int, verified: bool):
        self.n_layers, self.verified = n_layers, verified
        self.steps = 0            # layer calls
        self.tokens = 0           # tokens through those calls
        self.agree = 0
        self.disagree = 0
        self.dev_ms = 0.0         # CUDA-event time of the layer calls
        self.rescales = 0         # running-max rescales of the online softmax
        self.overflows = 0        # score + accumulator saturations
        self.clips = 0            # wire values saturated at the seam
        self.flagged = 0          # calls with a saturation or overflow

    def add_call(self, n_tokens: int, dev_ms: float, stats, clips: int) -> None:
        """One layer call: its tokens, device time, scan statistics (n, n_kv, 6)
        in AttentionStats order, and the seam's saturated-value count."""
        st = np.asarray(stats)
        over = int(st[..., 2].sum() + st[..., 3].sum())
        self.steps += 1
        self.tokens += n_tokens
        self.dev_ms += dev_ms
        self.rescales += int(st[..., 1].sum())
        self.overflows += over
        self.clips += int(clips)
        if over or clips:
            self.flagged += 1

    def compare(self, got, want):
        """Channel-by-channel agreement; None when equal, else what differs."""
        got, want = np.asarray(got), np.asarray(want)
        want = want.reshape(got.shape[0], -1) if want.size == got.size else want
        got = got.reshape(got.shape[0], -1)
        if got.shape == want.shape and np.array_equal(got, want):
            self.agree += 1
            return None
        self.disagree += 1
        if got.shape != want.shape:
            return f"shape {want.shape} against {got.shape}"
        return f"{int(np.count_nonzero(got != want))} of {got.size} channels"

    def summary(self) -> str:
        if self.steps == 0:
            return "!!! THE GPU WAS NEVER ASKED. No layer call went through this route."
        per = max(self.n_layers, 1)
        lines = [f"decode steps on the GPU: {self.steps} ({self.n_layers} layers x "
                 f"{self.steps // per} calls, {self.tokens} tokens)"]
        if self.verified:
            lines.append(f"  agreement with the check: {self.agree} exact, {self.disagree} different")
        lines.append(f"  device time: {self.dev_ms:.1f} ms total, "
                     f"{self.dev_ms * 1e3 / self.steps:.0f} us/step")
        lines.append(f"  online rescales {self.rescales}, overflows {self.overflows}, "
                     f"seam clips {self.clips}, steps with a range/saturation flag {self.flagged}")
        return "\n".join(lines)


class GpuLayers(RouteCounters):
    """Routes every grafted layer's attention to one GPU cache pool."""

    def __init__(self, model, layers, capacity: int, *, verify=None, quiet: bool = False,
                 trace: bool = False, key_bits: int = DEFAULT_KEY_BITS,
                 value_bits: int = DEFAULT_VALUE_BITS, quant: QuantConfig | None = None,
                 fmt: FixedFormat | None = None, decode_only: bool = True, device=None):
        if verify is not None and not callable(verify):
            raise TypeError("verify is a callable check(layer, wq, wk, wv) -> expected output")
        self.layers = list(layers)
        if not self.layers:
            raise ValueError("no layers to route")
        super().__init__(len(self.layers), verify is not None)
        self.verify, self.quiet, self.trace = verify, quiet, trace
        cfg = model.config
        hq, hk = cfg.num_attention_heads, cfg.num_key_value_heads
        d = getattr(cfg, "head_dim", None) or cfg.hidden_size // hq
        self.quant = quant or QuantConfig(key_bits=key_bits, value_bits=value_bits)
        self.fmt = fmt or FixedFormat()
        self.dec = DecodeAttention(self.quant, self.fmt, Geometry(hk, hq // hk, d),
                                   max_seqs=len(self.layers), capacity=capacity, device=device)
        self.capacity = self.dec.pc.capacity
        self.slots = {L: i for i, L in enumerate(self.layers)}
        self._original = graft(model, self.layers, slots=self.slots, decoder=self.dec,
                               quant=self.quant, fmt=self.fmt, capacity=capacity, device=device,
                               softmax="online")
        self._model = model
        self.mods = {L: model.model.layers[L].self_attn for L in self.layers}
        for m in self.mods.values():
            m.decode_only = decode_only
            m.observer = self._observe
        # without verify or trace a call's events and statistics are kept on
        # the device and read in batches (drain), so a layer call does not
        # wait for the GPU; a kernel's latched error then surfaces at the next
        # drain: summary(), close(), or every DRAIN_EVERY calls
        self._pending = []

    @property
    def bytes_used(self) -> int:
        """Cache bytes the route's layers can hold (capacity rows per layer)."""
        return len(self.layers) * self.capacity * self.dec.geo.n_kv_heads * self.dec.row_bytes

    DRAIN_EVERY = 512

    def _observe(self, L: int, layer, merged: torch.Tensor, t0, t1) -> None:
        if self.verify is None and not self.trace:
            self._pending.append((merged.shape[0], t0, t1, layer.last_stats, layer._last_conv))
            if len(self._pending) >= self.DRAIN_EVERY:
                self.drain()
            return
        self.drain()
        t1.synchronize()
        dt = t0.elapsed_time(t1)
        self.add_call(merged.shape[0], dt, layer.last_stats.cpu().numpy(),
                      layer.last_conversion["n_saturated"])
        self.dec.pc.status()
        token = self.dec.pc.length(self.slots[L])
        if self.trace:
            print(f"    L{L:<2} tok {token:<5} {dt * 1e3:8.1f} us")
        if self.verify is not None:
            wq, wk, wv = (w.cpu().numpy() if torch.is_tensor(w) else np.asarray(w)
                          for w in layer.last_wire)
            bad = self.compare(merged.cpu().numpy(), self.verify(L, wq, wk, wv))
            if bad is not None and not self.quiet:
                print(f"    !! layer {L} token {token}: {bad} differ from the check")

    def drain(self) -> None:
        """Fold the deferred calls into the counters (one sync)."""
        if not self._pending:
            return
        pending, self._pending = self._pending, []
        pending[-1][2].synchronize()
        for n, t0, t1, st, conv in pending:
            self.add_call(n, t0.elapsed_time(t1), st.cpu().numpy(), int(conv[1].item()))
        self.dec.pc.status()

    def summary(self) -> str:
        self.drain()
        return super().summary()

    def reset(self) -> None:
        """Empty every layer's cache (a new sequence)."""
        self.drain()
        self.dec.pc.reset()

    def close(self) -> None:
        """Put the model's own attention modules back and free the pool."""
        if self._original is not None:
            self.drain()
            for m in self.mods.values():
                m.observer = None
            ungraft(self._model, self._original)
            self._original = None
            self.dec.close()
