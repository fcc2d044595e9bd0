"""ins_scan_noalloc, the scan for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc once they are running (an
engine that gave all of HBM to its own pool at start-up, an allocator that may
not be entered from the decode thread). ins_scan_noalloc serves them with the
same chunked online scan, its scratch carved from a static device array. This
file runs last so that a failure here leaves every other test already run, and
it builds all it needs itself, so it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _pc(max_seqs, capacity):
    from insitu_b200 import FixedFormat, Geometry, PagedCache, QuantConfig
    return PagedCache(QuantConfig(key_bits=4, value_bits=2), FixedFormat(), Geometry(8, 4, 64),
                      max_seqs=max_seqs, capacity=capacity)


def _wire(rng, shape, scale=1.0):
    x = np.rint(rng.standard_normal(shape) * scale * 65536.0)
    return np.clip(x, -(1 << 23), (1 << 23) - 1).astype(np.int32)


def _noalloc(pc, seq_ids, q_rot, lengths=None):
    from insitu_b200 import _lib
    L = _lib.lib()
    B = q_rot.shape[0]
    out = torch.empty((B, 32, 64), dtype=torch.int64, device=pc.device)
    st = torch.empty((B, 8, 6), dtype=torch.int64, device=pc.device)
    ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
    lens = None if lengths is None else np.ascontiguousarray(lengths, dtype=np.int64)
    stream = C.c_void_p(torch.cuda.current_stream(pc.device).cuda_stream)
    rc = L.ins_scan_noalloc(pc._h, B, ids.ctypes.data_as(C.c_void_p),
                            None if lens is None else lens.ctypes.data_as(C.c_void_p),
                            C.c_void_p(q_rot.data_ptr()), C.c_void_p(out.data_ptr()),
                            C.c_void_p(st.data_ptr()), stream)
    _lib.check(rc)
    return out, st


def test_noalloc_scan_equals_scan_on_two_calls_in_a_row():
    rng = np.random.default_rng(31)
    lens = [5000, 1, 2100]
    pc = _pc(max_seqs=3, capacity=6000)
    for b, T in enumerate(lens):
        pc.ingress(np.full(T, b, np.int32), _wire(rng, (T, 8, 64)), _wire(rng, (T, 8, 64)))
    q_rot = pc.rotate(torch.from_numpy(_wire(rng, (3, 32, 64), 1.0 / 8.0)))
    ids = np.arange(3)
    want, want_st = pc.scan(ids, q_rot)
    for call in range(2):
        out, st = _noalloc(pc, ids, q_rot)
        torch.cuda.synchronize(pc.device)
        pc.status()
        assert torch.equal(out, want), f"call {call}: outputs differ"
        assert torch.equal(st, want_st), f"call {call}: stats differ"
    # a causal prefix through both entry points
    pre = [4097, 0, 1000]
    want, want_st = pc.scan(ids, q_rot, lengths=pre)
    out, st = _noalloc(pc, ids, q_rot, lengths=pre)
    assert torch.equal(out, want) and torch.equal(st, want_st)


def test_noalloc_scan_refuses_work_beyond_its_array():
    from insitu_b200._lib import CapacityError
    # 4096 sequences of one token each: 32,768 (sequence, KV head) items,
    # each with its tile and block records, need more than the 192 MiB array
    B = 4096
    pc = _pc(max_seqs=B, capacity=256)
    rng = np.random.default_rng(33)
    pc.ingress(np.arange(B, dtype=np.int32), _wire(rng, (B, 8, 64)), _wire(rng, (B, 8, 64)))
    q_rot = pc.rotate(torch.from_numpy(_wire(rng, (B, 32, 64), 1.0 / 8.0)))
    with pytest.raises(CapacityError, match="scratch"):
        _noalloc(pc, np.arange(B), q_rot)
    # the regular entry point still serves the same scan
    out, _ = pc.scan(np.arange(B), q_rot)
    torch.cuda.synchronize(pc.device)
    assert out.shape == (B, 32, 64)


def test_noalloc_scan_of_a_large_batch_stays_on_the_fast_path():
    """256 sequences of 4K tokens: the rescale-segment pool gets the room the
    rest of the array leaves, so no item is handed to the sequential kernel,
    and the result equals ins_scan's on two calls in a row."""
    rng = np.random.default_rng(35)
    B, T = 256, 4096
    pc = _pc(max_seqs=B, capacity=T)
    g = torch.Generator(device=pc.device)
    g.manual_seed(36)
    for b in range(B):
        kv = (torch.randn((2, T, 8, 64), generator=g, device=pc.device) * 65536.0).round_().clamp_(
            -(1 << 23), (1 << 23) - 1).to(torch.int32)
        pc.ingress(np.full(T, b, np.int32), kv[0], kv[1])
    q_rot = pc.rotate(torch.from_numpy(_wire(rng, (B, 32, 64), 1.0 / 8.0)))
    ids = np.arange(B)
    want, want_st = pc.scan(ids, q_rot)
    for call in range(2):
        before = pc.recomputed_total()
        out, st = _noalloc(pc, ids, q_rot)
        pc.status()
        assert pc.recomputed_total() == before, f"call {call}: items left the fast path"
        assert torch.equal(out, want), f"call {call}: outputs differ"
        assert torch.equal(st, want_st), f"call {call}: stats differ"
