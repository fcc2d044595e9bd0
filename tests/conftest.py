"""Shared fixtures. GPU tests carry ``@pytest.mark.gpu``; everything else runs on CPU."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def tbvec():
    return golden("tbvec_c64_k4v2.npz")


@pytest.fixture(scope="session")
def widths():
    return golden("widths.npz")


@pytest.fixture(scope="session")
def config1():
    return golden("config1_ctx512.npz")


@pytest.fixture(scope="session")
def ref_tables():
    return golden("tables.npz")


def make_oracle(key_bits=4, value_bits=2, seed=0, rounds=1, d=64, kind="gaussian"):
    """An oracle configured from this package's own tables (pinned separately)."""
    import oracle
    from insitu_b200 import tables as T
    from insitu_b200.config import FixedFormat
    kc, kb = T.codebook(kind, key_bits)
    vc, vb = T.codebook(kind, value_bits)
    table, log2e, _ = T.exp_table(FixedFormat())
    return oracle.Oracle(d=d, key_bits=key_bits, value_bits=value_bits, k_centroids=kc,
                         k_bounds=kb, v_centroids=vc, v_bounds=vb,
                         signs=T.sign_diagonal(d, seed, rounds), exp_table=table, log2e=log2e)


@pytest.fixture(scope="session")
def orc():
    return make_oracle()


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


LONG_T = 32768
LONG_SEEDS = {(4, 2): 3242, (3, 3): 3333}


def long_inputs(kb: int, vb: int, T: int = LONG_T):
    """k, v (T, 8, 64) and q (32, 64) of ``tests/golden/long32k.npz``, from the
    seeds its generator used (numpy PCG64 normals, Q8.16 in 24-bit lanes); the
    fixture's SHA-256 of the packed rows confirms the regeneration."""
    rng = np.random.default_rng(LONG_SEEDS[(kb, vb)])

    def wire(shape, scale=1.0):
        x = np.rint(rng.standard_normal(shape) * scale * 65536.0).astype(np.int64)
        return np.clip(x, -(1 << 23), (1 << 23) - 1)

    k = wire((T, 8, 64))
    v = wire((T, 8, 64))
    q = wire((32, 64), 1.0 / 8.0)
    return k, v, q
