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
