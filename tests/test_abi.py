"""The C ABI and the host-side logic, without a GPU.

The library must load and export every function ``include/insitu_b200.h``
declares; pure host entry points (version, row size, configuration checks)
must answer without touching a device; the host row codec must agree with the
reference's packed rows.
"""

from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "insitu_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ins_[a-z_0-9]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from insitu_b200 import _lib
    L = _lib.lib()
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/insitu_b200.h but not exported"
    assert sorted(_lib.SYMBOLS) == names


def test_no_fallback_when_the_library_is_missing(monkeypatch, tmp_path):
    from insitu_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def _cfg(**kw):
    from insitu_b200 import _lib
    base = dict(head_dim=64, n_kv_heads=8, kv_groups=4, key_bits=4, value_bits=2, norm_bits=16,
                norm_frac=9, qk_frac=16, centroid_frac=15, acc_frac=16, acc_width=32,
                score_width=48, prob_frac=15, exp_lut_bits=8, saturate=1, rot_rounds=1,
                rot_shift=3, rot_inv_sqrt_q15=4096, page_tokens=256, max_seqs=1,
                max_pages_per_seq=4, reserved0=0, n_pages=4)
    base.update(kw)
    return _lib.Config(**base)


def test_host_entry_points_answer_without_a_device():
    from insitu_b200 import _lib
    L = _lib.lib()
    assert L.ins_abi_version() == 1
    assert L.ins_bytes_per_token(C.byref(_cfg())) == 52
    assert L.ins_bytes_per_token(C.byref(_cfg(key_bits=3, value_bits=3))) == 52
    assert L.ins_bytes_per_token(C.byref(_cfg(key_bits=3, value_bits=2))) == 44
    assert L.ins_bytes_per_token(C.byref(_cfg(key_bits=6, value_bits=6))) == 100


@pytest.mark.parametrize("bad", [dict(head_dim=32), dict(kv_groups=3), dict(key_bits=9),
                                 dict(norm_bits=8), dict(page_tokens=100),
                                 dict(centroid_frac=5, norm_frac=2), dict(rot_rounds=9),
                                 dict(max_seqs=0)])
def test_invalid_configs_are_refused_before_any_device_work(bad):
    from insitu_b200 import _lib
    L = _lib.lib()
    h = C.c_void_p()
    tb = _lib.Tables()
    rc = L.ins_cache_create(C.byref(_cfg(**bad)), C.byref(tb), 0, C.byref(h))
    assert rc == _lib.INS_EINVAL
    assert L.ins_last_error()
    assert not h.value


def test_null_handles_are_errors_not_crashes():
    from insitu_b200 import _lib
    L = _lib.lib()
    assert L.ins_cache_destroy(None) == 0
    assert L.ins_ingress(None, 0, None, None, None, None, None, 0, None) == _lib.INS_EINVAL
    assert L.ins_scan(None, 0, None, None, None, None, None, 0, None) == _lib.INS_EINVAL
    assert L.ins_cache_length(None, 0) == -1


def test_row_codec_matches_reference_rows(tbvec, widths):
    from insitu_b200 import KVQuantizer, QuantConfig
    qz = KVQuantizer(64, QuantConfig(key_bits=4, value_bits=2))
    cache = tbvec["cache_rows"]
    np.testing.assert_array_equal(qz.pack(qz.unpack(cache)), cache)
    for kb, vb in ((4, 2), (3, 3), (3, 2), (4, 4), (6, 6), (1, 1)):
        t = f"k{kb}v{vb}"
        qz = KVQuantizer(64, QuantConfig(key_bits=kb, value_bits=vb))
        kv = qz.unpack(widths[f"{t}_rows"])
        np.testing.assert_array_equal(kv.k_idx, widths[f"{t}_k_idx"])
        np.testing.assert_array_equal(kv.v_idx, widths[f"{t}_v_idx"])
        np.testing.assert_array_equal(kv.k_norm, widths[f"{t}_k_norm"])
        np.testing.assert_array_equal(qz.pack(kv), widths[f"{t}_rows"])


def test_config_mirrors_reference_defaults():
    from insitu_b200 import FixedFormat, QuantConfig
    q, f = QuantConfig(), FixedFormat()
    assert (q.key_bits, q.value_bits, q.norm_bits, q.norm_frac, q.rot_rounds) == (3, 2, 16, 9, 1)
    assert f.score_shift_for(QuantConfig(4, 2)) == 24 and f.acc_shift_for(QuantConfig(4, 2)) == 23
    assert QuantConfig(4, 2).bytes_per_token(64) == 52
    with pytest.raises(ValueError):
        QuantConfig(key_bits=0)
