"""Time the reference's own numpy path on this machine's CPU.

Test and measurement infrastructure, not product code. The reference (INSITU's
numpy model) cannot travel to the GPU machine, so its CPU timings are taken
where it is installed and committed as ``cpu_reference_timings.json``;
bench.py reports them beside its live timings of the oracle's C port.

    python tests/golden/time_reference.py --ref /path/to/INSITU

Each timing is one KV head's work at 4 query heads per KV head, the benchmark
geometry (d 64, 4b K / 2b V), on seeded N(0,1) Q8.16 inputs:

* ``attend_online`` (ops/attention.py:451-513), the board's oracle: a Python
  loop over tokens;
* ``attend_two_pass`` (ops/attention.py:429-449): vectorised;
* ``encode`` + ``pack`` (ops/quantize.py:198-252) of rotated k and v.

numpy runs these on one core (elementwise work, no BLAS).
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from make_golden import _import_reference, _wire  # noqa: E402


def _best(fn, reps):
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--ref", required=True, help="a checkout of the INSITU repository")
    a = ap.parse_args(argv)
    _import_reference(a.ref)
    from kernel.config import FixedFormat, QuantConfig
    from kernel.ops.attention import CompressedAttention
    from kernel.ops.quantize import KVQuantizer

    fmt = FixedFormat()
    quant = QuantConfig(key_bits=4, value_bits=2, seed=0)
    qz = KVQuantizer(64, quant, fmt)
    att = CompressedAttention(qz, fmt, quant)
    rng = np.random.default_rng(2024)
    res = {"machine": platform.processor() or platform.machine(), "cpu_count": os.cpu_count(),
           "numpy": np.__version__, "cores_used": 1, "units": "microseconds per cached token "
           "of one KV head (4 query heads)"}
    for T in (4096, 32768):
        k, v = _wire(rng, (T, 64)), _wire(rng, (T, 64))
        q = _wire(rng, (4, 64), 1.0 / 8.0)
        kr, vr, qr = qz.rotation.apply(k), qz.rotation.apply(v), qz.rotation.apply(q)
        kv = qz.encode(kr, vr)
        reps = 3 if T <= 4096 else 1
        t_on = _best(lambda: att.attend_online(qr, kv), reps)
        t_tp = _best(lambda: att.attend_two_pass(qr, kv), 3)
        t_enc = _best(lambda: qz.pack(qz.encode(kr, vr)), 3)
        res[str(T)] = {"attend_online_us_per_token": round(t_on / T * 1e6, 3),
                       "attend_two_pass_us_per_token": round(t_tp / T * 1e6, 3),
                       "encode_pack_us_per_token": round(t_enc / T * 1e6, 3),
                       "attend_online_GBps": round(52 * T / t_on / 1e9, 6),
                       "attend_two_pass_GBps": round(52 * T / t_tp / 1e9, 6)}
        print(T, res[str(T)], flush=True)
    with open(os.path.join(HERE, "cpu_reference_timings.json"), "w") as f:
        json.dump(res, f, indent=1)
        f.write("\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
