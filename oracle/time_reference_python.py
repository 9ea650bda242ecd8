#!/usr/bin/env python3
"""Time the reference's unchanged Python decoder beside the oracle's C port,
on the same tile and one host core.

Run from the repository root, in a container where the reference is mounted
(the reference's Python cannot travel to a machine without it):

    python oracle/time_reference_python.py <path of a drxddy/ecq checkout>

Workload: 1024x1024 symbols, Laplace b = 0.5, one tile of 256 interleaved
streams (the reference's bench shape, src/interleaved_rans.py:220-262), a
clamped table where the reference normaliser would zero a present symbol.
The reference's interleaved_rans_decode (src/interleaved_rans.py:156-217) is
timed on that tile; the oracle's decode_interleaved (oracle/rans_oracle.c)
on the same bytes. Both results are checked against the input symbols.
Prints one JSON line with symbols/s for each and their ratio.
"""
from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests" / "golden"))

from ecq_b200 import synthetic as syn  # noqa: E402
from make_golden import load_reference, make_table  # noqa: E402
from oracle import oracle  # noqa: E402


def _best_of(fn, reps: int) -> float:
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def main(ref_root: str) -> None:
    os.sched_setaffinity(0, {sorted(os.sched_getaffinity(0))[0]})  # one core for both
    rans, il = load_reference(ref_root)
    sym = syn.laplace_symbols(1024, 1024, b=0.5, seed=1).reshape(-1).astype(np.uint8)
    S = 256
    table, norm = make_table(rans, sym)
    tile = il.interleaved_rans_encode(sym, table, n_streams=S)
    out = il.interleaved_rans_decode(tile)
    assert np.array_equal(out, sym)
    t_ref = _best_of(lambda: il.interleaved_rans_decode(tile), 2)

    data = np.frombuffer(tile.data, dtype=np.uint8)
    lengths = np.array(tile.stream_lengths, dtype=np.uint32)
    freq = table.freq.astype(np.uint32)
    got, bad, _, _ = oracle.decode_interleaved(data, lengths, S, sym.size, freq)
    assert bad == 0 and np.array_equal(got, sym)
    t_port = _best_of(lambda: oracle.decode_interleaved(data, lengths, S, sym.size, freq), 5)

    print(json.dumps({
        "workload": "1024x1024 symbols, Laplace b=0.5, 256 interleaved streams, one tile",
        "table": norm,
        "cores": 1,
        "reference_python_sym_per_s": round(sym.size / t_ref),
        "oracle_c_port_sym_per_s": round(sym.size / t_port),
        "port_over_reference": round(t_ref / t_port, 1),
        "bits_per_symbol": round(8 * data.size / sym.size, 3),
    }))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
