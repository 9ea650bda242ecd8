"""Host-only checks of bench.py's derived views (no GPU): the integer-issue
roofline of the decode and the committed instruction counts it reads."""
import importlib.util
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_issue_roofline_arithmetic(bench):
    # 32 instructions per 32 symbols: one symbol per lane-instruction, so the
    # ceiling is 4 schedulers x 32 lanes x clock per SM
    shapes = [(64, 512), (128, 256)]
    inst = {"64x512": 64 * 512, "128x256": 128 * 256}
    r = bench.issue_roofline(1e12, shapes, inst, sm_count=148, sm_mhz=2000.0)
    assert r["inst_per_32_symbols"] == pytest.approx(32.0)
    assert r["ceiling_symbols_per_s"] == pytest.approx(148 * 4 * 2e9)
    assert r["frac"] == pytest.approx(1e12 / (148 * 4 * 2e9), rel=1e-3)


def test_issue_roofline_weights_shapes_by_symbols(bench):
    shapes = [(32, 32), (32, 96)]
    inst = {"32x32": 10 * 32, "32x96": 30 * 3 * 32}  # 10 and 30 instructions per 32 symbols
    r = bench.issue_roofline(1.0, shapes, inst, sm_count=1, sm_mhz=1.0)
    assert r["inst_per_32_symbols"] == pytest.approx((10 * 1 + 30 * 3) / 4)


def test_issue_roofline_needs_every_shape(bench):
    assert bench.issue_roofline(1.0, [(8, 8)], {"8x16": 1}, 1, 1.0) is None
    assert bench.issue_roofline(1.0, [(8, 8)], None, 1, 1.0) is None


def test_committed_instruction_counts_cover_the_sweep(bench):
    inst = json.loads((ROOT / "profiles" / "gemv_issue.json").read_text())["inst_executed"]
    r = bench.issue_roofline(0.84e12, bench.SHAPES, inst, sm_count=148, sm_mhz=1965.0)
    assert r is not None
    # the ncu capture counts 24.5-27.4 warp instructions per 32 symbols per shape
    assert 20.0 < r["inst_per_32_symbols"] < 30.0
    assert 0.0 < r["frac"] < 1.0


def test_cpu_baseline_runs_until_its_time_bound(bench):
    # one small matrix through the oracle's decode + dequant + matvec
    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn

    M, K = 64, 1024
    sym = syn.laplace_symbols(M, K, b=0.5, seed=0)
    d = dict(M=M, K=K, sym=sym, scales=syn.group_scales(M, K, bench.GROUP, seed=1),
             x=syn.activations(1, K, seed=2), enc=ecq.encode_matrix(sym, group_size=bench.GROUP))
    gbs, secs, sweeps = bench.cpu_baseline([d], threads=1, repeats=2, min_seconds=0.05)
    assert sweeps >= 2 and secs >= 0.05 and gbs > 0
    gbs1, secs1, sweeps1 = bench.cpu_baseline([d], threads=1, repeats=1)
    assert sweeps1 == 1 and secs1 > 0 and gbs1 > 0


def test_reference_arm_encoding_matches_the_library(bench):
    # the reference arm encodes with the oracle (no libecq); its bytes must be
    # the library's for the same symbols and table
    import numpy as np

    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn

    sym = syn.laplace_symbols(24, 1024, b=0.5, seed=3)
    o = bench.OracleEncoded(sym, 512)
    e = ecq.encode_matrix(sym, group_size=bench.GROUP)
    assert np.array_equal(o.table.freq, e.table.freq)
    assert np.array_equal(o.data, e.data)
    assert np.array_equal(o.tile_offset, e.tile_offset)
    assert np.array_equal(o.stream_len, e.stream_len)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_k_split_shards_cover_the_columns(bench, world):
    # every sweep shape's columns split into contiguous, group-aligned shards,
    # each with a tile width that the kernels support
    from ecq_b200.model import shard_tile_cols

    for M, K in bench.SHAPES:
        edges = [bench._shard_cols(K, world, r) for r in range(world)]
        assert edges[0][0] == 0 and edges[-1][1] == K
        for (a0, a1), (b0, b1) in zip(edges, edges[1:]):
            assert a1 == b0
        for c0, c1 in edges:
            assert c0 % bench.GROUP == 0 and c1 > c0
            tc = shard_tile_cols(M, c1 - c0)
            assert (c1 - c0) % tc == 0 and tc in (128, 256, 512)
