"""The CPU oracle against the reference codec's own outputs (golden vectors
written by tests/golden/make_golden.py from the reference's src/rans.py and
src/interleaved_rans.py). These pin the oracle before anything is compared
with it."""
import numpy as np
import pytest

from conftest import GOLDEN, load_cases
from oracle import oracle


def test_table_normaliser_matches_reference():
    z = np.load(GOLDEN / "tables.npz")
    for counts, freq, rt in zip(z["counts"], z["freq"], z["roundtrip_freq"]):
        f, _ = oracle.table_reference(counts)
        assert np.array_equal(f, freq), counts
        # from_bytes re-runs from_counts on the stored freq (src/rans.py:67-71)
        f2, _ = oracle.table_reference(freq.astype(np.uint64))
        assert np.array_equal(f2, rt)
        assert int(f.sum()) == 16384


def test_table_blob_layout():
    z = np.load(GOLDEN / "tables.npz")
    for freq, blob in zip(z["freq"], z["blob"]):
        expect = np.concatenate([np.array([16], "<u2"), freq.astype("<u2")]).view(np.uint8)
        assert np.array_equal(blob, expect)


def test_zero_frequency_hazard_detected():
    z = np.load(GOLDEN / "tables.npz")
    # the Laplace b=0.3 and b=0.5 histograms have present symbols the reference gives freq 0
    hz = [oracle.table_reference(c)[1] for c in z["counts"]]
    assert hz[5] > 0 and hz[6] > 0
    f = oracle.table_clamped(z["counts"][6])
    assert f.min() >= 1 and int(f.sum()) == 16384
    # the clamped table survives the to_bytes/from_bytes round trip unchanged
    f2, bad = oracle.table_reference(f.astype(np.uint64))
    assert bad == 0 and np.array_equal(f2, f)


def test_derived_tables():
    z = np.load(GOLDEN / "tables.npz")
    for freq in z["freq"]:
        cum, st = oracle.table_derive(freq)
        assert cum[0] == 0 and cum[-1] == 16384
        for s in range(16):
            assert np.all(st[cum[s]:cum[s + 1]] == s)


@pytest.fixture(scope="module")
def codec_cases():
    cases, _ = load_cases(GOLDEN / "codec.npz")
    return cases


def test_encode_matches_reference_bytes(codec_cases):
    for c in codec_cases:
        data, lens, ml = oracle.encode_interleaved(c["symbols"], c["freq"], int(c["S"]))
        assert ml == int(c["max_len"]), str(c["name"])
        assert np.array_equal(lens, c["lengths"]), str(c["name"])
        assert np.array_equal(data, c["data"]), str(c["name"])
        if "single" in c:
            # single-stream rans_encode (src/rans.py:99-138) is the S == 1 stream
            assert np.array_equal(data[: int(lens[0])], c["single"])


def test_decode_matches_reference(codec_cases):
    for c in codec_cases:
        n = c["symbols"].size
        out, bad, es, ep = oracle.decode_interleaved(c["data"], c["lengths"], int(c["S"]), n, c["freq"])
        assert np.array_equal(out, c["symbols"]), str(c["name"])
        assert bad == 0
        used = c["lengths"] >= 4
        assert np.all(es[used] == 1 << 23) and np.array_equal(ep[used], c["lengths"][used])


def test_to_bytes_layout(codec_cases):
    import struct

    for c in codec_cases:
        if "to_bytes" not in c:
            continue
        S = int(c["S"])
        hdr = struct.pack(f"<BII{S}I", S, c["symbols"].size, int(c["max_len"]), *c["lengths"].tolist())
        tbl = struct.pack("<H16H", 16, *c["freq"].tolist())
        assert bytes(c["to_bytes"]) == hdr + tbl + bytes(c["data"])


def test_corrupt_tiles_decode_like_reference():
    cases, z = load_cases(GOLDEN / "corrupt.npz", prefix="k")
    n = int(z["n_symbols"])
    for c in cases:
        out, bad, _, _ = oracle.decode_interleaved(c["data"], c["lengths"], 32, n, z["freq"])
        assert np.array_equal(out, c["out"]), str(c["name"])
        assert (bad == 0) == (str(c["name"]) == "intact")


def test_c1_matrix_and_gemv():
    z = np.load(GOLDEN / "c1.npz")
    sym = z["symbols"]
    out, bad, _, _ = oracle.decode_interleaved(z["data"], z["lengths"], int(z["S"]), sym.size, z["freq"])
    assert bad == 0 and np.array_equal(out.reshape(sym.shape), sym)
    y = oracle.dequant_gemv(sym, z["scales"].astype(np.float32), 128, z["x"].astype(np.float32))
    assert np.max(np.abs(y - z["y"])) <= 1e-5 * np.max(np.abs(z["y"]))
    yc = oracle.dequant_gemv_c(sym, z["scales"].astype(np.float32), 128, z["x"].astype(np.float32))
    assert np.max(np.abs(yc - z["y"])) <= 1e-5 * np.max(np.abs(z["y"]))


def test_tiled_encoding_matches_reference():
    z = np.load(GOLDEN / "tiled.npz")
    tiles = oracle.encode_matrix_tiles(z["symbols"], z["freq"], int(z["tile_rows"]), int(z["tile_cols"]), 32)
    assert len(tiles) == int(z["n_tiles"])
    for i, (data, lens, _) in enumerate(tiles):
        assert np.array_equal(data, z[f"t{i}_data"])
        assert np.array_equal(lens, z[f"t{i}_lengths"])
