"""Host half of the product (C++ codec in libecq) against the oracle and the
reference golden vectors. CPU only: no device calls."""
import numpy as np
import pytest

from conftest import GOLDEN, load_cases
from oracle import oracle

import ecq_b200 as ecq
from ecq_b200 import synthetic as syn


@pytest.fixture(scope="module")
def codec_cases():
    return load_cases(GOLDEN / "codec.npz")[0]


def test_table_from_counts_matches_reference_where_safe():
    z = np.load(GOLDEN / "tables.npz")
    for counts, freq in zip(z["counts"], z["freq"]):
        t = ecq.RANSTable.from_counts(counts)
        _, hazard = oracle.table_reference(counts)
        if hazard:
            assert t.normaliser == "clamped"
            assert np.array_equal(t.freq, oracle.table_clamped(counts))
        else:
            assert t.normaliser == "reference"
            assert np.array_equal(t.freq, freq)
        assert int(t.freq.sum()) == 16384


def test_table_bytes_roundtrip():
    z = np.load(GOLDEN / "tables.npz")
    for counts, blob in zip(z["counts"], z["blob"]):
        t = ecq.RANSTable.from_counts(counts)
        if t.normaliser == "reference":
            assert t.to_bytes() == bytes(blob)
        t2 = ecq.RANSTable.from_bytes(t.to_bytes())
        assert np.array_equal(t2.freq, t.freq)


def test_host_encoder_bytes_equal_reference(codec_cases):
    for c in codec_cases:
        t = ecq.RANSTable.from_freq(c["freq"])
        tile = ecq.interleaved_rans_encode(c["symbols"], t, int(c["S"]))
        assert tile.data == bytes(c["data"]), str(c["name"])
        assert tile.stream_lengths == c["lengths"].tolist()
        assert tile.max_stream_len == int(c["max_len"])
        if "to_bytes" in c:
            assert tile.to_bytes() == bytes(c["to_bytes"])
            back = ecq.InterleavedEncodedTile.from_bytes(bytes(c["to_bytes"]))
            assert back.data == tile.data and back.stream_lengths == tile.stream_lengths
            assert back.n_symbols == tile.n_symbols and back.n_streams == tile.n_streams


def test_zero_frequency_symbol_is_an_error_not_a_hang():
    f = np.zeros(16, np.uint32)
    f[8] = 16384
    with pytest.raises(ecq.codec._lib.EcqError):
        ecq.interleaved_rans_encode(np.array([8, 7, 8], np.uint8), ecq.RANSTable.from_freq(f), 4)


def test_encoder_default_handles_laplace_hazard():
    sym = syn.laplace_symbols(1, 50000, b=0.3, seed=5).reshape(-1)
    tile = ecq.InterleavedRANSEncoder(n_streams=8).encode(sym)
    assert tile.table.normaliser == "clamped"
    out, bad, _, _ = oracle.decode_interleaved(tile.data, tile.stream_lengths, 8, sym.size, tile.table.freq)
    assert bad == 0 and np.array_equal(out, sym)


def test_decode_table_entries():
    for b in (0.3, 0.5, 2.0, 100.0):
        t = ecq.RANSTable.from_symbols(syn.laplace_symbols(64, 256, b=b, seed=3))
        e, flags = t.decode_table()
        assert flags == 0
        slot = np.arange(16384)
        sym = (e >> 14) & 15
        f = e >> 18
        bias = e & 16383
        assert np.array_equal(sym, t.sym_table)
        assert np.array_equal(f, t.freq[sym])
        assert np.array_equal(bias, slot - t.cumfreq[sym])


def test_decode_table_constant_flag():
    f = np.zeros(16, np.uint32)
    f[3] = 16384
    _, flags = ecq.RANSTable.from_freq(f).decode_table()
    assert flags & 1 and (flags >> 4) & 15 == 3


def test_matrix_encoder_matches_reference_tiles():
    z = np.load(GOLDEN / "tiled.npz")
    t = ecq.RANSTable.from_freq(z["freq"])
    enc = ecq.encode_matrix(z["symbols"], t, tile_rows=int(z["tile_rows"]), tile_cols=int(z["tile_cols"]),
                            group_size=128)
    assert enc.n_tiles == int(z["n_tiles"])
    for i in range(enc.n_tiles):
        tile = enc.tile(i)
        assert tile.data == bytes(z[f"t{i}_data"])
        assert tile.stream_lengths == z[f"t{i}_lengths"].tolist()


@pytest.mark.parametrize("rows,cols,tc,b", [(36, 768, 256, 0.5), (64, 512, 512, 2.0), (17, 384, 128, 100.0)])
def test_matrix_encoder_matches_oracle(rows, cols, tc, b):
    sym = syn.laplace_symbols(rows, cols, b=b, seed=7)
    t = ecq.RANSTable.from_symbols(sym)
    enc = ecq.encode_matrix(sym, t, tile_rows=8, tile_cols=tc, group_size=128, n_threads=3)
    tiles = oracle.encode_matrix_tiles(sym, t.freq, 8, tc, 32)
    assert enc.n_tiles == len(tiles)
    for i, (data, lens, _) in enumerate(tiles):
        tile = enc.tile(i)
        assert tile.data == data.tobytes() and tile.stream_lengths == lens.tolist()
    # the packer accepts reference-format tiles unchanged
    packed = ecq.pack_reference_tiles([enc.tile(i) for i in range(enc.n_tiles)], rows, cols, 8, tc)
    assert np.array_equal(packed.data, enc.data) and np.array_equal(packed.tile_offset, enc.tile_offset)


def test_choose_tile_cols():
    assert ecq.choose_tile_cols(4096, 128) == 512
    assert ecq.choose_tile_cols(11008, 128) == 256
    assert ecq.choose_tile_cols(4096, 64) == 512
    with pytest.raises(ValueError):
        ecq.choose_tile_cols(100, 128)


def test_split_even():
    """Even partition of K-tiles / row slabs over ranks: contiguous, covering,
    sizes differing by at most one with the larger parts first."""
    from ecq_b200.codec import split_even

    for n in (0, 1, 7, 43, 512):
        for parts in (1, 2, 3, 8):
            r = split_even(n, parts)
            assert len(r) == parts and r[0][0] == 0 and r[-1][1] == n
            sizes = [b - a for a, b in r]
            assert all(r[i][1] == r[i + 1][0] for i in range(parts - 1))
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)


@pytest.mark.parametrize("s0,s1,k0,k1", [(0, 5, 0, 3), (1, 4, 1, 2), (4, 5, 2, 3), (0, 5, 2, 3)])
def test_slice_matrix_is_the_sub_block(s0, s1, k0, k1):
    """A slice of a packed matrix (row slabs x K-tiles, same tile bytes) runs
    through the reference CPU path like the same block of symbols."""
    from ecq_b200.codec import slice_matrix

    rows, cols, tc, g = 36, 768, 256, 128
    sym = syn.laplace_symbols(rows, cols, b=0.5, seed=31)
    sc = syn.group_scales(rows, cols, g, seed=32).astype(np.float32)
    x = syn.activations(1, cols, seed=33).astype(np.float32)
    enc = ecq.encode_matrix(sym, tile_cols=tc, group_size=g)
    part = slice_matrix(enc, s0, s1, k0, k1)
    r0, r1, c0, c1 = s0 * 8, min(s1 * 8, rows), k0 * tc, k1 * tc
    assert (part.rows, part.cols) == (r1 - r0, c1 - c0)
    sub_sc = np.ascontiguousarray(sc[r0:r1, c0 // g:c1 // g])
    y, bad = oracle.gemv_packed(part.data, part.tile_offset, part.stream_len, part.rows, part.cols, 8, tc,
                                enc.table.freq, sub_sc, g, x[:, c0:c1])
    assert bad == 0
    y_ref = oracle.dequant_gemv(sym[r0:r1, c0:c1], sub_sc, g, x[:, c0:c1])[0]
    assert np.allclose(y, y_ref, rtol=1e-5, atol=1e-5)


def test_concat_rows_stacks_matrices():
    """Packed matrices that share columns, tile width and table stack into one
    (the fused q|k|v and gate|up projections)."""
    from ecq_b200.codec import concat_rows

    cols, tc, g = 512, 256, 128
    a = syn.laplace_symbols(16, cols, b=0.5, seed=41)
    b = syn.laplace_symbols(13, cols, b=0.5, seed=42)
    t = ecq.RANSTable.from_symbols(np.concatenate([a, b]))
    enc = concat_rows([ecq.encode_matrix(a, t, tile_cols=tc, group_size=g),
                       ecq.encode_matrix(b, t, tile_cols=tc, group_size=g)])
    both = np.concatenate([a, b])
    assert (enc.rows, enc.cols) == both.shape
    sc = syn.group_scales(*both.shape, g, seed=43).astype(np.float32)
    x = syn.activations(1, cols, seed=44).astype(np.float32)
    y, bad = oracle.gemv_packed(enc.data, enc.tile_offset, enc.stream_len, enc.rows, cols, 8, tc, t.freq, sc, g, x)
    assert bad == 0
    assert np.allclose(y, oracle.dequant_gemv(both, sc, g, x)[0], rtol=1e-5, atol=1e-5)
