"""The .ecq containers on the host: v2 (packed tiles) write/read round trips
and the reference's v1 files (tests/golden/v1_two_tensors.ecq, written by the
reference's ModelCompressor)."""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle

import ecq_b200 as ecq
from ecq_b200 import container
from ecq_b200 import synthetic as syn


def test_reference_normaliser_restatement():
    z = np.load(GOLDEN / "tables.npz")
    for counts, freq in zip(z["counts"], z["freq"]):
        assert np.array_equal(ecq.RANSTable.from_counts_reference(counts).freq, freq)


def test_v2_roundtrip(tmp_path):
    w1 = syn.student_t_weights(40, 512, seed=1).astype(np.float32)
    w2 = syn.student_t_weights(64, 768, seed=2).astype(np.float32)
    t1 = container.compress_weights(w1, 128)
    t2 = container.compress_weights(w2, 64, tile_cols=256)
    t2.meta = {"bias": None, "note": "layer 2"}
    p = tmp_path / "m.ecq"
    container.save_ecq2(p, {"l1.weight": t1, "l2.weight": t2})
    back = container.load_ecq2(p)
    assert list(back) == ["l1.weight", "l2.weight"]
    for name, t in (("l1.weight", t1), ("l2.weight", t2)):
        b = back[name]
        assert (b.enc.rows, b.enc.cols, b.enc.tile_cols, b.group_size) == (t.enc.rows, t.enc.cols, t.enc.tile_cols,
                                                                         t.group_size)
        assert np.array_equal(b.enc.data, t.enc.data)
        assert np.array_equal(b.enc.tile_offset, t.enc.tile_offset)
        assert np.array_equal(b.enc.stream_len, t.enc.stream_len)
        assert np.array_equal(b.scales, t.scales)
        assert np.array_equal(b.enc.table.freq, t.enc.table.freq)
    assert back["l2.weight"].meta["note"] == "layer 2"
    # every tile decodes (oracle) to the quantised symbols
    sym, _ = syn.quantize_symmetric_groups(w1, 128)
    tiles = oracle.encode_matrix_tiles(sym, back["l1.weight"].enc.table.freq, 8, back["l1.weight"].enc.tile_cols)
    for i, (d, l, _) in enumerate(tiles):
        assert back["l1.weight"].enc.tile(i).data == d.tobytes()


def test_v2_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.ecq"
    p.write_bytes(b"ECQ9" + b"\0" * 60)
    with pytest.raises(ValueError):
        container.load_ecq2(p)


def _oracle_v1(t):
    idx, _, _, _ = oracle.decode_interleaved(t.data, [len(t.data)], 1, t.n_elements, t.table.freq)
    return (idx.astype(np.float32) * np.float32(t.scale) + np.float32(t.zero_point)).reshape(t.shape)


def test_v1_reference_layout_and_as_written():
    path = GOLDEN / "v1_two_tensors.ecq"
    z = np.load(GOLDEN / "v1.npz")
    assert int(z["b_reference_raises"]) == 1
    # the recorded offsets: tensor a decodes the wrong bytes (as the reference
    # does), tensor b has no table there (the reference raises)
    ref = container.read_ecq_v1(path, layout="reference")
    assert np.array_equal(_oracle_v1(ref["a"]), z["a_reference"])
    assert not np.allclose(z["a_reference"], z["a_dequant"])
    with pytest.raises(ValueError):
        ref["b"].tile()
    # where the writer put the blocks: both decode to the quantiser's values
    tens = container.read_ecq_v1(path, layout="as_written")
    for name in ("a", "b"):
        assert np.allclose(_oracle_v1(tens[name]), z[f"{name}_dequant"], atol=1e-7)


def _bad_offsets(enc, offs):
    from ecq_b200.codec import EncodedMatrix

    return EncodedMatrix(rows=enc.rows, cols=enc.cols, tile_rows=enc.tile_rows, tile_cols=enc.tile_cols,
                         table=enc.table, data=enc.data[:96].copy(), tile_offset=np.array(offs, dtype=np.uint32),
                         stream_len=enc.stream_len)


def test_inconsistent_tile_offsets_are_rejected_on_the_host(tmp_path):
    # 24 x 512 in 8x512 tiles: 3 tiles. Offsets whose largest step is small but
    # that decrease, or start past 0, or run past a 96-byte blob, would send the
    # kernels' bulk copies outside the data allocation: they must be refused
    # before anything is copied to a device (device="cpu" would fail later).
    from ecq_b200.device import DeviceMatrix

    sym = syn.laplace_symbols(24, 512, b=0.5, seed=4)
    enc = ecq.encode_matrix(sym, group_size=128)
    enc.validate()
    for offs in ([0, 4992, 5008, 96], [32, 64, 96, 96], [0, 64, 32, 96], [0, 32, 64, 128], [0, 40, 64, 96]):
        bad = _bad_offsets(enc, offs)
        with pytest.raises(ValueError):
            bad.validate()
        with pytest.raises(ValueError):
            DeviceMatrix.from_encoded(bad, device="cpu")
    # the same through a v2 file whose offset blob was edited
    p = tmp_path / "m.ecq"
    t = container.PackedTensor(enc=enc, scales=syn.group_scales(24, 512, 128, seed=5), group_size=128)
    container.save_ecq2(p, {"w": t})
    raw = bytearray(p.read_bytes())
    good = enc.tile_offset.astype("<u4").tobytes()
    at = raw.find(good)
    assert at > 0
    raw[at:at + len(good)] = np.array([0, 4992, 5008, enc.data.size], dtype="<u4").tobytes()
    p.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        container.load_ecq2(p)
