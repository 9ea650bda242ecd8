#!/usr/bin/env python3
"""Generate the golden vectors that pin the oracle (and the CUDA path) to the
reference codec.

Run from the repository root, in a container where the reference is mounted:

    python tests/golden/make_golden.py <path of a drxddy/ecq checkout>

It imports the reference's own ``src/rans.py`` and ``src/interleaved_rans.py``
(drxddy/ecq) and records, for seeded inputs, what they produce:

* tables.npz      RANSTable.from_counts (src/rans.py:39-60) and the
                  to_bytes/from_bytes round trip (src/rans.py:62-71);
* codec.npz       interleaved_rans_encode / interleaved_rans_decode
                  (src/interleaved_rans.py:76-217) for many stream counts and
                  sizes, InterleavedEncodedTile.to_bytes (:63-73), and the
                  single-stream rans_encode (src/rans.py:99-138) for S == 1;
* corrupt.npz     what interleaved_rans_decode returns for damaged tiles
                  (truncated lengths, flipped bytes, short streams);
* c1.npz          the 1024x1024 single-matrix case (Laplace b=0.5, S=4, the
                  reference default), with group-128 scales, x and y = W.x in
                  float64;
* tiled.npz       a matrix cut into 8x256 tiles, each tile's row-major symbols
                  encoded with 32 interleaved streams (the packed format's tile
                  encoding);
* v1_two_tensors.ecq + v1.npz  a two-tensor ".ecq" v1 file written by the
                  reference's ModelCompressor (src/compressed_format.py:109-259),
                  what its ModelDecompressor returns for each tensor (the second
                  raises: the writer's offsets assume interleaved table/data
                  blocks but it writes all tables first), and the dequantised
                  quantize_affine output for each tensor.

Where the reference normaliser gives frequency 0 to a symbol that occurs (its
encoder never terminates on such input), a clamped table (every frequency at
least 1, remainder to the largest) is passed to the reference encoder instead;
the case records which normaliser was used.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from ecq_b200 import synthetic as syn  # noqa: E402


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    from src import rans, interleaved_rans  # type: ignore
    return rans, interleaved_rans


def clamped_freq(counts) -> np.ndarray:
    c = np.maximum(np.asarray(counts), 1).astype(np.float64)
    f = (c / c.sum() * 16384).astype(np.uint32)
    f = np.maximum(f, 1)
    f[np.argmax(f)] += np.int64(16384) - np.int64(f.sum())
    return f.astype(np.uint32)


def make_table(rans, symbols, n=16):
    counts = np.bincount(np.asarray(symbols).reshape(-1), minlength=n)
    t = rans.RANSTable.from_counts(counts)
    present = counts > 0
    if np.any(present & (t.freq == 0)):
        f = clamped_freq(counts)
        cum = np.zeros(n + 1, dtype=np.uint32)
        cum[1:] = np.cumsum(f)
        st = np.zeros(16384, dtype=np.uint8)
        for s in range(n):
            st[cum[s]:cum[s + 1]] = s
        return rans.RANSTable(freq=f, cumfreq=cum, sym_table=st, n_symbols=n), "clamped"
    return t, "reference"


def main(ref_root: str) -> None:
    rans, il = load_reference(ref_root)
    out = Path(__file__).resolve().parent

    # ---------------- tables ----------------
    count_cases = [
        [100, 200, 50, 150, 100, 100, 100, 100, 100, 100, 100, 100, 50, 50, 50, 50],
        [0] * 8 + [20000] + [0] * 7,
        [0] * 16,
        [1] * 16,
        [5, 0, 0, 0, 0, 0, 0, 0, 7, 0, 0, 0, 0, 0, 0, 3],
    ]
    rng = np.random.default_rng(0)
    for b in (0.3, 0.5, 1.0, 2.0, 100.0):
        s = rng.choice(16, size=1 << 20, p=syn.laplace_probs(b))
        count_cases.append(np.bincount(s, minlength=16).tolist())
    counts = np.array(count_cases, dtype=np.uint64)
    freqs, rt_freqs, blobs = [], [], []
    for c in counts:
        t = rans.RANSTable.from_counts(c.astype(np.int64))
        freqs.append(t.freq.astype(np.uint32))
        blob = t.to_bytes()
        blobs.append(np.frombuffer(blob, dtype=np.uint8))
        rt_freqs.append(rans.RANSTable.from_bytes(blob).freq.astype(np.uint32))
    np.savez_compressed(out / "tables.npz", counts=counts, freq=np.array(freqs),
                        roundtrip_freq=np.array(rt_freqs), blob=np.array(blobs))

    # ---------------- codec cases ----------------
    cases = []

    def add(name, symbols, S):
        symbols = np.asarray(symbols, dtype=np.uint8).reshape(-1)
        t, norm = make_table(rans, symbols)
        tile = il.interleaved_rans_encode(symbols, t, n_streams=S)
        dec = il.interleaved_rans_decode(tile)
        assert np.array_equal(dec, symbols), name
        rec = dict(name=name, symbols=symbols, S=S, freq=t.freq.astype(np.uint32),
                   normaliser=norm, data=np.frombuffer(tile.data, dtype=np.uint8),
                   lengths=np.array(tile.stream_lengths, dtype=np.uint32),
                   max_len=tile.max_stream_len)
        if S <= 255:
            rec["to_bytes"] = np.frombuffer(tile.to_bytes(), dtype=np.uint8)
        if S == 1 and symbols.size:
            rec["single"] = np.frombuffer(rans.rans_encode(symbols, t), dtype=np.uint8)
        cases.append(rec)

    lap = syn.laplace_symbols(1, 10000, b=0.5, seed=10).reshape(-1)
    for S in (1, 2, 3, 4, 8, 16, 32, 64, 128, 255):
        add(f"laplace0.5_n10000_S{S}", lap, S)
    add("laplace0.3_n20000_S32", syn.laplace_symbols(1, 20000, b=0.3, seed=11), 32)
    add("laplace1_n5000_S32", syn.laplace_symbols(1, 5000, b=1.0, seed=12), 32)
    add("laplace2_n5003_S32", syn.laplace_symbols(1, 5003, b=2.0, seed=13), 32)
    add("uniform_n4099_S32", np.random.default_rng(14).integers(0, 16, 4099), 32)
    add("uniform_n4096_S4", np.random.default_rng(15).integers(0, 16, 4096), 4)
    add("n1_S4", [8], 4)
    add("n3_S4", [7, 8, 9], 4)
    add("n31_S32", syn.laplace_symbols(1, 31, b=0.5, seed=16), 32)
    add("n33_S32", syn.laplace_symbols(1, 33, b=0.5, seed=17), 32)
    add("constant8_n20000_S4", np.full(20000, 8), 4)
    add("constant3_n1000_S32", np.full(1000, 3), 32)
    add("two_symbols_n3000_S16", np.random.default_rng(18).choice([0, 15], 3000), 16)
    wq, _ = syn.quantize_symmetric_groups(syn.student_t_weights(64, 256, seed=19), 128)
    add("studentt_64x256_S32", wq, 32)
    add("reference_gaussian_minmax_S4",
        np.clip(np.round((lambda r: (r - r.min()) / (r.max() - r.min()) * 15)(np.random.default_rng(42).standard_normal(10000))), 0, 15), 4)

    flat = {}
    for i, c in enumerate(cases):
        for k, v in c.items():
            flat[f"c{i}_{k}"] = np.asarray(v)
    flat["n_cases"] = np.array(len(cases))
    np.savez_compressed(out / "codec.npz", **flat)

    # ---------------- corrupt tiles: what the reference decoder returns ----------------
    base_sym = syn.laplace_symbols(1, 4096, b=0.5, seed=20).reshape(-1)
    t, _ = make_table(rans, base_sym)
    tile = il.interleaved_rans_encode(base_sym, t, n_streams=32)
    corrupt = []

    def add_c(name, data, lengths):
        bad = il.InterleavedEncodedTile(data=bytes(data), stream_lengths=list(map(int, lengths)),
                                        max_stream_len=tile.max_stream_len, n_symbols=tile.n_symbols,
                                        n_streams=32, table=t, original_bytes=tile.original_bytes)
        dec = il.interleaved_rans_decode(bad)
        corrupt.append(dict(name=name, data=np.frombuffer(bytes(data), dtype=np.uint8),
                            lengths=np.array(lengths, dtype=np.uint32), out=dec))

    d0 = bytearray(tile.data)
    L0 = list(tile.stream_lengths)
    add_c("intact", d0, L0)
    L = L0.copy(); L[5] -= 3; L[17] = max(4, L[17] // 2)
    add_c("truncated_lengths", d0, L)
    L = L0.copy(); L[0] = 2; L[31] = 0
    add_c("short_streams", d0, L)
    d = bytearray(d0)
    for p in (40, 41, 300, 555):
        d[p] ^= 0x5A
    add_c("flipped_bytes", d, L0)
    d = bytearray(d0)
    for j in range(32):
        d[j] = 0
    add_c("zero_first_bytes", d, L0)
    flat = {f"k{i}_{k}": np.asarray(v) for i, c in enumerate(corrupt) for k, v in c.items()}
    flat["n_cases"] = np.array(len(corrupt))
    flat["freq"] = t.freq.astype(np.uint32)
    flat["n_symbols"] = np.array(tile.n_symbols)
    flat["max_len"] = np.array(tile.max_stream_len)
    np.savez_compressed(out / "corrupt.npz", **flat)

    # ---------------- C1: 1024x1024 single matrix ----------------
    M = K = 1024
    sym = syn.laplace_symbols(M, K, b=0.5, seed=0)
    sc = syn.group_scales(M, K, 128, seed=1)
    x = syn.activations(1, K, seed=2)
    t, norm = make_table(rans, sym)
    tile = il.interleaved_rans_encode(sym.reshape(-1), t, n_streams=4)
    dec = il.interleaved_rans_decode(tile)
    assert np.array_equal(dec, sym.reshape(-1))
    w = (dec.reshape(M, K).astype(np.float64) - 8.0) * np.repeat(sc.astype(np.float64), 128, axis=1)
    y = (w @ x.astype(np.float64).reshape(-1)).astype(np.float32)
    np.savez_compressed(out / "c1.npz", symbols=sym, scales=sc, x=x, y=y, freq=t.freq.astype(np.uint32),
                        normaliser=norm, data=np.frombuffer(tile.data, dtype=np.uint8),
                        lengths=np.array(tile.stream_lengths, dtype=np.uint32), max_len=tile.max_stream_len,
                        S=4)

    # ---------------- tiled: 8x256 tiles, 32 streams each ----------------
    M, K, R, C = 36, 768, 8, 256
    sym = syn.laplace_symbols(M, K, b=0.5, seed=21)
    t, norm = make_table(rans, sym)
    flat = dict(symbols=sym, freq=t.freq.astype(np.uint32), tile_rows=R, tile_cols=C, S=32)
    i = 0
    for r0 in range(0, M, R):
        for c0 in range(0, K, C):
            blk = sym[r0:r0 + R, c0:c0 + C].reshape(-1)
            tile = il.interleaved_rans_encode(blk, t, n_streams=32)
            flat[f"t{i}_data"] = np.frombuffer(tile.data, dtype=np.uint8)
            flat[f"t{i}_lengths"] = np.array(tile.stream_lengths, dtype=np.uint32)
            i += 1
    flat["n_tiles"] = np.array(i)
    np.savez_compressed(out / "tiled.npz", **flat)
    # ---------------- .ecq v1 container written by the reference ----------------
    from src.compressed_format import CompressedModel, ModelCompressor, ModelDecompressor  # type: ignore
    from src.quantizer import quantize_affine  # type: ignore

    mc = ModelCompressor()
    rng = np.random.default_rng(5)
    metas, tbs, dbs, off = {}, [], [], 0
    expect = {}
    for name, shape in (("a", (48, 64)), ("b", (32, 100))):
        wv = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        meta, tb, db = mc.compress_tensor(name, wv)
        meta.table_offset = off
        off += len(tb)
        meta.data_offset = off
        off += len(db)
        metas[name] = meta
        tbs.append(tb)
        dbs.append(db)
        expect[f"{name}_dequant"] = quantize_affine(wv, bits=4).dequantize().astype(np.float32)
    v1 = out / "v1_two_tensors.ecq"
    mc._write_file(v1, CompressedModel(tensors=metas, data=b"".join(tbs) + b"".join(dbs)))
    md = ModelDecompressor()
    loaded = md.load(v1)
    expect["a_reference"] = md.decompress_tensor(loaded, "a")
    try:
        md.decompress_tensor(loaded, "b")
        expect["b_reference_raises"] = np.array(0)
    except Exception:
        expect["b_reference_raises"] = np.array(1)
    np.savez_compressed(out / "v1.npz", **expect)
    print("golden vectors written to", out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of a drxddy/ecq checkout>")
    main(sys.argv[1])
