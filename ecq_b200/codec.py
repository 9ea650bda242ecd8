"""Host-side codec: frequency tables, the interleaved rANS tile type and its
encoder, with the reference's Python interface (drxddy/ecq
src/rans.py:30-71, src/interleaved_rans.py:26-153, :241-256).

Encoding runs in C++ (libecq ``ecq_encode_*_host``) and produces exactly the
reference encoder's bytes; it is the offline half of the path. Decoding is
on the GPU (``ecq_b200.interleaved``).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import List

import numpy as np

from . import _lib
from ._lib import check, lib, ptr

PROB_BITS = 14
PROB_SCALE = 1 << PROB_BITS
RANS_BYTE_L = 1 << 23
NSYM = 16


@dataclass
class RANSTable:
    """Frequency table (src/rans.py:30-71): freq (sums to 16384), cumfreq,
    the 16384-entry slot->symbol table and the symbol count."""

    freq: np.ndarray
    cumfreq: np.ndarray
    sym_table: np.ndarray
    n_symbols: int = NSYM
    normaliser: str = "reference"

    @classmethod
    def from_freq(cls, freq, normaliser: str = "reference") -> "RANSTable":
        f = np.asarray(freq, dtype=np.uint32).copy()
        if f.shape != (NSYM,) or int(f.sum()) != PROB_SCALE:
            raise ValueError("a table needs 16 frequencies summing to 16384")
        cum = np.zeros(NSYM + 1, dtype=np.uint32)
        cum[1:] = np.cumsum(f)
        st = np.repeat(np.arange(NSYM, dtype=np.uint8), f.astype(np.int64))
        return cls(freq=f, cumfreq=cum, sym_table=st, n_symbols=NSYM, normaliser=normaliser)

    @classmethod
    def from_counts(cls, counts) -> "RANSTable":
        """The reference normaliser (src/rans.py:39-60), except where it
        would give frequency 0 to a symbol that occurs: the reference encoder
        never terminates on such input, so every frequency is then raised to
        at least 1 (``normaliser == "clamped"``). Other histograms give the
        reference's table exactly."""
        c = np.ascontiguousarray(np.asarray(counts, dtype=np.uint64))
        if c.shape != (NSYM,):
            raise ValueError("counts must have 16 bins")
        f = np.zeros(NSYM, dtype=np.uint32)
        norm = np.zeros(1, dtype=np.int32)
        check(lib().ecq_table_from_counts(ptr(c), ptr(f), ptr(norm)), "table_from_counts")
        return cls.from_freq(f, "clamped" if norm[0] else "reference")

    @classmethod
    def from_counts_reference(cls, counts) -> "RANSTable":
        """Exactly the reference normaliser (src/rans.py:39-60), including the
        frequency-0 outcome for rare symbols. For reading reference files,
        whose RANSTable.from_bytes re-runs it on the stored frequencies."""
        c = np.maximum(np.asarray(counts, dtype=np.float64), 1.0)
        f = (c / c.sum() * PROB_SCALE).astype(np.uint32)
        f[np.argmax(f)] += np.uint32(PROB_SCALE - int(f.sum()))
        cum = np.zeros(NSYM + 1, dtype=np.uint32)
        cum[1:] = np.cumsum(f)
        st = np.repeat(np.arange(NSYM, dtype=np.uint8), f.astype(np.int64))
        return cls(freq=f, cumfreq=cum, sym_table=st, n_symbols=NSYM, normaliser="reference")

    @classmethod
    def from_symbols(cls, symbols) -> "RANSTable":
        return cls.from_counts(np.bincount(np.asarray(symbols, dtype=np.uint8).reshape(-1), minlength=NSYM))

    def to_bytes(self) -> bytes:
        """``<H n><16H freq>``, as src/rans.py:62-64."""
        return struct.pack(f"<H{NSYM}H", NSYM, *self.freq.tolist())

    @classmethod
    def from_bytes(cls, data: bytes) -> "RANSTable":
        """Inverse of to_bytes. The reference re-normalises the stored
        frequencies (src/rans.py:67-71), which changes any table holding a
        0 frequency; here a stored table that sums to 16384 is used as is."""
        n = struct.unpack("<H", data[:2])[0]
        f = np.array(struct.unpack(f"<{n}H", data[2:2 + 2 * n]), dtype=np.uint32)
        if int(f.sum()) == PROB_SCALE:
            return cls.from_freq(f)
        return cls.from_counts(f)

    def decode_table(self) -> tuple[np.ndarray, int]:
        """16384 packed device entries (slot - cumfreq) | sym << 14 | freq << 18
        and the flags word (ECQ_FLAG_CONSTANT for a single-symbol table)."""
        e = np.zeros(PROB_SCALE, dtype=np.uint32)
        fl = np.zeros(1, dtype=np.uint32)
        check(lib().ecq_build_decode_table(ptr(np.ascontiguousarray(self.freq)), ptr(e), ptr(fl)), "decode table")
        return e, int(fl[0])


@dataclass
class InterleavedEncodedTile:
    """A compressed tile with physically interleaved streams
    (src/interleaved_rans.py:26-73): byte p of stream j at data[j + p*S]."""

    data: bytes
    stream_lengths: List[int]
    max_stream_len: int
    n_symbols: int
    n_streams: int
    table: RANSTable
    original_bytes: int = 0

    @property
    def stream_offsets(self) -> List[int]:
        return list(range(self.n_streams))

    @property
    def compressed_bytes(self) -> int:
        return len(self.data)

    @property
    def compression_ratio(self) -> float:
        return self.original_bytes / self.compressed_bytes if self.compressed_bytes > 0 else float("inf")

    @property
    def bits_per_symbol(self) -> float:
        return (self.compressed_bytes * 8) / self.n_symbols if self.n_symbols > 0 else 0

    def to_bytes(self) -> bytes:
        """Header ``<B S><I n><I max_len><S*I lengths>`` + table + data, as
        src/interleaved_rans.py:63-73 (so, like the reference, S <= 255)."""
        header = struct.pack(f"<BII{self.n_streams}I", self.n_streams, self.n_symbols, self.max_stream_len,
                             *self.stream_lengths)
        return header + self.table.to_bytes() + self.data

    @classmethod
    def from_bytes(cls, blob: bytes) -> "InterleavedEncodedTile":
        """Parse a to_bytes() image (the reference has no parser)."""
        S = blob[0]
        n, ml = struct.unpack_from("<II", blob, 1)
        lens = list(struct.unpack_from(f"<{S}I", blob, 9))
        off = 9 + 4 * S
        table = RANSTable.from_bytes(blob[off:off + 2 + 2 * NSYM])
        off += 2 + 2 * NSYM
        data = bytes(blob[off:off + S * ml])
        if len(data) != S * ml:
            raise ValueError("truncated tile image")
        return cls(data=data, stream_lengths=lens, max_stream_len=ml, n_symbols=n, n_streams=S, table=table,
                   original_bytes=(n * 4 + 7) // 8)


def interleaved_rans_encode(symbols, table: RANSTable, n_streams: int = 4) -> InterleavedEncodedTile:
    """Byte-identical replacement of src/interleaved_rans.py:76-153, in C++."""
    sym = np.ascontiguousarray(np.asarray(symbols).reshape(-1).astype(np.uint8))
    n = sym.size
    S = int(n_streams)
    if S < 1:
        raise ValueError("n_streams must be >= 1")
    if n and int(sym.max()) >= NSYM:
        raise ValueError("symbols must be < 16")
    per = (n + S - 1) // S
    cap = S * (2 * per + 4)
    data = np.zeros(max(cap, 1), dtype=np.uint8)
    lens = np.zeros(S, dtype=np.uint32)
    ml = np.zeros(1, dtype=np.uint32)
    nb = lib().ecq_encode_interleaved_host(ptr(sym), n, S, ptr(np.ascontiguousarray(table.freq, dtype=np.uint32)),
                                           ptr(data), cap, ptr(lens), ptr(ml))
    check(nb, "interleaved_rans_encode")
    return InterleavedEncodedTile(data=data[:nb].tobytes(), stream_lengths=[int(v) for v in lens],
                                  max_stream_len=int(ml[0]), n_symbols=n, n_streams=S, table=table,
                                  original_bytes=(n * 4 + 7) // 8)


class InterleavedRANSEncoder:
    """src/interleaved_rans.py:241-256."""

    def __init__(self, n_streams: int = 4, bits: int = 4):
        if bits != 4:
            raise ValueError("only 4-bit symbols are supported")
        self.n_streams = n_streams
        self.bits = bits

    def encode(self, indices) -> InterleavedEncodedTile:
        indices = np.asarray(indices).reshape(-1)
        return interleaved_rans_encode(indices, RANSTable.from_symbols(indices), self.n_streams)


@dataclass
class EncodedMatrix:
    """Host-side packed matrix (see include/ecq.h ``ecq_matrix_view``):
    tiles of tile_rows x tile_cols, each one 32-stream reference tile."""

    rows: int
    cols: int
    tile_rows: int
    tile_cols: int
    table: RANSTable
    data: np.ndarray          # uint8, all tiles concatenated
    tile_offset: np.ndarray   # uint32 [n_tiles + 1]
    stream_len: np.ndarray    # uint16 [n_tiles * 32]
    extra: dict = field(default_factory=dict)

    @property
    def n_tiles(self) -> int:
        return int(self.tile_offset.size - 1)

    @property
    def max_tile_bytes(self) -> int:
        return int(np.diff(self.tile_offset.astype(np.int64)).max()) if self.n_tiles else 0

    @property
    def compressed_bytes(self) -> int:
        return int(self.data.size)

    @property
    def bits_per_symbol(self) -> float:
        return 8.0 * self.compressed_bytes / (self.rows * self.cols)

    def validate(self) -> None:
        """Reject an inconsistent tile index before anything reaches the
        device. The kernels bulk-copy tile t from data + tile_offset[t] and
        cannot see the blob's length, so offsets from an untrusted file must
        start at 0, never decrease and end inside the data; a tile's size must
        be a whole number of 32-byte stream rows, and the tile and stream
        counts must match the shape. Raises ValueError."""
        if self.tile_rows != _lib.TILE_ROWS or self.tile_cols <= 0 or self.tile_cols % 32 or self.cols % self.tile_cols:
            raise ValueError("unsupported tile shape")
        n_slabs = (self.rows + self.tile_rows - 1) // self.tile_rows
        n_tiles = n_slabs * (self.cols // self.tile_cols)
        off = np.asarray(self.tile_offset).astype(np.int64)
        if off.ndim != 1 or off.size != n_tiles + 1:
            raise ValueError("tile_offset must hold n_tiles + 1 entries")
        if np.asarray(self.stream_len).size != 32 * n_tiles:
            raise ValueError("stream_len must hold 32 entries per tile")
        if off[0] != 0:
            raise ValueError("tile_offset[0] must be 0")
        sizes = np.diff(off)
        if np.any(sizes < 0):
            raise ValueError("tile offsets decrease")
        if np.any(sizes % 32):
            raise ValueError("a tile's size is not a multiple of 32 bytes")
        if int(off[-1]) > int(np.asarray(self.data).size):
            raise ValueError("tile offsets run past the data")

    def tile(self, t: int) -> InterleavedEncodedTile:
        """Tile t as a reference InterleavedEncodedTile."""
        o0, o1 = int(self.tile_offset[t]), int(self.tile_offset[t + 1])
        slabs_k = self.cols // self.tile_cols
        slab = t // slabs_k
        nr = min(self.tile_rows, self.rows - slab * self.tile_rows)
        n = nr * self.tile_cols
        return InterleavedEncodedTile(data=self.data[o0:o1].tobytes(),
                                      stream_lengths=[int(v) for v in self.stream_len[32 * t:32 * t + 32]],
                                      max_stream_len=(o1 - o0) // 32, n_symbols=n, n_streams=32, table=self.table,
                                      original_bytes=(n * 4 + 7) // 8)


def choose_tile_cols(cols: int, group_size: int, prefer: int = 512) -> int:
    """Largest supported tile width (512, 256 or 128 columns) that divides
    cols and is compatible with the group size."""
    for c in (prefer, 512, 256, 128):
        if c > prefer:
            continue
        if cols % c:
            continue
        if group_size < c and c % group_size:
            continue
        if group_size >= c and group_size % c:
            continue
        return c
    raise ValueError(f"no supported tile width for cols={cols}, group_size={group_size}")


def encode_matrix(symbols, table: RANSTable | None = None, tile_rows: int = 8, tile_cols: int | None = None,
                  group_size: int = 128, n_threads: int = 0) -> EncodedMatrix:
    """Encode a row-major [rows, cols] uint8 symbol matrix into the packed
    format over all host threads."""
    sym = np.ascontiguousarray(np.asarray(symbols, dtype=np.uint8))
    if sym.ndim != 2:
        raise ValueError("symbols must be 2-D")
    rows, cols = sym.shape
    if tile_rows != _lib.TILE_ROWS:
        raise ValueError("the packed format uses 8-row tiles")
    if tile_cols is None:
        tile_cols = choose_tile_cols(cols, group_size)
    if table is None:
        table = RANSTable.from_symbols(sym)
    bound = lib().ecq_matrix_encoded_bound(rows, cols, tile_rows, tile_cols)
    check(bound, "encoded bound")
    slabs = (rows + tile_rows - 1) // tile_rows
    n_tiles = slabs * (cols // tile_cols)
    data = np.zeros(bound, dtype=np.uint8)
    offs = np.zeros(n_tiles + 1, dtype=np.uint32)
    lens = np.zeros(n_tiles * 32, dtype=np.uint16)
    total = np.zeros(1, dtype=np.int64)
    check(lib().ecq_encode_matrix_host(ptr(sym), rows, cols, tile_rows, tile_cols,
                                       ptr(np.ascontiguousarray(table.freq, dtype=np.uint32)), int(n_threads),
                                       ptr(data), bound, ptr(offs), ptr(lens), ptr(total)), "encode_matrix")
    return EncodedMatrix(rows=rows, cols=cols, tile_rows=tile_rows, tile_cols=tile_cols, table=table,
                         data=data[: int(total[0])].copy(), tile_offset=offs, stream_len=lens)


def pack_reference_tiles(tiles, rows: int, cols: int, tile_rows: int, tile_cols: int) -> EncodedMatrix:
    """Build the packed format from reference InterleavedEncodedTile objects
    (one per tile, in row-slab-major order, 32 streams each, one shared
    table): the bytes are used unchanged."""
    tiles = list(tiles)
    if not tiles:
        raise ValueError("no tiles")
    table = tiles[0].table
    offs = [0]
    lens = []
    for t in tiles:
        if t.n_streams != 32:
            raise ValueError("packed tiles have 32 streams")
        if not np.array_equal(np.asarray(t.table.freq), np.asarray(table.freq)):
            raise ValueError("all tiles of a matrix share one table")
        if len(t.data) != 32 * t.max_stream_len:
            raise ValueError("tile data size does not match max_stream_len")
        offs.append(offs[-1] + len(t.data))
        lens.extend(int(v) for v in t.stream_lengths)
    tbl = RANSTable.from_freq(np.asarray(table.freq, dtype=np.uint32), getattr(table, "normaliser", "reference"))
    return EncodedMatrix(rows=rows, cols=cols, tile_rows=tile_rows, tile_cols=tile_cols, table=tbl,
                         data=np.frombuffer(b"".join(t.data for t in tiles), dtype=np.uint8).copy(),
                         tile_offset=np.array(offs, dtype=np.uint32), stream_len=np.array(lens, dtype=np.uint16))


def slice_matrix(enc: EncodedMatrix, slab0: int, slab1: int, kt0: int, kt1: int) -> EncodedMatrix:
    """The packed sub-matrix made of row slabs [slab0, slab1) and K-tiles
    [kt0, kt1) of `enc` (same table, same tile bytes). Tensor-parallel ranks
    take their shard this way, so one encoding serves every TP size."""
    nk = enc.cols // enc.tile_cols
    n_slabs = (enc.rows + enc.tile_rows - 1) // enc.tile_rows
    if not (0 <= slab0 < slab1 <= n_slabs and 0 <= kt0 < kt1 <= nk):
        raise ValueError("slice out of range")
    t = (np.arange(slab0, slab1)[:, None] * nk + np.arange(kt0, kt1)[None, :]).reshape(-1)
    o0 = enc.tile_offset[t].astype(np.int64)
    o1 = enc.tile_offset[t + 1].astype(np.int64)
    sizes = o1 - o0
    offs = np.zeros(t.size + 1, dtype=np.int64)
    np.cumsum(sizes, out=offs[1:])
    idx = np.repeat(o0 - offs[:-1], sizes) + np.arange(int(offs[-1]))
    lens = enc.stream_len.reshape(-1, 32)[t].reshape(-1)
    rows = min(slab1 * enc.tile_rows, enc.rows) - slab0 * enc.tile_rows
    return EncodedMatrix(rows=rows, cols=(kt1 - kt0) * enc.tile_cols, tile_rows=enc.tile_rows,
                         tile_cols=enc.tile_cols, table=enc.table, data=enc.data[idx],
                         tile_offset=offs.astype(np.uint32), stream_len=np.ascontiguousarray(lens))


def split_even(n: int, parts: int) -> list[tuple[int, int]]:
    """[lo, hi) ranges splitting n units into `parts` contiguous pieces whose
    sizes differ by at most one (the first n % parts pieces get one more)."""
    base, extra = divmod(n, parts)
    out, lo = [], 0
    for i in range(parts):
        hi = lo + base + (1 if i < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def concat_rows(parts) -> EncodedMatrix:
    """Stack packed matrices that share columns, tile width and table into
    one (e.g. a fused q|k|v projection): their tiles are concatenated in order.
    Every part but the last must have a whole number of 8-row slabs."""
    parts = list(parts)
    p0 = parts[0]
    for q in parts:
        if (q.cols, q.tile_cols, q.tile_rows) != (p0.cols, p0.tile_cols, p0.tile_rows):
            raise ValueError("parts differ in columns or tile shape")
        if not np.array_equal(q.table.freq, p0.table.freq):
            raise ValueError("parts must share one table")
    for q in parts[:-1]:
        if q.rows % q.tile_rows:
            raise ValueError("only the last part may end in a short slab")
    offs = [np.zeros(1, np.int64)]
    base = 0
    for q in parts:
        offs.append(q.tile_offset[1:].astype(np.int64) + base)
        base += int(q.tile_offset[-1])
    return EncodedMatrix(rows=sum(q.rows for q in parts), cols=p0.cols, tile_rows=p0.tile_rows,
                         tile_cols=p0.tile_cols, table=p0.table, data=np.concatenate([q.data for q in parts]),
                         tile_offset=np.concatenate(offs).astype(np.uint32),
                         stream_len=np.concatenate([q.stream_len for q in parts]))
