"""The ``.ecq`` container: the reference's v1 files (read) and the packed v2
format (read/write).

v1 (src/compressed_format.py:22-350, magic ``ECQ1``): a 64-byte header
(magic, u32 version, u32 n_tensors, u64 metadata offset, u64 data offset),
JSON metadata and a data section of 34-byte tables and single-stream rANS
bitstreams; each tensor has one per-tensor scale and zero point. The
reference's writer (:148-259) records offsets for interleaved [table, data]
blocks but writes all tables first, so in a multi-tensor file its own reader
decodes the wrong bytes for the first tensor and finds no table for the
others. ``read_ecq_v1`` follows the recorded offsets by default (the
reference's behaviour, bit for bit); ``layout="as_written"`` reads the blocks
where the writer actually put them.

v2 (magic ``ECQ2``): the packed device format of this package. Header: magic,
u32 version (2), u32 n_tensors, u64 metadata offset, u64 metadata size, u64
data offset, zero padding to 64 bytes. Metadata: UTF-8 JSON
``{"format": "ecq-packed-tiles", "tensors": {name: {...}}}`` with, per tensor,
rows, cols, tile_rows, tile_cols, group_size, streams (32), the 16
frequencies and the normaliser, and the [offset, size] of four blobs relative
to the data offset: the tiles' interleaved stream bytes (each tile is one
reference ``InterleavedEncodedTile.data``), tile_offset (u32, n_tiles + 1),
stream_len (u16, 32 per tile) and the fp16 group scales [rows, cols/g]. Every
blob starts 256-byte aligned, so the file can be memory-mapped and its blobs
copied straight to the device.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .codec import (EncodedMatrix, InterleavedEncodedTile, RANSTable, encode_matrix,
                    choose_tile_cols)
from .synthetic import quantize_symmetric_groups

MAGIC_V1 = b"ECQ1"
MAGIC_V2 = b"ECQ2"
ALIGN = 256


@dataclass
class PackedTensor:
    enc: EncodedMatrix
    scales: np.ndarray  # fp16 [rows, ceil(cols/g)]
    group_size: int
    meta: dict = field(default_factory=dict)

    def to_device(self, device="cuda"):
        import torch

        from .device import DeviceMatrix

        m = DeviceMatrix.from_encoded(self.enc, group_size=self.group_size, device=device)
        sc = np.ascontiguousarray(self.scales)
        if not sc.flags.writeable:  # a memory-mapped blob: torch wants writable host memory
            sc = sc.copy()
        return m, torch.from_numpy(sc).to(device)


def _pad(n: int) -> int:
    return (-n) % ALIGN


def save_ecq2(path, tensors: dict) -> None:
    """Write {name: PackedTensor} as a v2 file."""
    blobs, meta, off = [], {}, 0

    def put(arr: np.ndarray):
        nonlocal off
        b = np.ascontiguousarray(arr).tobytes()
        start = off
        blobs.append(b)
        off += len(b)
        pad = _pad(off)
        if pad:
            blobs.append(b"\0" * pad)
            off += pad
        return [start, len(b)]

    for name, t in tensors.items():
        e = t.enc
        meta[name] = {
            "rows": e.rows, "cols": e.cols, "tile_rows": e.tile_rows, "tile_cols": e.tile_cols,
            "group_size": t.group_size, "streams": 32, "freq": [int(v) for v in e.table.freq],
            "normaliser": e.table.normaliser, "bits_per_symbol": e.bits_per_symbol,
            "data": put(e.data), "tile_offset": put(e.tile_offset.astype("<u4")),
            "stream_len": put(e.stream_len.astype("<u2")), "scales": put(t.scales.astype("<f2")),
            "extra": t.meta,
        }
    md = json.dumps({"format": "ecq-packed-tiles", "tensors": meta}).encode("utf-8")
    meta_off = 64
    data_off = meta_off + len(md) + _pad(meta_off + len(md))
    with open(path, "wb") as f:
        f.write(MAGIC_V2 + struct.pack("<IIQQQ", 2, len(tensors), meta_off, len(md), data_off))
        f.write(b"\0" * (64 - f.tell()))
        f.write(md)
        f.write(b"\0" * (data_off - f.tell()))
        for b in blobs:
            f.write(b)


def load_ecq2(path, mmap: bool = True) -> dict:
    """Read a v2 file into {name: PackedTensor} (memory-mapped blobs)."""
    raw = np.memmap(path, dtype=np.uint8, mode="r") if mmap else np.fromfile(path, dtype=np.uint8)
    head = bytes(raw[:40])
    if head[:4] != MAGIC_V2:
        raise ValueError(f"not an ECQ2 file: magic {head[:4]!r}")
    version, n, meta_off, meta_size, data_off = struct.unpack_from("<IIQQQ", head, 4)
    if version != 2:
        raise ValueError(f"unsupported ECQ2 version {version}")
    md = json.loads(bytes(raw[meta_off:meta_off + meta_size]).decode("utf-8"))
    if md.get("format") != "ecq-packed-tiles":
        raise ValueError("unknown ECQ2 payload format")
    out = {}
    for name, t in md["tensors"].items():
        def blob(key, dtype):
            o, s = t[key]
            return raw[data_off + o:data_off + o + s].view(dtype)
        table = RANSTable.from_freq(np.array(t["freq"], dtype=np.uint32), t.get("normaliser", "reference"))
        rows, cols, g = t["rows"], t["cols"], t["group_size"]
        enc = EncodedMatrix(rows=rows, cols=cols, tile_rows=t["tile_rows"], tile_cols=t["tile_cols"], table=table,
                            data=blob("data", np.uint8), tile_offset=blob("tile_offset", "<u4"),
                            stream_len=blob("stream_len", "<u2"))
        try:
            enc.validate()
        except ValueError as exc:
            raise ValueError(f"{name}: {exc}") from None
        scales = blob("scales", "<f2").reshape(rows, (cols + g - 1) // g)
        out[name] = PackedTensor(enc=enc, scales=scales, group_size=g, meta=t.get("extra", {}))
    if len(out) != n:
        raise ValueError("tensor count does not match the header")
    return out


def compress_weights(weights: np.ndarray, group_size: int = 128, tile_cols: int | None = None) -> PackedTensor:
    """Quantise a float [rows, cols] weight symmetrically per group (absmax/7,
    zero point 8) and encode it into packed tiles with one table."""
    w = np.asarray(weights, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("weights must be 2-D")
    sym, sc = quantize_symmetric_groups(w, group_size)
    tc = tile_cols or choose_tile_cols(w.shape[1], group_size)
    return PackedTensor(enc=encode_matrix(sym, tile_cols=tc, group_size=group_size), scales=sc, group_size=group_size)


def compress_safetensors(input_path, output_path, group_size: int = 128, min_elements: int = 1000) -> dict:
    """Compress every 2-D tensor of a safetensors file with at least
    `min_elements` elements (src/compressed_format.py:148-218 skips tensors
    under 1000 elements too) into a v2 file. Returns {name: bits/weight}."""
    from safetensors import safe_open

    tensors, stats = {}, {}
    with safe_open(str(input_path), framework="np") as f:
        for name in f.keys():
            w = f.get_tensor(name)
            if w.ndim != 2 or w.size < min_elements or w.shape[1] % group_size:
                continue
            try:
                t = compress_weights(w, group_size)
            except ValueError:
                continue
            tensors[name] = t
            stats[name] = t.enc.bits_per_symbol
    save_ecq2(output_path, tensors)
    return stats


# ---------------------------------------------------------------- v1 (reference)
@dataclass
class V1Tensor:
    name: str
    shape: list
    scale: float
    zero_point: float
    n_elements: int
    table: RANSTable | None
    data: bytes
    error: str | None = None  # why the recorded offsets hold no usable table

    def tile(self) -> InterleavedEncodedTile:
        if self.error:
            raise ValueError(f"{self.name}: {self.error}")
        """The single stream as a one-stream interleaved tile (same bytes)."""
        return InterleavedEncodedTile(data=self.data, stream_lengths=[len(self.data)], max_stream_len=len(self.data),
                                      n_symbols=self.n_elements, n_streams=1, table=self.table,
                                      original_bytes=(self.n_elements * 4 + 7) // 8)


def read_ecq_v1(path, layout: str = "reference") -> dict:
    """Parse a reference .ecq v1 file into {name: V1Tensor}.

    layout="reference": blocks at the offsets the metadata records (what the
    reference's ModelDecompressor reads; it raises on tensors whose recorded
    offsets do not hold a table). layout="as_written": all tables first, then
    all bitstreams, in metadata order (where the reference's writer puts them)."""
    raw = Path(path).read_bytes()
    if raw[:4] != MAGIC_V1:
        raise ValueError(f"not an ECQ1 file: magic {raw[:4]!r}")
    version, n = struct.unpack_from("<II", raw, 4)
    meta_off, data_off = struct.unpack_from("<QQ", raw, 12)
    if version != 1:
        raise ValueError(f"unsupported ECQ1 version {version}")
    md = json.loads(raw[meta_off:data_off].decode("utf-8"))
    data = raw[data_off:]
    out = {}
    t_pos = 0
    d_pos = sum(t["table_size"] for t in md.values())
    for name, t in md.items():
        if layout == "reference":
            tb = data[t["table_offset"]:t["table_offset"] + t["table_size"]]
            db = data[t["data_offset"]:t["data_offset"] + t["data_size"]]
        elif layout == "as_written":
            tb = data[t_pos:t_pos + t["table_size"]]
            db = data[d_pos:d_pos + t["data_size"]]
            t_pos += t["table_size"]
            d_pos += t["data_size"]
        else:
            raise ValueError("layout is 'reference' or 'as_written'")
        table, err = None, None
        nsym = struct.unpack_from("<H", tb, 0)[0] if len(tb) >= 2 else 0
        if nsym != 16 or len(tb) < 2 + 2 * nsym:
            err = "no 16-symbol frequency table at the recorded offset"
        else:
            freq = np.array(struct.unpack_from(f"<{nsym}H", tb, 2), dtype=np.uint32)
            # the reference re-normalises the stored frequencies (src/rans.py:67-71)
            table = RANSTable.from_counts_reference(freq)
        out[name] = V1Tensor(name=name, shape=list(t["shape"]), scale=float(t["scale"]),
                             zero_point=float(t["zero_point"]), n_elements=int(t["n_elements"]), table=table,
                             data=bytes(db), error=err)
    return out


def decompress_v1_tensor(t: V1Tensor) -> np.ndarray:
    """Decode (GPU) and dequantise one v1 tensor: indices * scale + zero_point
    (src/compressed_format.py:314-350), float32 in the tensor's shape."""
    from .interleaved import interleaved_rans_decode

    idx = interleaved_rans_decode(t.tile())
    return (idx.astype(np.float32) * np.float32(t.scale) + np.float32(t.zero_point)).reshape(t.shape)
