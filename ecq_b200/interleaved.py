"""GPU decode of reference interleaved tiles: the drop-in replacements of
``interleaved_rans_decode`` / ``InterleavedRANSDecoder``
(drxddy/ecq src/interleaved_rans.py:156-217, :259-263) and of the Metal host
driver ``MetalInterleavedRANS.decode`` (src/metal_interleaved.py:833-885).

Decoding runs in libecq's ``decode_interleaved_exact`` kernel (one thread per
stream) with the reference decoder's semantics, guards included, so
damaged tiles decode to the bytes the reference returns. There is no CPU
path: without a CUDA device these functions raise.
"""
from __future__ import annotations

import numpy as np
import torch

from ._lib import check, lib, ptr
from .codec import (InterleavedEncodedTile, InterleavedRANSEncoder, RANSTable,  # noqa: F401 (re-export)
                    interleaved_rans_encode)
from . import _lib


def _need_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("ecq_b200 decodes on the GPU; no CUDA device is available")


class CudaInterleavedRANS:
    """CUDA counterpart of MetalInterleavedRANS (src/metal_interleaved.py:776-885):
    ``decode(tile)`` copies the tile to the device, decodes it and returns the
    symbols as numpy uint8."""

    def __init__(self, device: str | int | torch.device = "cuda"):
        _need_cuda()
        self.device = torch.device(device)
        self.last_status = 0
        self._tables: dict[bytes, tuple[torch.Tensor, int]] = {}

    def _table(self, table: RANSTable):
        key = np.asarray(table.freq, dtype=np.uint32).tobytes()
        hit = self._tables.get(key)
        if hit is None:
            entries, flags = RANSTable.from_freq(np.asarray(table.freq, dtype=np.uint32)).decode_table()
            hit = (torch.from_numpy(entries.view(np.int32)).to(self.device), flags)
            if len(self._tables) > 64:
                self._tables.clear()
            self._tables[key] = hit
        return hit

    def decode_device(self, tile: InterleavedEncodedTile, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Decode on the device; returns (symbols uint8 cuda tensor, status int32[1])."""
        S = int(tile.n_streams)
        n = int(tile.n_symbols)
        lens = np.asarray(tile.stream_lengths, dtype=np.uint32)
        if lens.size != S:
            raise ValueError("stream_lengths must have n_streams entries")
        ml = int(tile.max_stream_len)
        data = np.frombuffer(bytes(tile.data), dtype=np.uint8)
        if n and lens.size and int(lens.max()) > ml:
            raise ValueError("a stream is longer than max_stream_len")
        if data.size < S * ml:
            # the reference would index past its buffer (IndexError)
            raise ValueError("tile data shorter than n_streams * max_stream_len")
        dev = self.device
        d_data = torch.from_numpy(data.copy() if data.size else np.zeros(16, np.uint8)).to(dev, non_blocking=False)
        d_lens = torch.from_numpy(lens.view(np.int32).copy()).to(dev)
        table, flags = self._table(tile.table)
        out = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        check(lib().ecq_decode_interleaved(ptr(d_data), ptr(d_lens), S, n, ml, ptr(table), flags, ptr(out),
                                           ptr(status), int(s.cuda_stream)), "decode_interleaved")
        return out[:n], status

    def decode(self, tile: InterleavedEncodedTile) -> np.ndarray:
        out, status = self.decode_device(tile)
        res = out.cpu().numpy()
        self.last_status = int(status.item())
        return res


_default: CudaInterleavedRANS | None = None


def interleaved_rans_decode(tile: InterleavedEncodedTile) -> np.ndarray:
    """Drop-in for src/interleaved_rans.py:156-217, decoded on the GPU."""
    global _default
    if _default is None:
        _default = CudaInterleavedRANS()
    return _default.decode(tile)


class InterleavedRANSDecoder:
    """src/interleaved_rans.py:259-263."""

    def decode(self, tile: InterleavedEncodedTile) -> np.ndarray:
        return interleaved_rans_decode(tile)


def verify_interleaved_roundtrip(indices, n_streams: int = 4, bits: int = 4):
    """src/interleaved_rans.py:220-238: encode (host) then decode (GPU)."""
    indices = np.asarray(indices).reshape(-1)
    tile = InterleavedRANSEncoder(n_streams, bits).encode(indices)
    decoded = interleaved_rans_decode(tile)
    return bool(np.array_equal(indices, decoded)), tile.compression_ratio


STATUS_CORRUPT = _lib.STATUS_CORRUPT
