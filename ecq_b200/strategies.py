"""Decode strategies on the GPU: the reference's SmartDecoder interface
(drxddy/ecq src/decode_strategies.py:22-284) with every mode backed by
libecq's kernels instead of numpy threads or Metal queues.

* FUSED     -- get_weights returns None: the GEMV kernel decodes (ops.py).
* CACHED    -- load_layer decodes once on the GPU and keeps the weights as
  plain packed 4-bit (DecodeOnceStrategy's "store as 4-bit"); a packed
  matrix's cached weights multiply with the plain 4-bit GEMV
  (``DecodedWeights.packed.gemv``).
* LRU       -- decode on first use, keep within a byte budget, evict LRU.
* PREFETCH / GPU_ASYNC -- prefetch_layer decodes on a side CUDA stream and
  records an event; get_weights makes the caller's stream wait on it (no
  host synchronisation), is_ready queries the event.

A layer is either a reference ``InterleavedEncodedTile`` (decoded with the
reference-semantics kernel) or a packed ``DeviceMatrix`` (decoded by the
persistent kernel). Decoded weights stay on the device: ``indices`` is a
uint8 CUDA tensor (call ``.numpy()`` on the result for host symbols).
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass
from enum import Enum
from typing import Any, Dict, Optional

import numpy as np
import torch

from .codec import InterleavedEncodedTile
from .device import DeviceMatrix, Packed4Matrix


class DecodeMode(Enum):
    FUSED = "fused"
    CACHED = "cached"
    LRU = "lru"
    PREFETCH = "prefetch"
    GPU_ASYNC = "gpu_async"


@dataclass
class DecodedWeights:
    """src/decode_strategies.py:31-40, with device-resident weights: either
    uint8 indices, or (CACHED mode, packed matrices) a ``Packed4Matrix`` whose
    indices are unpacked only when asked for."""

    _indices: Optional[torch.Tensor]  # uint8 on the device, reshaped to `shape`
    scale: Any
    zero_point: Any
    shape: tuple
    packed: Optional[Packed4Matrix] = None

    @property
    def indices(self) -> torch.Tensor:
        if self._indices is None:
            self._indices = self.packed.symbols().reshape(self.shape)
        return self._indices

    @property
    def nbytes(self) -> int:
        """Bytes the cache holds: 4 bits per weight when packed."""
        return self.packed.nbytes if self.packed is not None else int(self._indices.numel())

    def numpy(self) -> np.ndarray:
        return self.indices.cpu().numpy()

    def dequantize(self) -> torch.Tensor:
        """indices * scale + zero_point (src/quantizer.py:33-35), fp32 on device."""
        s = torch.as_tensor(self.scale, device=self.indices.device, dtype=torch.float32)
        z = torch.as_tensor(self.zero_point, device=self.indices.device, dtype=torch.float32)
        return self.indices.float() * s + z


def _decode_async(layer, shape, stream: torch.cuda.Stream) -> tuple[torch.Tensor, torch.Tensor, Any]:
    """Decode on `stream`; returns (indices, status tensor, keep-alive)."""
    with torch.cuda.stream(stream):
        if isinstance(layer, DeviceMatrix):
            out = layer.decode(stream=stream)
            status, keep = layer.status, None
        elif isinstance(layer, InterleavedEncodedTile):
            from .interleaved import CudaInterleavedRANS

            dec = CudaInterleavedRANS(torch.cuda.current_device())
            out, status = dec.decode_device(layer, stream=stream)
            keep = dec
        else:
            raise TypeError("a layer is an InterleavedEncodedTile or a DeviceMatrix")
    return out.reshape(shape) if shape else out, status, keep


class SmartDecoder:
    """Unified interface over the decode strategies (src/decode_strategies.py:178-284)."""

    def __init__(self, mode: str = "fused", **kwargs):
        self.mode = DecodeMode(mode)
        self.max_bytes = int(kwargs.get("max_memory_bytes", 2 * 1024 ** 3))
        self.lock = threading.Lock()
        self.cache: "OrderedDict[str, DecodedWeights]" = OrderedDict()
        self.pending: Dict[str, tuple] = {}
        self.hits = 0
        self.misses = 0
        self.side = torch.cuda.Stream() if self.mode in (DecodeMode.PREFETCH, DecodeMode.GPU_ASYNC) else None

    # -- load time ---------------------------------------------------------
    def load_layer(self, name: str, tile, scale=0.0, zero_point=0.0, shape: tuple = ()) -> None:
        """Decode a layer now (CACHED mode), as DecodeOnceStrategy.load_layer."""
        if self.mode != DecodeMode.CACHED:
            return
        if isinstance(tile, DeviceMatrix):
            pk = Packed4Matrix.from_matrix(tile)
            self._check(tile.status)
            dw = DecodedWeights(None, scale, zero_point, tuple(shape) or (tile.rows, tile.cols), packed=pk)
        else:
            out, status, _ = _decode_async(tile, shape, torch.cuda.current_stream())
            self._check(status)
            dw = DecodedWeights(out, scale, zero_point, tuple(shape) or tuple(out.shape))
        with self.lock:
            self.cache[name] = dw

    def prefetch_layer(self, name: str, tile, scale=0.0, zero_point=0.0, shape: tuple = ()) -> None:
        """Start decoding on the side stream (PREFETCH / GPU_ASYNC)."""
        if self.mode not in (DecodeMode.PREFETCH, DecodeMode.GPU_ASYNC):
            return
        self.side.wait_stream(torch.cuda.current_stream())
        out, status, keep = _decode_async(tile, shape, self.side)
        ev = torch.cuda.Event()
        ev.record(self.side)
        with self.lock:
            self.pending[name] = (out, status, keep, ev, scale, zero_point, tuple(shape) or tuple(out.shape))

    # -- use time ----------------------------------------------------------
    def get_weights(self, name: str, tile=None, scale=0.0, zero_point=0.0, shape: tuple = ()) -> Optional[DecodedWeights]:
        if self.mode == DecodeMode.FUSED:
            return None
        if self.mode == DecodeMode.CACHED:
            return self.cache[name]
        if self.mode == DecodeMode.LRU:
            with self.lock:
                if name in self.cache:
                    self.cache.move_to_end(name)
                    self.hits += 1
                    return self.cache[name]
            self.misses += 1
            out, status, _ = _decode_async(tile, shape, torch.cuda.current_stream())
            self._check(status)
            dw = DecodedWeights(out, scale, zero_point, tuple(shape) or tuple(out.shape))
            with self.lock:
                while self.cache and self.memory_usage() + dw.nbytes > self.max_bytes:
                    self.cache.popitem(last=False)
                self.cache[name] = dw
            return dw
        # PREFETCH / GPU_ASYNC
        with self.lock:
            entry = self.pending.pop(name, None)
        if entry is None:
            raise KeyError(f"Layer {name} not found in pending or decoded")
        out, status, _keep, ev, sc, zp, shp = entry
        torch.cuda.current_stream().wait_event(ev)
        out.record_stream(torch.cuda.current_stream())
        return DecodedWeights(out, sc, zp, shp)

    def is_ready(self, name: str) -> bool:
        if self.mode in (DecodeMode.PREFETCH, DecodeMode.GPU_ASYNC):
            with self.lock:
                entry = self.pending.get(name)
            return entry is not None and entry[3].query()
        if self.mode == DecodeMode.CACHED:
            return name in self.cache
        return True

    def memory_usage(self) -> int:
        return sum(w.nbytes for w in self.cache.values())

    @property
    def stats(self) -> Dict[str, Any]:
        if self.mode == DecodeMode.LRU:
            total = self.hits + self.misses
            return {"hit_rate": self.hits / total if total else 0.0, "hits": self.hits, "misses": self.misses,
                    "memory_bytes": self.memory_usage()}
        if self.mode in (DecodeMode.PREFETCH, DecodeMode.GPU_ASYNC):
            return {"pending_decodes": len(self.pending), "memory_bytes": self.memory_usage()}
        return {}

    @staticmethod
    def _check(status: torch.Tensor) -> None:
        s = int(status.item())
        if s:
            from ._lib import EcqError

            raise EcqError(f"device decode reported status {s:#x}")
