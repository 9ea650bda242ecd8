"""Device-resident packed matrices and the GPU entry points behind them.

``DeviceMatrix`` holds one packed matrix in HBM (torch tensors own the
memory): the tiles' interleaved stream bytes, tile offsets, per-stream
lengths and the packed decode table, plus the fused GEMV's workspace and a
device status word. Its methods call libecq's C ABI on the current torch
stream; nothing here synchronises the host unless asked to.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import MatrixView, EcqError, check, lib, ptr
from .codec import EncodedMatrix, RANSTable


def _stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# Token batches up to this size run the fused GEMV, which decodes each tile once
# for the whole batch; larger ones a tensor-core path. Measured on 28672 x 8192:
# the GEMV's CUDA-core math for 8 tokens costs 2x its single-token time, more
# than the tcgen05 kernel (1.3x) or decoding W to fp16 once for cuBLAS (1.35x).
GEMV_MAX_BATCH = 4
# Token batches above GEMV_MAX_BATCH and up to this size run the tcgen05 kernel;
# larger ones decode W once to fp16 for cuBLAS. Measured on 28672 x 8192 (8x256
# tiles): the two are level at 32 tokens and the decode-once path is 12 % faster
# at 128, where re-reading x for every weight item costs the tcgen05 kernel more
# than it saves by never writing W.
TENSOR_CORE_MAX_BATCH = 32


@dataclass
class DeviceMatrix:
    rows: int
    cols: int
    tile_rows: int
    tile_cols: int
    group_size: int
    table: RANSTable
    flags: int
    max_tile_bytes: int
    data: torch.Tensor        # uint8
    tile_offset: torch.Tensor  # int32 (bit pattern of uint32)
    stream_len: torch.Tensor   # int16 (bit pattern of uint16)
    dec_table: torch.Tensor    # int32 (bit pattern of uint32)
    workspace: torch.Tensor    # uint8, zero-filled
    status: torch.Tensor       # int32 [1]
    mm_workspace: torch.Tensor | None = None  # uint8, zero-filled (tensor-core path)

    @classmethod
    def from_encoded(cls, enc: EncodedMatrix, group_size: int = 128, device="cuda") -> "DeviceMatrix":
        enc.validate()  # offsets from a file are checked before any device copy
        entries, flags = enc.table.decode_table()
        dev = torch.device(device)
        data = np.ascontiguousarray(enc.data)
        if data.size == 0:
            data = np.zeros(16, dtype=np.uint8)
        def to(a, dt):
            a = np.ascontiguousarray(a)
            if not a.flags.writeable:  # e.g. a memory-mapped container blob: torch wants writable host memory
                a = a.copy()
            return torch.from_numpy(a.view(dt)).to(dev)

        m = cls(rows=enc.rows, cols=enc.cols, tile_rows=enc.tile_rows, tile_cols=enc.tile_cols,
                group_size=int(group_size), table=enc.table, flags=flags, max_tile_bytes=enc.max_tile_bytes,
                data=to(data, np.uint8), tile_offset=to(enc.tile_offset.astype(np.uint32), np.int32),
                stream_len=to(enc.stream_len.astype(np.uint16), np.int16), dec_table=to(entries, np.int32),
                workspace=torch.zeros(0, dtype=torch.uint8, device=dev),
                status=torch.zeros(1, dtype=torch.int32, device=dev))
        ws = lib().ecq_gemv_workspace_bytes(ctypes_view(m), 1)
        check(ws, "workspace size")
        m.workspace = torch.zeros(int(ws), dtype=torch.uint8, device=dev)
        return m

    @property
    def n_tiles(self) -> int:
        return int(self.tile_offset.numel() - 1)

    @property
    def compressed_bytes(self) -> int:
        return int(self.data.numel())

    @property
    def device(self) -> torch.device:
        return self.data.device

    def view(self) -> MatrixView:
        return ctypes_view(self)

    # ---- entry points ----
    def decode(self, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Decode to row-major uint8 symbols [rows, cols] on the device."""
        if out is None:
            out = torch.empty(self.rows, self.cols, dtype=torch.uint8, device=self.device)
        _require_cuda(out, "out")
        if out.numel() != self.rows * self.cols or out.dtype != torch.uint8:
            raise ValueError("out must be uint8 [rows, cols]")
        v = self.view()
        check(lib().ecq_matrix_decode(v, ptr(out), ptr(self.status), _stream_ptr(stream)), "matrix decode")
        return out

    def decode_packed4(self, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Decode to plain packed 4-bit [rows, cols/2] uint8 on the device:
        column 2i in the low nibble of byte i of its row, 2i+1 in the high."""
        if out is None:
            out = torch.empty(self.rows, self.cols // 2, dtype=torch.uint8, device=self.device)
        _require_cuda(out, "out")
        if out.numel() * 2 != self.rows * self.cols or out.dtype != torch.uint8:
            raise ValueError("out must be uint8 [rows, cols/2]")
        check(lib().ecq_matrix_decode_packed4(self.view(), ptr(out), ptr(self.status), _stream_ptr(stream)),
              "matrix decode to packed 4-bit")
        return out

    def dequantize(self, scales: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Decode to dequantised fp16 weights [rows, cols] = (sym - 8) * scale."""
        ng = (self.cols + self.group_size - 1) // self.group_size
        if scales.dtype != torch.float16 or tuple(scales.shape) != (self.rows, ng):
            raise ValueError(f"scales must be float16 [{self.rows}, {ng}]")
        _require_cuda(scales, "scales")
        if out is None:
            out = torch.empty(self.rows, self.cols, dtype=torch.float16, device=self.device)
        _require_cuda(out, "out")
        check(lib().ecq_matrix_dequantize(self.view(), ptr(scales), ptr(out), ptr(self.status), _stream_ptr(stream)),
              "matrix dequantize")
        return out

    def tensor_core_ok(self) -> bool:
        """True when the tile layout has a tcgen05 kernel (tile widths 128, 256)."""
        return int(lib().ecq_matmul_workspace_bytes(self.view(), 1)) > 0

    def matmul_tc(self, x: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
        """y = x @ W^T for x [B, cols] fp16 on the tcgen05 tensor cores, each
        tile decoded straight into the MMA's shared-memory operand (no decoded
        weight in memory); fp32 accumulation, fp16 y [B, rows]."""
        x2 = x.reshape(-1, self.cols)
        if x2.dtype != torch.float16:
            raise ValueError("x must be float16")
        _require_cuda(x2, "x")
        _require_cuda(scales, "scales")
        ng = (self.cols + self.group_size - 1) // self.group_size
        if scales.dtype != torch.float16 or tuple(scales.shape) != (self.rows, ng):
            raise ValueError(f"scales must be float16 [{self.rows}, {ng}]")
        if not x2.is_contiguous() or x2.data_ptr() % 16:
            x2 = x2.contiguous().clone()
        B = x2.shape[0]
        if out is None:
            out = torch.empty(B, self.rows, dtype=torch.float16, device=self.device)
        _require_cuda(out, "out")
        v = self.view()
        need = int(lib().ecq_matmul_workspace_bytes(v, B))
        check(need, "matmul workspace size")
        if self.mm_workspace is None or self.mm_workspace.numel() < need:
            self.mm_workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        check(lib().ecq_matmul(v, ptr(x2), ptr(scales), ptr(out), B, ptr(self.mm_workspace),
                               self.mm_workspace.numel(), ptr(self.status), _stream_ptr(stream)), "matmul")
        return out

    def matmul(self, x: torch.Tensor, scales: torch.Tensor, fused_max_batch: int = GEMV_MAX_BATCH,
               tensor_core_max_batch: int = TENSOR_CORE_MAX_BATCH) -> torch.Tensor:
        """y = x @ W^T for x [..., cols] fp16: the one dispatch every batched
        entry point uses. Up to `fused_max_batch` token rows run the fused
        GEMV, which decodes each tile once for the whole batch. Batches up to
        `tensor_core_max_batch` run the tcgen05 kernel (matmul_tc) when the
        tile layout has one (tile widths 128 and 256); otherwise, and for
        larger batches, W is decoded once to fp16 (dequantize) for a
        tensor-core GEMM."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.cols)
        if x2.shape[0] <= fused_max_batch:
            y = self.gemv(x2.contiguous(), scales)
        elif x2.shape[0] <= tensor_core_max_batch and self.tensor_core_ok():
            y = self.matmul_tc(x2, scales)
        else:
            w = self.dequantize(scales)
            y = torch.mm(x2, w.t(), out_dtype=torch.float32).to(torch.float16)
        return y.reshape(*lead, self.rows)

    def ensure_workspace(self, batch: int) -> None:
        """Grow the GEMV workspace (zero-filled) to what a `batch`-token call
        needs. Call it outside stream capture before capturing such calls."""
        need = int(lib().ecq_gemv_workspace_bytes(self.view(), int(batch)))
        check(need, "workspace size")
        if self.workspace.numel() < need:
            self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)

    def gemv(self, x: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """y[b] = W_deq x[b] (fp16 in/out, fp32 accumulation); x [B, cols] or [cols]."""
        squeeze = x.dim() == 1
        x2 = x.reshape(-1, self.cols)
        if x2.dtype != torch.float16:
            raise ValueError("x must be float16")
        _require_cuda(x2, "x")
        _require_cuda(scales, "scales")
        ng = (self.cols + self.group_size - 1) // self.group_size
        if scales.dtype != torch.float16 or tuple(scales.shape) != (self.rows, ng):
            raise ValueError(f"scales must be float16 [{self.rows}, {ng}]")
        B = x2.shape[0]
        if out is None:
            out = torch.empty(B, self.rows, dtype=torch.float16, device=self.device)
        _require_cuda(out, "out")
        if B > 1 and not torch.cuda.is_current_stream_capturing():
            self.ensure_workspace(B)
        v = self.view()
        check(lib().ecq_gemv(v, ptr(x2), ptr(scales), ptr(out), B, ptr(self.workspace), self.workspace.numel(),
                             ptr(self.status), _stream_ptr(stream)), "gemv")
        return out[0] if squeeze else out

    def gemv_rope_kv(self, x: torch.Tensor, scales: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     k_slot: torch.Tensor, v_slot: torch.Tensor, head_dim: int, cache_head_stride: int,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Batch-1 GEMV of a fused q|k|v projection (rows = 3 * heads *
        head_dim) with the rotary embedding and the KV-cache store fused in:
        returns y = q | k | v with q and k rotated (pairs (2i, 2i+1) by angle
        index i), and writes the rotated k and v into k_slot / v_slot (head h
        at h * cache_head_stride)."""
        epi = _lib.GemvEpilogue(kind=_lib.EPI_ROPE_KV, part_rows=self.rows // 3, head_dim=int(head_dim), reserved=0,
                                cache_head_stride=int(cache_head_stride), cos_f16=ptr(cos), sin_f16=ptr(sin),
                                k_cache_f16=ptr(k_slot), v_cache_f16=ptr(v_slot))
        if out is None:
            out = torch.empty(1, self.rows, dtype=torch.float16, device=self.device)
        return self._gemv_fused(x, scales, epi, out, stream)

    def gemv_silu_mul(self, x: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None,
                      stream=None) -> torch.Tensor:
        """Batch-1 GEMV of a projection whose rows interleave gate and up
        (row 2j gate j, 2j+1 up j) with SwiGLU fused in: returns
        silu(gate) * up [1, rows / 2]."""
        epi = _lib.GemvEpilogue(kind=_lib.EPI_SILU_MUL)
        if out is None:
            out = torch.empty(1, self.rows // 2, dtype=torch.float16, device=self.device)
        return self._gemv_fused(x, scales, epi, out, stream)

    def _gemv_fused(self, x, scales, epi, out, stream):
        x2 = x.reshape(1, self.cols)
        if x2.dtype != torch.float16:
            raise ValueError("x must be float16")
        _require_cuda(x2, "x")
        _require_cuda(scales, "scales")
        _require_cuda(out, "out")
        check(lib().ecq_gemv_fused(self.view(), ptr(x2), ptr(scales), ptr(out), epi, ptr(self.workspace),
                                   self.workspace.numel(), ptr(self.status), _stream_ptr(stream)), "gemv_fused")
        return out

    def read_status(self, reset: bool = True) -> int:
        """Synchronising read of the device status word (ECQ_STATUS_* bits)."""
        s = int(self.status.item())
        if reset and s:
            self.status.zero_()
            # a call that did not finish may leave slab counters or partial sums set
            self.workspace.zero_()
            if self.mm_workspace is not None:
                self.mm_workspace.zero_()
        return s

    def check(self) -> None:
        s = self.read_status()
        if s & _lib.STATUS_CORRUPT:
            raise EcqError("corrupt rANS stream (end-of-stream state check failed)")
        if s & _lib.STATUS_TIMEOUT:
            raise EcqError("device wait timed out")
        if s:
            raise EcqError(f"device status {s:#x}")


@dataclass
class Packed4Matrix:
    """A plain (not entropy-coded) 4-bit matrix on the device: q [rows,
    cols/2] uint8 packed nibbles (column 2i low, 2i+1 high), zero point 8,
    group scales passed per call. The CACHED strategy's store (decode once
    with ``DeviceMatrix.decode_packed4``) and the bench's plain-4-bit
    control; ``gemv`` runs ``ecq_plain4_gemv``."""

    rows: int
    cols: int
    group_size: int
    q: torch.Tensor  # uint8 [rows, cols // 2]

    @classmethod
    def from_symbols(cls, symbols, group_size: int = 128, device="cuda") -> "Packed4Matrix":
        """Pack a host [rows, cols] symbol matrix (values < 16)."""
        sym = np.ascontiguousarray(np.asarray(symbols, dtype=np.uint8))
        if sym.ndim != 2 or sym.shape[1] % 2:
            raise ValueError("symbols must be [rows, cols] with even cols")
        q = (sym[:, 0::2] & 15) | ((sym[:, 1::2] & 15) << 4)
        return cls(rows=sym.shape[0], cols=sym.shape[1], group_size=int(group_size),
                   q=torch.from_numpy(np.ascontiguousarray(q)).to(torch.device(device)))

    @classmethod
    def from_matrix(cls, m: DeviceMatrix, stream=None) -> "Packed4Matrix":
        """Decode an entropy-coded matrix once (on the GPU) into packed 4-bit."""
        return cls(rows=m.rows, cols=m.cols, group_size=m.group_size, q=m.decode_packed4(stream=stream))

    @property
    def nbytes(self) -> int:
        return int(self.q.numel())

    @property
    def device(self) -> torch.device:
        return self.q.device

    def gemv(self, x: torch.Tensor, scales: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """y[b] = (q - 8) * scale @ x[b], x [B, cols] or [cols] fp16 (fp16 y)."""
        squeeze = x.dim() == 1
        x2 = x.reshape(-1, self.cols)
        if x2.dtype != torch.float16:
            raise ValueError("x must be float16")
        _require_cuda(x2, "x")
        if x2.data_ptr() % 16:
            x2 = x2.clone()
        _require_cuda(scales, "scales")
        ng = (self.cols + self.group_size - 1) // self.group_size
        if scales.dtype != torch.float16 or tuple(scales.shape) != (self.rows, ng):
            raise ValueError(f"scales must be float16 [{self.rows}, {ng}]")
        B = x2.shape[0]
        if out is None:
            out = torch.empty(B, self.rows, dtype=torch.float16, device=self.device)
        _require_cuda(out, "out")
        check(lib().ecq_plain4_gemv(ptr(self.q), ptr(scales), ptr(x2), ptr(out), self.rows, self.cols,
                                    self.group_size, B, _stream_ptr(stream)), "plain 4-bit gemv")
        return out[0] if squeeze else out

    def symbols(self) -> torch.Tensor:
        """Unpacked uint8 [rows, cols] symbols (a device copy)."""
        out = torch.empty(self.rows, self.cols, dtype=torch.uint8, device=self.device)
        out[:, 0::2] = self.q & 15
        out[:, 1::2] = self.q >> 4
        return out


def ctypes_view(m: DeviceMatrix) -> MatrixView:
    return MatrixView(rows=m.rows, cols=m.cols, tile_rows=m.tile_rows, tile_cols=m.tile_cols,
                      group_size=m.group_size, n_tiles=m.n_tiles, max_tile_bytes=m.max_tile_bytes, flags=m.flags,
                      data=ptr(m.data), tile_offset=ptr(m.tile_offset), stream_len=ptr(m.stream_len),
                      dec_table=ptr(m.dec_table))


def device_info(m: DeviceMatrix | None = None) -> dict:
    sms = np.zeros(1, dtype=np.int32)
    ctas = np.zeros(1, dtype=np.int32)
    warps = np.zeros(1, dtype=np.int32)
    v = ctypes_view(m) if m is not None else None
    check(lib().ecq_device_info(ptr(sms), ptr(ctas), ptr(warps), v), "device_info")
    return {"sm_count": int(sms[0]), "gemv_ctas": int(ctas[0]), "gemv_warps_per_cta": int(warps[0])}
