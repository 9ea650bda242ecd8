"""PyTorch-facing entry points of the fused decode + dequant + GEMV.

* ``torch.ops.ecq.rans_gemv`` -- a custom op over libecq's ``ecq_gemv``
  (with a fake implementation for shape propagation), so the fused GEMV can
  sit inside torch programs and CUDA graphs.
* ``torch.ops.ecq.rans_matmul`` -- the same over ``ecq_matmul``, the
  batched-token kernel on the tcgen05 tensor cores.
* ``entropy_coded_matmul`` -- the fused op with the argument list of the
  reference's MLX plan (docs/mlx_integration_plan.md:222-237).
* ``EntropyCodedLinear`` -- an ``nn.Linear`` replacement built with
  ``from_linear`` (experiments/real_model_test.py:135-181), FUSED or CACHED.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import MatrixView, check, lib
from .codec import RANSTable, encode_matrix
from .device import GEMV_MAX_BATCH, TENSOR_CORE_MAX_BATCH, DeviceMatrix, Packed4Matrix
from .synthetic import quantize_symmetric_groups


def _view(data, tile_offset, stream_len, dec_table, rows, cols, tile_rows, tile_cols, group_size, flags,
          max_tile_bytes) -> MatrixView:
    return MatrixView(rows=rows, cols=cols, tile_rows=tile_rows, tile_cols=tile_cols, group_size=group_size,
                      n_tiles=tile_offset.numel() - 1, max_tile_bytes=max_tile_bytes, flags=flags,
                      data=data.data_ptr(), tile_offset=tile_offset.data_ptr(), stream_len=stream_len.data_ptr(),
                      dec_table=dec_table.data_ptr())


@torch.library.custom_op("ecq::rans_gemv", mutates_args=("workspace", "status"))
def rans_gemv_op(x: torch.Tensor, data: torch.Tensor, tile_offset: torch.Tensor, stream_len: torch.Tensor,
                 dec_table: torch.Tensor, scales: torch.Tensor, workspace: torch.Tensor, status: torch.Tensor,
                 rows: int, cols: int, tile_rows: int, tile_cols: int, group_size: int, flags: int,
                 max_tile_bytes: int) -> torch.Tensor:
    """y[B, rows] = dequant(W) @ x[B, cols]^T, fp16 in/out, fp32 accumulation."""
    if not x.is_cuda:
        raise RuntimeError("ecq::rans_gemv runs on CUDA tensors only")
    x2 = x.reshape(-1, cols).contiguous()
    y = torch.empty(x2.shape[0], rows, dtype=torch.float16, device=x.device)
    v = _view(data, tile_offset, stream_len, dec_table, rows, cols, tile_rows, tile_cols, group_size, flags,
              max_tile_bytes)
    check(lib().ecq_gemv(v, x2.data_ptr(), scales.data_ptr(), y.data_ptr(), x2.shape[0], workspace.data_ptr(),
                         workspace.numel(), status.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream),
          "ecq::rans_gemv")
    return y


@rans_gemv_op.register_fake
def _(x, data, tile_offset, stream_len, dec_table, scales, workspace, status, rows, cols, tile_rows, tile_cols,
      group_size, flags, max_tile_bytes):
    return x.new_empty((x.numel() // cols, rows), dtype=torch.float16)


def rans_gemv(x: torch.Tensor, m: DeviceMatrix, scales: torch.Tensor) -> torch.Tensor:
    """The custom op on a DeviceMatrix; x [B, cols] or [cols] fp16. Token
    batches share one decode of each tile (up to 8 tokens per launch)."""
    B = x.numel() // m.cols
    if B > 1 and not torch.cuda.is_current_stream_capturing():
        m.ensure_workspace(B)
    y = torch.ops.ecq.rans_gemv(x, m.data, m.tile_offset, m.stream_len, m.dec_table, scales, m.workspace,
                                m.status, m.rows, m.cols, m.tile_rows, m.tile_cols, m.group_size, m.flags,
                                m.max_tile_bytes)
    return y[0] if x.dim() == 1 else y


@torch.library.custom_op("ecq::rans_matmul", mutates_args=("workspace", "status"))
def rans_matmul_op(x: torch.Tensor, data: torch.Tensor, tile_offset: torch.Tensor, stream_len: torch.Tensor,
                   dec_table: torch.Tensor, scales: torch.Tensor, workspace: torch.Tensor, status: torch.Tensor,
                   rows: int, cols: int, tile_rows: int, tile_cols: int, group_size: int, flags: int,
                   max_tile_bytes: int) -> torch.Tensor:
    """y[B, rows] = x[B, cols] @ dequant(W)^T on the tensor cores (tile widths
    128 and 256), fp16 in/out, fp32 accumulation. `workspace` holds at least
    ecq_matmul_workspace_bytes(B) zero bytes."""
    if not x.is_cuda:
        raise RuntimeError("ecq::rans_matmul runs on CUDA tensors only")
    x2 = x.reshape(-1, cols).contiguous()
    y = torch.empty(x2.shape[0], rows, dtype=torch.float16, device=x.device)
    v = _view(data, tile_offset, stream_len, dec_table, rows, cols, tile_rows, tile_cols, group_size, flags,
              max_tile_bytes)
    check(lib().ecq_matmul(v, x2.data_ptr(), scales.data_ptr(), y.data_ptr(), x2.shape[0], workspace.data_ptr(),
                           workspace.numel(), status.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream),
          "ecq::rans_matmul")
    return y


@rans_matmul_op.register_fake
def _(x, data, tile_offset, stream_len, dec_table, scales, workspace, status, rows, cols, tile_rows, tile_cols,
      group_size, flags, max_tile_bytes):
    return x.new_empty((x.numel() // cols, rows), dtype=torch.float16)


def rans_matmul(x: torch.Tensor, m: DeviceMatrix, scales: torch.Tensor) -> torch.Tensor:
    """x [B, cols] fp16 -> y [B, rows], routed as DeviceMatrix.matmul routes:
    up to GEMV_MAX_BATCH tokens the fused GEMV (each tile decoded once for the
    batch), up to TENSOR_CORE_MAX_BATCH the tcgen05 kernel when the tile
    layout has one, else W decoded once to fp16 for a tensor-core GEMM."""
    x2 = x.reshape(-1, m.cols)
    if x2.shape[0] <= GEMV_MAX_BATCH:
        return rans_gemv(x2.contiguous(), m, scales)
    if x2.shape[0] > TENSOR_CORE_MAX_BATCH or not m.tensor_core_ok():
        w = m.dequantize(scales)
        return torch.mm(x2.contiguous(), w.t(), out_dtype=torch.float32).to(torch.float16)
    need = int(lib().ecq_matmul_workspace_bytes(m.view(), x2.shape[0]))
    check(need, "matmul workspace size")
    if m.mm_workspace is None or m.mm_workspace.numel() < need:
        m.mm_workspace = torch.zeros(need, dtype=torch.uint8, device=m.device)
    return torch.ops.ecq.rans_matmul(x2, m.data, m.tile_offset, m.stream_len, m.dec_table, scales, m.mm_workspace,
                                     m.status, m.rows, m.cols, m.tile_rows, m.tile_cols, m.group_size, m.flags,
                                     m.max_tile_bytes)


def entropy_coded_matmul(x: torch.Tensor, compressed_w: DeviceMatrix, stream_offsets=None, freq_table=None,
                         cumfreq_table=None, sym_table=None, scales: torch.Tensor | None = None,
                         biases: torch.Tensor | None = None, transpose: bool = True, group_size: int = 64,
                         bits: int = 4, n_streams: int = 32) -> torch.Tensor:
    """Fused decode + dequant + matmul with the argument list of the MLX plan
    (docs/mlx_integration_plan.md:222-237): ``x @ dequant(W)^T``.

    ``compressed_w`` is a ``DeviceMatrix`` (packed tiles, offsets, stream
    lengths and decode table in HBM), so ``stream_offsets``, ``freq_table``,
    ``cumfreq_table`` and ``sym_table`` are checked against it rather than
    re-uploaded. Weights dequantise as ``w = sym * scale + bias`` per group;
    ``biases=None`` means the symmetric zero-point 8 (bias = -8 * scale),
    which the kernel applies in fp32. Other biases add
    ``(bias + 8*scale) . sum_group(x)`` on top (a [rows, groups] product)."""
    m = compressed_w
    if not transpose:
        raise NotImplementedError("only x @ W^T (transpose=True) is implemented")
    if bits != 4:
        raise ValueError("only 4-bit symbols are supported")
    if n_streams != 32:
        raise ValueError("packed matrices use 32 streams per tile")
    if group_size != m.group_size:
        raise ValueError(f"group_size {group_size} does not match the matrix ({m.group_size})")
    if freq_table is not None and not np.array_equal(np.asarray(freq_table, dtype=np.uint32).reshape(-1)[:16],
                                                     m.table.freq):
        raise ValueError("freq_table differs from the matrix's table")
    if cumfreq_table is not None and not np.array_equal(np.asarray(cumfreq_table, dtype=np.uint32).reshape(-1)[:17],
                                                        m.table.cumfreq):
        raise ValueError("cumfreq_table differs from the matrix's table")
    if scales is None:
        raise ValueError("scales are required")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, m.cols).to(torch.float16).contiguous()
    y = rans_matmul(x2, m, scales)
    if biases is not None:
        ng = scales.shape[1]
        pad = ng * group_size - m.cols
        xs = torch.nn.functional.pad(x2.float(), (0, pad)).reshape(x2.shape[0], ng, group_size).sum(-1)
        corr = xs @ (biases.float() + 8.0 * scales.float()).t()
        y = (y.float() + corr).to(torch.float16)
    return y.reshape(*lead, m.rows)


class EntropyCodedLinear(torch.nn.Module):
    """An nn.Linear whose weight is held rANS-coded in HBM (the reference's
    out-of-tree EntropyCodedLinear, experiments/real_model_test.py:135-181).

    decode_mode "fused": every forward runs the fused decode+dequant+GEMV.
    decode_mode "cached": the weight is decoded once on the GPU at load into
    plain packed 4-bit (the reference's CACHED strategy, "store as 4-bit",
    src/decode_strategies.py:43-73) and each forward runs the plain 4-bit
    GEMV on it (up to 4 tokens per pass over the weights); batches above
    `cached_gemv_max_batch` expand the 4-bit weight to fp16 for one
    tensor-core GEMM instead."""

    cached_gemv_max_batch = 8

    def __init__(self, matrix: DeviceMatrix, scales: torch.Tensor, bias: torch.Tensor | None = None,
                 decode_mode: str = "fused"):
        super().__init__()
        if decode_mode not in ("fused", "fused_v2", "cached"):
            raise ValueError(f"unknown decode_mode {decode_mode!r}")
        self.matrix = matrix
        self.register_buffer("scales", scales)
        self.register_buffer("bias", bias)
        self.decode_mode = "cached" if decode_mode == "cached" else "fused"
        self.in_features = matrix.cols
        self.out_features = matrix.rows
        self._packed = None
        if self.decode_mode == "cached":
            self._packed = Packed4Matrix.from_matrix(matrix)
            matrix.check()

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, n_streams: int = 32, decode_mode: str = "fused",
                    group_size: int = 128, tile_cols: int | None = None) -> "EntropyCodedLinear":
        if n_streams != 32:
            raise ValueError("packed matrices use 32 streams per tile")
        w = linear.weight.detach().float().cpu().numpy()
        sym, sc = quantize_symmetric_groups(w, group_size)
        enc = encode_matrix(sym, RANSTable.from_symbols(sym), tile_cols=tile_cols, group_size=group_size)
        dev = linear.weight.device if linear.weight.is_cuda else torch.device("cuda")
        m = DeviceMatrix.from_encoded(enc, group_size=group_size, device=dev)
        bias = linear.bias.detach().to(dev, torch.float16) if linear.bias is not None else None
        return cls(m, torch.from_numpy(sc).to(dev), bias, decode_mode)

    @property
    def compression_ratio(self) -> float:
        return (self.matrix.rows * self.matrix.cols / 2) / self.matrix.compressed_bytes

    @property
    def bits_per_weight(self) -> float:
        return 8.0 * self.matrix.compressed_bytes / (self.matrix.rows * self.matrix.cols)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).to(torch.float16)
        if self.decode_mode == "cached":
            if x2.shape[0] <= self.cached_gemv_max_batch:
                y = self._packed.gemv(x2.contiguous(), self.scales)
            else:
                sc = self.scales.float().repeat_interleave(self.matrix.group_size, dim=1)[:, : self.in_features]
                w = ((self._packed.symbols().float() - 8.0) * sc).to(torch.float16)
                y = torch.mm(x2, w.t(), out_dtype=torch.float32).to(torch.float16)
        else:
            y = rans_matmul(x2.contiguous(), self.matrix, self.scales)
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*lead, self.out_features)


__all__ = ["rans_gemv", "rans_gemv_op", "rans_matmul", "rans_matmul_op", "entropy_coded_matmul", "EntropyCodedLinear",
           "_lib"]
