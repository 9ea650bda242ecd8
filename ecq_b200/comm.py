"""The tensor-parallel exchange of the batch-1 decode step over NVLink peer
memory (include/ecq_comm.h).

Each rank allocates one exchange buffer in libecq, exports it with CUDA IPC,
and opens every other rank's export; the handles travel through
``torch.distributed.all_gather_object``. A row-parallel layer then runs
``ecq_gemv_tp`` (the fused GEMV pushing its fp32 partial y to every rank)
followed by ``ecq_tp_add_rmsnorm_f16`` (wait for every rank's partial, sum in
rank order, residual add + RMSNorm) in place of GEMV -> NCCL all-reduce ->
add + RMSNorm. All ranks must issue the same sequence of those calls.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import TPComm, check, lib, ptr


class PeerExchange:
    """One rank's exchange buffer, the peers' buffers mapped into this process
    and the ``ecq_tp_comm`` descriptor the kernels take."""

    def __init__(self, n_max: int, group=None, device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 1 <= self.world <= _lib.TP_MAX_RANKS:
            raise ValueError(f"the exchange supports up to {_lib.TP_MAX_RANKS} ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.n_max = int(n_max)
        self._opened: list[int] = []
        self._local = None
        with torch.cuda.device(self.device):
            nbytes = int(lib().ecq_comm_buffer_bytes(self.n_max, self.world))
            check(nbytes, "exchange buffer size")
            buf = ctypes.c_void_p()
            check(lib().ecq_comm_alloc(nbytes, ctypes.byref(buf)), "exchange buffer")
            self._local = buf.value
            handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            check(lib().ecq_ipc_get_handle(self._local, handle), "IPC export")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            peers = []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    peers.append(self._local)
                    continue
                mapped = ctypes.c_void_p()
                h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                check(lib().ecq_ipc_open(h, ctypes.byref(mapped)), f"IPC open of rank {r}")
                self._opened.append(mapped.value)
                peers.append(mapped.value)
        arr = (ctypes.c_void_p * _lib.TP_MAX_RANKS)(*(peers + [None] * (_lib.TP_MAX_RANKS - self.world)))
        self.desc = TPComm(world=self.world, rank=self.rank, n_max=self.n_max, reserved=0, local=self._local,
                           peers=arr)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def gemv_push(self, m, x: torch.Tensor, scales: torch.Tensor) -> None:
        """Row-parallel fused GEMV at batch 1 whose partial y goes to every rank."""
        v = m.view()
        check(lib().ecq_gemv_tp(v, ptr(x), ptr(scales), ctypes.byref(self.desc), ptr(m.workspace),
                                m.workspace.numel(), ptr(m.status), torch.cuda.current_stream(self.device).cuda_stream),
              "gemv_tp")

    def add_rmsnorm(self, h: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        """h += sum over ranks of this epoch's partials (in place); returns
        rmsnorm(h) * w. h, w fp16 [n] or [1, n]."""
        y = torch.empty_like(h)
        check(lib().ecq_tp_add_rmsnorm_f16(ptr(h), ctypes.byref(self.desc), ptr(w), ptr(h), ptr(y), h.numel(),
                                           float(eps), ptr(self.status),
                                           torch.cuda.current_stream(self.device).cuda_stream), "tp_add_rmsnorm")
        return y

    def sum(self, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """y [n] fp16 = sum over ranks of this epoch's partials (after every
        rank's gemv_push): the all-reduce of a column-sharded GEMV."""
        if out is None:
            out = torch.empty(n, dtype=torch.float16, device=self.device)
        check(lib().ecq_tp_sum_f16(ctypes.byref(self.desc), ptr(out), int(n), ptr(self.status),
                                   torch.cuda.current_stream(self.device).cuda_stream), "tp_sum")
        return out

    def check(self) -> None:
        s = int(self.status.item())
        if s:
            self.status.zero_()
            # the ranks' epochs may now disagree: close() and rebuild the exchange on every rank
            raise _lib.EcqError(f"peer exchange status {s:#x} (a rank's partials did not arrive in time; "
                                "rebuild the exchange on every rank)")

    def close(self) -> None:
        """Release the mappings and the buffer. Every rank must be done with
        every kernel that touches them: this synchronises the device and the
        group first."""
        if self._local is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            lib().ecq_ipc_close(p)
        self._opened.clear()
        lib().ecq_comm_free(self._local)
        self._local = None


__all__ = ["PeerExchange"]
