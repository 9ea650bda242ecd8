"""Host-only checks of the PyTorch-facing API: the custom op's fake
(meta) implementation propagates shapes without a device."""
import pytest

torch = pytest.importorskip("torch")

from ecq_b200 import ops  # noqa: E402,F401  (registers torch.ops.ecq.rans_gemv)


def test_rans_gemv_fake_shapes():
    meta = torch.device("meta")
    x = torch.empty(3, 4096, dtype=torch.float16, device=meta)
    t = lambda n, dt: torch.empty(n, dtype=dt, device=meta)
    y = torch.ops.ecq.rans_gemv(x, t(100, torch.uint8), t(4097, torch.int32), t(4096 * 32, torch.int16),
                                t(16384, torch.int32), torch.empty(4096, 32, dtype=torch.float16, device=meta),
                                t(10, torch.uint8), t(1, torch.int32), 4096, 4096, 8, 512, 128, 0, 1024)
    assert y.shape == (3, 4096) and y.dtype == torch.float16 and y.device == meta


def test_rans_matmul_fake_shapes():
    meta = torch.device("meta")
    x = torch.empty(24, 2048, dtype=torch.float16, device=meta)
    t = lambda n, dt: torch.empty(n, dtype=dt, device=meta)
    y = torch.ops.ecq.rans_matmul(x, t(100, torch.uint8), t(4097, torch.int32), t(4096 * 32, torch.int16),
                                  t(16384, torch.int32), torch.empty(1024, 16, dtype=torch.float16, device=meta),
                                  t(10, torch.uint8), t(1, torch.int32), 1024, 2048, 8, 256, 128, 0, 700)
    assert y.shape == (24, 1024) and y.dtype == torch.float16 and y.device == meta


@pytest.mark.parametrize("B,tc_ok,want", [(1, True, "gemv"), (4, True, "gemv"), (5, True, "tc"), (32, True, "tc"),
                                          (33, True, "dequant"), (128, True, "dequant"), (8, False, "dequant")])
def test_matmul_dispatch_by_batch(B, tc_ok, want, monkeypatch):
    """DeviceMatrix.matmul routes by token count: the fused GEMV up to
    GEMV_MAX_BATCH, the tcgen05 kernel up to TENSOR_CORE_MAX_BATCH when the
    tile layout has one, else W decoded once for a dense GEMM."""
    from ecq_b200.device import DeviceMatrix

    m = object.__new__(DeviceMatrix)
    m.rows, m.cols = 16, 32
    called = []
    monkeypatch.setattr(DeviceMatrix, "tensor_core_ok", lambda self: tc_ok)
    monkeypatch.setattr(DeviceMatrix, "gemv",
                        lambda self, x, s: called.append("gemv") or x.new_empty(x.shape[0], 16))
    monkeypatch.setattr(DeviceMatrix, "matmul_tc",
                        lambda self, x, s: called.append("tc") or x.new_empty(x.shape[0], 16))
    monkeypatch.setattr(DeviceMatrix, "dequantize",
                        lambda self, s: called.append("dequant") or torch.empty(16, 32, dtype=torch.float16, device="meta"))
    y = m.matmul(torch.empty(B, 32, dtype=torch.float16, device="meta"), None)
    assert called == [want] and y.shape == (B, 16)
