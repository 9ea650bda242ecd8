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
