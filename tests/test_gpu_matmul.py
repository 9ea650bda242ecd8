"""The tcgen05 batched path (ecq_matmul): rANS tiles decoded straight into
the tensor core's shared-memory operand, x in tensor memory, fp32
accumulation. Checked against the oracle's fp32 dequant + matmul
(max|y - y_ref| / max|y_ref| <= 2e-3), on shapes that exercise partial row
blocks, row blocks split across CTAs, both tile widths, several group
sizes, a constant table and batches above one launch's 128 tokens."""
import numpy as np
import pytest

from oracle import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402

RTOL = 2e-3


def _rel_err(y, y_ref):
    return float(np.max(np.abs(y - y_ref)) / max(np.max(np.abs(y_ref)), 1e-30))


def _run(rows, cols, tc, g, B, b=0.5, seed=0, sym=None):
    if sym is None:
        sym = syn.laplace_symbols(rows, cols, b=b, seed=seed)
    sc = syn.group_scales(rows, cols, g, seed=seed + 1)
    x = syn.activations(B, cols, seed=seed + 2)
    enc = ecq.encode_matrix(sym, tile_cols=tc, group_size=g)
    m = ecq.DeviceMatrix.from_encoded(enc, group_size=g)
    assert m.tensor_core_ok()
    y = m.matmul_tc(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))
    assert y.shape == (B, rows)
    err = _rel_err(y.float().cpu().numpy(), y_ref)
    assert err <= RTOL, err
    # the workspace (partial sums and row-block counters) is back at zero
    assert int(m.mm_workspace.count_nonzero()) == 0
    return m, x, sc


@pytest.mark.parametrize("rows,cols,tc,g,B", [
    (224, 256, 256, 128, 8),      # one row block, one K-tile
    (520, 2048, 256, 128, 3),     # partial last row block
    (520, 2048, 256, 64, 32),
    (300, 1024, 128, 128, 16),    # 8x128 tiles
    (100, 512, 128, 32, 5),
    (1000, 1024, 256, 256, 128),  # full token tile
    (96, 768, 256, 256, 130),     # two launches (128 + 2)
    (4104, 4096, 256, 128, 8),    # row blocks split across many CTAs
])
def test_matmul_tc_parity(rows, cols, tc, g, B):
    _run(rows, cols, tc, g, B, seed=rows + cols + B)


@pytest.mark.parametrize("b", [0.3, 2.0, 100.0])
def test_matmul_tc_entropies(b):
    _run(640, 2048, 256, 128, 24, b=b, seed=7)


def test_matmul_tc_constant_table():
    sym = np.full((232, 512), 5, dtype=np.uint8)
    _run(232, 512, 256, 128, 9, sym=sym)


def test_matmul_tc_repeatable_and_matches_row_gemv():
    m, x, sc = _run(1800, 2048, 256, 128, 12, seed=3)
    xt = torch.from_numpy(x).cuda()
    st = torch.from_numpy(sc).cuda()
    y1 = m.matmul_tc(xt, st)
    y2 = m.matmul_tc(xt, st)
    m.check()
    # row blocks are shared by up to 8 CTAs here; the fixed-point partial sums
    # make y independent of the order in which they finish
    assert torch.equal(y1, y2)
    yg = m.gemv(xt[:2].contiguous(), st)
    m.check()
    assert _rel_err(y1[:2].float().cpu().numpy(), yg.float().cpu().numpy()) <= RTOL


def test_matmul_dispatch_uses_tensor_cores():
    sym = syn.laplace_symbols(256, 1024, b=0.5, seed=5)
    sc = torch.from_numpy(syn.group_scales(256, 1024, 128)).cuda()
    m256 = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=256, group_size=128), group_size=128)
    m512 = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=512, group_size=128), group_size=128)
    assert m256.tensor_core_ok() and not m512.tensor_core_ok()
    x = torch.from_numpy(syn.activations(16, 1024)).cuda()
    ya = m256.matmul(x, sc)
    yb = m512.matmul(x, sc)  # 8x512 tiles: decode to fp16 + GEMM
    m256.check()
    m512.check()
    assert m256.mm_workspace is not None
    assert _rel_err(ya.float().cpu().numpy(), yb.float().cpu().numpy()) <= RTOL


def test_matmul_tc_70b_mlp_shape():
    """28672 x 8192 (8x256 tiles) at batches 8 and 128 against the decode-to-
    fp16 + cuBLAS path on the same device (both round W once to fp16)."""
    M, K = 28672, 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    p = torch.tensor(syn.laplace_probs(0.5), device="cuda", dtype=torch.float32)
    sym = torch.multinomial(p, M * K, replacement=True, generator=g).to(torch.uint8).reshape(M, K).cpu().numpy()
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=256, group_size=128), group_size=128)
    sc = torch.from_numpy(syn.group_scales(M, K, 128, seed=1)).cuda()
    w = m.dequantize(sc)
    m.check()
    for B in (8, 128):
        x = torch.randn(B, K, device="cuda", dtype=torch.float16, generator=g)
        y = m.matmul_tc(x, sc)
        m.check()
        y_ref = torch.mm(x.float(), w.float().t())
        err = float((y.float() - y_ref).abs().max() / y_ref.abs().max())
        assert err <= RTOL, (B, err)
