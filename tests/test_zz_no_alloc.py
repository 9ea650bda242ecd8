"""ecq_gemv_noalloc: the fused GEMV for callers that cannot allocate device
memory (a plugin whose host framework owns the device-memory budget, a C host
without a device allocator, a serving loop that must not call cudaMalloc).
Its workspace is a fixed array inside libecq; these tests call it through the
C ABI and compare it with ecq_gemv on a caller-allocated workspace.

The file name makes pytest collect it last."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import _lib  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402

RTOL = 2e-3  # same bound as the other GEMV parity tests: max|dy| / max|y|


def _rel_err(y, y_ref):
    y = y.float().cpu().numpy().astype(np.float64)
    y_ref = y_ref.float().cpu().numpy().astype(np.float64)
    return float(np.max(np.abs(y - y_ref)) / max(np.max(np.abs(y_ref)), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _noalloc(m, x, sc):
    y = torch.full((1, m.rows), float("nan"), dtype=torch.float16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().ecq_gemv_noalloc(m.view(), _lib.ptr(x), _lib.ptr(sc), _lib.ptr(y), 1, _lib.ptr(status),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.ERRORS.get(rc, rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return y


def _case(M, K, g, seed, tile_cols=None):
    sym = syn.laplace_symbols(M, K, b=0.5, seed=seed)
    sc = torch.from_numpy(syn.group_scales(M, K, g, seed=seed + 1)).cuda()
    x = torch.from_numpy(syn.activations(1, K, seed=seed + 2)).cuda()
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=tile_cols, group_size=g), group_size=g)
    y_ref = m.gemv(x, sc)  # ecq_gemv with the matrix's own workspace
    m.check()
    return m, x, sc, y_ref.reshape(1, M)


def test_noalloc_matches_gemv_on_two_calls():
    m, x, sc, y_ref = _case(2056, 4096, 128, 31)  # a short last row slab
    for _ in range(2):
        assert _rel_err(_noalloc(m, x, sc), y_ref) <= RTOL


def test_noalloc_large_then_small_then_large():
    # The slab counters follow the per-tile partial sums, so a smaller matrix's
    # counters fall inside the larger one's partial sums: each call must clear
    # them. 11008 x 4096 in 8x256 tiles (22016 tiles), then 520 x 1024 (130
    # tiles, a short last slab), then the large one again.
    big = _case(11008, 4096, 128, 41, tile_cols=256)
    small = _case(520, 1024, 128, 51)
    for m, x, sc, y_ref in (big, small, big, small):
        assert _rel_err(_noalloc(m, x, sc), y_ref) <= RTOL


def test_noalloc_rejects_matrices_beyond_its_scratch():
    # 4096 x 1048576 in 8x512 tiles needs ~32 MiB of workspace: rejected on the
    # host before anything is launched (the pointers are never dereferenced)
    v = _lib.MatrixView(rows=4096, cols=1 << 20, tile_rows=8, tile_cols=512, group_size=128,
                        n_tiles=512 * 2048, max_tile_bytes=1024, flags=0,
                        data=ctypes.c_void_p(16).value, tile_offset=ctypes.c_void_p(16).value,
                        stream_len=ctypes.c_void_p(16).value, dec_table=ctypes.c_void_p(16).value)
    assert _lib.lib().ecq_gemv_workspace_bytes(v, 1) > _lib.NOALLOC_SCRATCH_BYTES
    rc = _lib.lib().ecq_gemv_noalloc(v, 16, 16, 16, 1, 16, None)
    assert rc == -9  # ECQ_ERR_WORKSPACE
