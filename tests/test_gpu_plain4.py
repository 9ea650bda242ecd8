"""The plain 4-bit path: decoding a packed rANS matrix once to packed nibbles
(the CACHED strategy's 4-bit store, src/decode_strategies.py:43-73) and the
plain 4-bit GEMV that consumes it (also the bench's HBM-bound control beside
the fused rANS GEMV). Packed bytes must be bit-exact; GEMV outputs within max
relative error 2e-3 of the float64 oracle's dequant + matvec (fp16 out)."""
import numpy as np
import pytest

from oracle import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import _lib  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402
from ecq_b200.device import Packed4Matrix  # noqa: E402

RTOL = 2e-3  # max|y - y_ref| / max|y_ref|, the path's stated tolerance


def _rel_err(y, y_ref):
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    return float(np.max(np.abs(y - y_ref)) / max(np.max(np.abs(y_ref)), 1e-30))


def _pack(sym):
    return (sym[:, 0::2] & 15) | ((sym[:, 1::2] & 15) << 4)


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


@pytest.mark.parametrize("M,K,tc,b", [(1024, 1024, 512, 0.5), (520, 1024, 512, 0.5), (264, 768, 256, 1.0),
                                      (40, 256, 128, 100.0), (4096, 11008, 256, 0.5), (11008, 4096, 512, 0.5)])
def test_decode_packed4_bit_exact(M, K, tc, b):
    sym = syn.laplace_symbols(M, K, b=b, seed=M + K)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=tc, group_size=128), group_size=128)
    q = m.decode_packed4()
    torch.cuda.synchronize()
    m.check()
    assert np.array_equal(q.cpu().numpy(), _pack(sym))


def test_decode_packed4_constant_matrix():
    sym = np.full((24, 512), 11, dtype=np.uint8)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    q = m.decode_packed4()
    torch.cuda.synchronize()
    m.check()
    assert np.array_equal(q.cpu().numpy(), _pack(sym))


@pytest.mark.parametrize("M,K,g,B", [(4096, 4096, 128, 1), (11008, 4096, 128, 1), (4096, 11008, 128, 1),
                                     (13, 64, 32, 1), (1000, 2048, 64, 1), (300, 1536, 256, 3),
                                     (777, 4096, 128, 2), (512, 11008, 128, 4), (96, 1024, 512, 9)])
def test_plain4_gemv_matches_oracle(M, K, g, B):
    sym = syn.laplace_symbols(M, K, b=0.5, seed=3 * M + K)
    sc = syn.group_scales(M, K, g, seed=M)
    x = syn.activations(B, K, seed=K)
    p = Packed4Matrix.from_symbols(sym, group_size=g)
    y = p.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    torch.cuda.synchronize()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_plain4_gemv_student_t_weights_and_determinism():
    w = syn.student_t_weights(2048, 4096, seed=9).astype(np.float32)
    sym, sc = syn.quantize_symmetric_groups(w, 128)
    x = torch.from_numpy(syn.activations(1, 4096, seed=10)).cuda()
    p = Packed4Matrix.from_symbols(sym, 128)
    s = torch.from_numpy(sc).cuda()
    y1 = p.gemv(x, s).clone()
    y2 = p.gemv(x, s)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.float().cpu().numpy())
    assert _rel_err(y1.float().cpu().numpy(), y_ref) <= RTOL


def test_cached_packed_gemv_matches_fused_gemv():
    M, K = 2056, 4096
    sym = syn.laplace_symbols(M, K, b=0.5, seed=77)
    sc = torch.from_numpy(syn.group_scales(M, K, 128, seed=78)).cuda()
    x = torch.from_numpy(syn.activations(1, K, seed=79)).cuda()
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    p = Packed4Matrix.from_matrix(m)  # decode once, then plain GEMV
    y_p = p.gemv(x, sc)
    y_f = m.gemv(x, sc)
    torch.cuda.synchronize()
    m.check()
    assert p.nbytes == M * K // 2
    y_ref = oracle.dequant_gemv(sym, sc.float().cpu().numpy(), 128, x.float().cpu().numpy())
    assert _rel_err(y_p.float().cpu().numpy(), y_ref) <= RTOL
    assert _rel_err(y_f.float().cpu().numpy(), y_ref) <= RTOL


@pytest.mark.parametrize("B", [1, 3, 16])
def test_entropy_coded_linear_cached_is_4bit(B):
    torch.manual_seed(1)
    lin = torch.nn.Linear(2048, 520, bias=False).cuda()
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    ecl = ecq.EntropyCodedLinear.from_linear(lin, decode_mode="cached", group_size=128)
    assert ecl._packed.nbytes == 520 * 2048 // 2
    x = torch.randn(B, 2048, device="cuda", dtype=torch.float16)
    y = ecl(x)
    torch.cuda.synchronize()
    sym, sc = syn.quantize_symmetric_groups(lin.weight.detach().float().cpu().numpy(), 128)
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.float().cpu().numpy())
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_plain4_gemv_argument_errors():
    L = _lib.lib()
    q = torch.zeros(64, 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, 128, dtype=torch.float16, device="cuda")
    s = torch.zeros(64, 2, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 64, dtype=torch.float16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    P = _lib.ptr
    assert L.ecq_plain4_gemv(P(q), P(s), P(x), P(y), 64, 128, 96, 1, st) == -8  # group not a power of two
    assert L.ecq_plain4_gemv(P(q), P(s), P(x), P(y), 64, 120, 64, 1, st) == -8  # cols % 32
    assert L.ecq_plain4_gemv(P(q) + 8, P(s), P(x), P(y), 64, 128, 64, 1, st) == -1  # unaligned q
    assert L.ecq_plain4_gemv(P(q), P(s), P(x), P(y), 64, 128, 64, 0, st) == -1  # empty batch
    assert L.ecq_plain4_gemv(P(q), P(s), P(x), P(y), 64, 128, 64, 1, st) == 0
    torch.cuda.synchronize()
