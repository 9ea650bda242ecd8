"""GPU parity: libecq's kernels against the oracle and the reference golden
vectors. Symbols must be bit-exact; GEMV outputs within max relative error
2e-3 of the float64 oracle (fp16 output). All calls go through the C ABI."""
import numpy as np
import pytest

from conftest import GOLDEN, load_cases
from oracle import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402

RTOL = 2e-3  # max|y - y_ref| / max|y_ref|, the path's stated tolerance


def _rel_err(y, y_ref):
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    return float(np.max(np.abs(y - y_ref)) / max(np.max(np.abs(y_ref)), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def test_decode_reference_tiles_bit_exact():
    cases, _ = load_cases(GOLDEN / "codec.npz")
    dec = ecq.CudaInterleavedRANS()
    for c in cases:
        tile = ecq.InterleavedEncodedTile(data=bytes(c["data"]), stream_lengths=c["lengths"].tolist(),
                                          max_stream_len=int(c["max_len"]), n_symbols=int(c["symbols"].size),
                                          n_streams=int(c["S"]), table=ecq.RANSTable.from_freq(c["freq"]))
        out = dec.decode(tile)
        assert np.array_equal(out, c["symbols"]), str(c["name"])
        assert dec.last_status == 0, str(c["name"])


def test_decode_corrupt_tiles_like_reference():
    cases, z = load_cases(GOLDEN / "corrupt.npz", prefix="k")
    dec = ecq.CudaInterleavedRANS()
    for c in cases:
        tile = ecq.InterleavedEncodedTile(data=bytes(c["data"]), stream_lengths=c["lengths"].tolist(),
                                          max_stream_len=int(z["max_len"]), n_symbols=int(z["n_symbols"]),
                                          n_streams=32, table=ecq.RANSTable.from_freq(z["freq"]))
        out = dec.decode(tile)
        assert np.array_equal(out, c["out"]), str(c["name"])
        assert (dec.last_status == 0) == (str(c["name"]) == "intact")


def test_c1_single_matrix():
    z = np.load(GOLDEN / "c1.npz")
    tile = ecq.InterleavedEncodedTile(data=bytes(z["data"]), stream_lengths=z["lengths"].tolist(),
                                      max_stream_len=int(z["max_len"]), n_symbols=int(z["symbols"].size),
                                      n_streams=int(z["S"]), table=ecq.RANSTable.from_freq(z["freq"]))
    out = ecq.interleaved_rans_decode(tile)
    assert np.array_equal(out.reshape(z["symbols"].shape), z["symbols"])
    # the same matrix through the packed format and the fused GEMV
    enc = ecq.encode_matrix(z["symbols"], ecq.RANSTable.from_freq(z["freq"]), group_size=128)
    m = ecq.DeviceMatrix.from_encoded(enc, group_size=128)
    y = m.gemv(torch.from_numpy(z["x"]).cuda(), torch.from_numpy(z["scales"]).cuda())
    m.check()
    assert _rel_err(y.float().cpu().numpy(), z["y"]) <= RTOL


CASES = [
    # rows, cols, tile_cols, group, b
    (64, 512, 512, 128, 0.5),
    (36, 768, 256, 128, 0.5),
    (17, 384, 128, 64, 2.0),
    (128, 1024, 512, 32, 0.3),
    (40, 1024, 256, 256, 1.0),
    (96, 2048, 512, 512, 100.0),
    (8, 128, 128, 128, 0.5),
    (1, 512, 512, 128, 0.5),
    (300, 1536, 512, 64, 0.5),
]


@pytest.mark.parametrize("rows,cols,tc,g,b", CASES)
def test_packed_decode_and_gemv(rows, cols, tc, g, b):
    sym = syn.laplace_symbols(rows, cols, b=b, seed=rows + cols)
    sc = syn.group_scales(rows, cols, g, seed=1)
    x = syn.activations(1, cols, seed=2)
    enc = ecq.encode_matrix(sym, tile_cols=tc, group_size=g)
    m = ecq.DeviceMatrix.from_encoded(enc, group_size=g)
    out = m.decode()
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), sym)
    y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_gemv_deterministic_and_workspace_reusable():
    sym = syn.laplace_symbols(512, 4096, b=0.5, seed=3)
    sc = torch.from_numpy(syn.group_scales(512, 4096, 128)).cuda()
    x = torch.from_numpy(syn.activations(1, 4096)).cuda()
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    ys = [m.gemv(x, sc).clone() for _ in range(3)]
    m.check()
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    assert int(m.workspace[:(512 // 8) * 4].count_nonzero()) == 0  # slab counters (first) back at zero


def test_constant_matrix():
    # > 16384 copies of one symbol: the reference normaliser gives it all 16384 slots
    sym = np.full((40, 512), 11, dtype=np.uint8)
    t = ecq.RANSTable.from_symbols(sym)
    assert t.freq.max() == 16384
    sc = syn.group_scales(40, 512, 128)
    x = syn.activations(1, 512)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, t, group_size=128), group_size=128)
    assert np.array_equal(m.decode().cpu().numpy(), sym)
    y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_student_t_quantised_weights():
    w = syn.student_t_weights(256, 1024, seed=3)
    sym, sc = syn.quantize_symmetric_groups(w, 128)
    x = syn.activations(1, 1024)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_corrupt_packed_tile_sets_status():
    sym = syn.laplace_symbols(64, 512, b=0.5, seed=9)
    enc = ecq.encode_matrix(sym, group_size=128)
    enc.data[enc.tile_offset[3] + 40] ^= 0xFF  # damage one byte of tile 3
    m = ecq.DeviceMatrix.from_encoded(enc, group_size=128)
    m.decode()
    assert m.read_status() & 1


@pytest.mark.parametrize("M,K,tc,g,B", [
    (96, 1024, 512, 128, 4),      # one launch of 4 tokens
    (520, 2048, 512, 128, 8),     # 8 tokens, a short last row slab
    (264, 768, 256, 64, 3),       # 3 tokens in a 4-token launch (one zero token)
    (200, 1024, 128, 32, 5),      # 8-token launch, 8x128 tiles, group 32
    (512, 4096, 512, 256, 9),     # 8 + 1 (the last token on the single-token kernel)
    (1024, 11008, 256, 128, 16),  # x of 8 tokens does not fit next to 11008 columns: 4 launches of 4
    (64, 512, 512, 512, 2),       # group = tile width
])
def test_batched_gemv_decodes_each_tile_once(M, K, tc, g, B):
    """Token batches share one decode of each tile (up to 8 tokens per
    launch); every token's y against the float64 oracle, and bit-identical
    replays."""
    sym = syn.laplace_symbols(M, K, b=0.5, seed=M + B)
    sc = syn.group_scales(M, K, g, seed=K)
    x = syn.activations(B, K, seed=B)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=tc, group_size=g), group_size=g)
    xs, ss = torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda()
    y = m.gemv(xs, ss).clone()
    y2 = m.gemv(xs, ss)
    m.check()
    assert torch.equal(y, y2)
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))
    assert y.shape == (B, M) and _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_batched_gemv_student_t_constant_and_small_workspace():
    # Student-t weights (wide symbol spread), a constant matrix, and a caller
    # workspace sized for one token (the batch then runs token by token)
    w = syn.student_t_weights(300, 2048, seed=3).astype(np.float32)
    sym, sc = syn.quantize_symmetric_groups(w, 128)
    x = syn.activations(6, 2048, seed=4)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL
    from ecq_b200 import _lib

    m1 = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    y1 = torch.empty(6, 300, dtype=torch.float16, device="cuda")
    ws1 = torch.zeros(int(_lib.lib().ecq_gemv_workspace_bytes(m1.view(), 1)), dtype=torch.uint8, device="cuda")
    xs = torch.from_numpy(x).cuda()
    ss = torch.from_numpy(sc).cuda()
    rc = _lib.lib().ecq_gemv(m1.view(), _lib.ptr(xs), _lib.ptr(ss), _lib.ptr(y1), 6, _lib.ptr(ws1), ws1.numel(),
                             _lib.ptr(m1.status), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    m1.check()
    assert _rel_err(y1.float().cpu().numpy(), y_ref) <= RTOL
    const = np.full((40, 512), 5, dtype=np.uint8)
    mc = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(const, group_size=128), group_size=128)
    sc_c = syn.group_scales(40, 512, 128, seed=6)
    xc = syn.activations(4, 512, seed=7)
    yc = mc.gemv(torch.from_numpy(xc).cuda(), torch.from_numpy(sc_c).cuda())
    mc.check()
    assert _rel_err(yc.float().cpu().numpy(), oracle.dequant_gemv(const, sc_c.astype(np.float32), 128,
                                                                   xc.astype(np.float32))) <= RTOL


@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008)])
def test_llama_shapes_full_size(M, K):
    """Full-size layer shapes: decode(encode(W)) == W and the fused GEMV
    against the float64 oracle."""
    sym = syn.laplace_symbols(M, K, b=0.5, seed=0)
    sc = syn.group_scales(M, K, 128, seed=1)
    x = syn.activations(1, K, seed=2)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    out = m.decode()
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), sym)
    y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.astype(np.float32))
    assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL


def test_dequantize_and_batched_matmul():
    M, K, g = 520, 2048, 128
    sym = syn.laplace_symbols(M, K, b=0.5, seed=12)
    sc = syn.group_scales(M, K, g, seed=13)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=g), group_size=g)
    s = torch.from_numpy(sc).cuda()
    w = m.dequantize(s)
    m.check()
    w_ref = ((sym.astype(np.float32) - 8.0) * np.repeat(sc.astype(np.float32), g, axis=1)).astype(np.float16)
    assert np.array_equal(w.cpu().numpy(), w_ref)
    for B in (1, 2, 3, 8, 32):
        x = syn.activations(B, K, seed=14 + B)
        y = m.matmul(torch.from_numpy(x).cuda(), s)
        m.check()
        y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))
        assert y.shape == (B, M) and _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL, B


@pytest.mark.parametrize("b", [0.3, 0.5, 1.0, 2.0, 100.0])
def test_entropy_sweep_8192(b):
    """The 8192x8192 entropy-sweep matrices (Laplace b from 0.3 to near-uniform):
    decode(encode(W)) == W and the fused GEMV at group 64 and 128 against the
    oracle's fp32 dequant + matvec."""
    M = K = 8192
    g = torch.Generator(device="cuda").manual_seed(int(b * 10))
    p = torch.tensor(syn.laplace_probs(b), device="cuda", dtype=torch.float32)
    sym = torch.multinomial(p, M * K, replacement=True, generator=g).to(torch.uint8).reshape(M, K).cpu().numpy()
    x = syn.activations(1, K, seed=2)
    for gs in (64, 128):
        enc = ecq.encode_matrix(sym, group_size=gs)
        m = ecq.DeviceMatrix.from_encoded(enc, group_size=gs)
        if gs == 64:
            out = m.decode()
            torch.cuda.synchronize()
            assert np.array_equal(out.cpu().numpy(), sym)
            del out
        sc = syn.group_scales(M, K, gs, seed=1)
        y = m.gemv(torch.from_numpy(x).cuda(), torch.from_numpy(sc).cuda())
        m.check()
        y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), gs, x.astype(np.float32))
        assert _rel_err(y.float().cpu().numpy(), y_ref) <= RTOL, gs


def test_gemv_with_unaligned_x():
    """x that does not start on a 16-byte boundary cannot be bulk-copied into
    shared memory: the kernel then reads it from global memory. Same result."""
    M, K = 136, 1024
    sym = syn.laplace_symbols(M, K, b=0.5, seed=21)
    sc = torch.from_numpy(syn.group_scales(M, K, 128, seed=22)).cuda()
    x = syn.activations(1, K, seed=23)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=128), group_size=128)
    buf = torch.zeros(K + 8, dtype=torch.float16, device="cuda")
    buf[1:K + 1] = torch.from_numpy(x[0]).cuda()
    xu = buf[1:K + 1].view(1, K)  # 2 bytes past an aligned address
    assert xu.data_ptr() % 16 != 0
    y_u = m.gemv(xu, sc)
    y_a = m.gemv(torch.from_numpy(x).cuda(), sc)
    m.check()
    assert torch.equal(y_u, y_a)
    y_ref = oracle.dequant_gemv(sym, sc.float().cpu().numpy(), 128, x.astype(np.float32))
    assert _rel_err(y_u.float().cpu().numpy(), y_ref) <= RTOL
