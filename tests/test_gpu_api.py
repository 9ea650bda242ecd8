"""The PyTorch-facing API (custom op, entropy_coded_matmul, EntropyCodedLinear)
and the SmartDecoder strategies, on the GPU, against the oracle."""
import numpy as np
import pytest

from oracle import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402
from ecq_b200 import ops, strategies  # noqa: E402

RTOL = 2e-3


def _rel(y, y_ref):
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    return float(np.max(np.abs(y - y_ref)) / max(np.max(np.abs(y_ref)), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def mat():
    M, K, g = 520, 1024, 64
    sym = syn.laplace_symbols(M, K, b=0.5, seed=41)
    sc = syn.group_scales(M, K, g, seed=42)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, group_size=g), group_size=g)
    return sym, sc, m


def test_custom_op_matches_device_gemv(mat):
    sym, sc, m = mat
    x = torch.from_numpy(syn.activations(3, m.cols, seed=43)).cuda()
    s = torch.from_numpy(sc).cuda()
    y = ecq.rans_gemv(x, m, s)
    m.check()
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 64, x.float().cpu().numpy())
    assert y.shape == (3, m.rows) and _rel(y.float().cpu().numpy(), y_ref) <= RTOL
    assert torch.equal(y, m.gemv(x, s))


def test_custom_op_in_cuda_graph(mat):
    sym, sc, m = mat
    x = torch.from_numpy(syn.activations(1, m.cols, seed=44)).cuda()
    s = torch.from_numpy(sc).cuda()
    y0 = ecq.rans_gemv(x, m, s).clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = ecq.rans_gemv(x, m, s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    m.check()
    assert torch.equal(y, y0)


def test_entropy_coded_matmul_with_affine_biases(mat):
    sym, sc, m = mat
    x = torch.from_numpy(syn.activations(2, m.cols, seed=45)).cuda()
    s = torch.from_numpy(sc).cuda()
    rng = np.random.default_rng(46)
    biases = (rng.uniform(-0.2, 0.0, sc.shape)).astype(np.float16)
    y = ecq.entropy_coded_matmul(x, m, freq_table=m.table.freq, scales=s, biases=torch.from_numpy(biases).cuda(),
                                 group_size=64)
    w = sym.astype(np.float64) * np.repeat(sc.astype(np.float64), 64, 1) + np.repeat(biases.astype(np.float64), 64, 1)
    y_ref = x.double().cpu().numpy() @ w.T
    assert _rel(y.float().cpu().numpy(), y_ref) <= RTOL
    # without biases: the symmetric zero point 8
    y8 = ecq.entropy_coded_matmul(x, m, scales=s, group_size=64)
    assert _rel(y8.float().cpu().numpy(), oracle.dequant_gemv(sym, sc.astype(np.float32), 64,
                                                               x.float().cpu().numpy())) <= RTOL
    with pytest.raises(ValueError):
        ecq.entropy_coded_matmul(x, m, freq_table=np.ones(16, np.uint32) * 1024, scales=s, group_size=64)


@pytest.mark.parametrize("mode", ["fused", "cached"])
def test_entropy_coded_linear(mode):
    torch.manual_seed(0)
    lin = torch.nn.Linear(1024, 384, bias=True).cuda()
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    ecl = ecq.EntropyCodedLinear.from_linear(lin, decode_mode=mode, group_size=128)
    x = torch.randn(4, 1024, device="cuda", dtype=torch.float16)
    y = ecl(x)
    ecl.matrix.check()
    sym, sc = syn.quantize_symmetric_groups(lin.weight.detach().float().cpu().numpy(), 128)
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.float().cpu().numpy()) + \
        lin.bias.detach().float().cpu().numpy()
    assert _rel(y.float().cpu().numpy(), y_ref) <= RTOL
    assert 1.0 < ecl.compression_ratio and ecl.bits_per_weight < 4.0


def test_smart_decoder_modes(mat):
    sym, sc, m = mat
    tile = ecq.interleaved_rans_encode(sym[:64].reshape(-1), m.table, 8)
    shape = (64, m.cols)
    assert strategies.SmartDecoder("fused").get_weights("l0") is None

    d = strategies.SmartDecoder("cached")
    d.load_layer("l0", tile, 0.02, -0.16, shape)
    d.load_layer("m", m, 0.02, -0.16, (m.rows, m.cols))
    assert np.array_equal(d.get_weights("l0").numpy(), sym[:64])
    assert np.array_equal(d.get_weights("m").numpy(), sym)
    assert d.memory_usage() == sym[:64].size + sym.size // 2  # the packed matrix is cached as 4-bit
    assert d.get_weights("m").packed is not None

    d = strategies.SmartDecoder("lru", max_memory_bytes=sym.size + 10)
    assert np.array_equal(d.get_weights("m", m, 1.0, 0.0, (m.rows, m.cols)).numpy(), sym)
    d.get_weights("m", m, 1.0, 0.0, (m.rows, m.cols))
    d.get_weights("l0", tile, 1.0, 0.0, shape)  # evicts "m"
    assert d.stats["hits"] == 1 and d.stats["misses"] == 2 and "m" not in d.cache

    for mode in ("prefetch", "gpu_async"):
        d = strategies.SmartDecoder(mode)
        d.prefetch_layer("l0", tile, 0.02, -0.16, shape)
        d.prefetch_layer("m", m, 0.02, -0.16, (m.rows, m.cols))
        w = d.get_weights("m")
        torch.cuda.synchronize()
        assert d.is_ready("l0")
        assert np.array_equal(w.numpy(), sym)
        assert np.array_equal(d.get_weights("l0").numpy(), sym[:64])
        with pytest.raises(KeyError):
            d.get_weights("absent")
    dq = strategies.DecodedWeights(torch.from_numpy(sym[:2]).cuda(), 0.5, -4.0, (2, m.cols)).dequantize()
    assert torch.allclose(dq.cpu(), torch.from_numpy(sym[:2].astype(np.float32) * 0.5 - 4.0))


def test_containers_on_gpu(tmp_path):
    from conftest import GOLDEN
    from ecq_b200 import container

    z = np.load(GOLDEN / "v1.npz")
    ref = container.read_ecq_v1(GOLDEN / "v1_two_tensors.ecq", layout="reference")
    assert np.array_equal(container.decompress_v1_tensor(ref["a"]), z["a_reference"])
    aw = container.read_ecq_v1(GOLDEN / "v1_two_tensors.ecq", layout="as_written")
    for name in ("a", "b"):
        assert np.allclose(container.decompress_v1_tensor(aw[name]), z[f"{name}_dequant"], atol=1e-7)
    # v2: write, memory-map, load to the device, fused GEMV
    w = syn.student_t_weights(264, 1024, seed=8).astype(np.float32)
    container.save_ecq2(tmp_path / "m.ecq", {"w": container.compress_weights(w, 128)})
    t = container.load_ecq2(tmp_path / "m.ecq")["w"]
    m, s = t.to_device()
    x = syn.activations(1, 1024, seed=9)
    y = m.gemv(torch.from_numpy(x).cuda(), s)
    m.check()
    sym, sc = syn.quantize_symmetric_groups(w, 128)
    assert _rel(y.float().cpu().numpy(), oracle.dequant_gemv(sym, sc.astype(np.float32), 128,
                                                             x.astype(np.float32))) <= RTOL


def test_rans_matmul_op_tensor_cores_and_graph():
    """ecq::rans_matmul (tcgen05 path, 8x256 tiles) against the oracle, then
    captured in a CUDA graph: replays give the same bits (fixed-point sums)."""
    M, K, g = 456, 2048, 128
    sym = syn.laplace_symbols(M, K, b=0.5, seed=51)
    sc = syn.group_scales(M, K, g, seed=52)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=256, group_size=g), group_size=g)
    assert m.tensor_core_ok()
    x = torch.from_numpy(syn.activations(12, K, seed=53)).cuda()
    s = torch.from_numpy(sc).cuda()
    y0 = ecq.rans_matmul(x, m, s).clone()
    m.check()
    assert _rel(y0.float().cpu().numpy(), oracle.dequant_gemv(sym, sc.astype(np.float32), g,
                                                              x.float().cpu().numpy())) <= RTOL
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        y = ecq.rans_matmul(x, m, s)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    m.check()
    assert torch.equal(y, y0)


def test_entropy_coded_linear_batched_tensor_cores():
    torch.manual_seed(1)
    lin = torch.nn.Linear(2048, 520, bias=False).cuda()
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    ecl = ecq.EntropyCodedLinear.from_linear(lin, group_size=128, tile_cols=256)
    assert ecl.matrix.tensor_core_ok()
    x = torch.randn(2, 7, 2048, device="cuda", dtype=torch.float16)
    y = ecl(x)
    ecl.matrix.check()
    assert ecl.matrix.mm_workspace is not None  # the batched call ran on the tensor cores
    sym, sc = syn.quantize_symmetric_groups(lin.weight.detach().float().cpu().numpy(), 128)
    y_ref = oracle.dequant_gemv(sym, sc.astype(np.float32), 128, x.reshape(14, 2048).float().cpu().numpy())
    assert y.shape == (2, 7, 520) and _rel(y.reshape(14, 520).float().cpu().numpy(), y_ref) <= RTOL
